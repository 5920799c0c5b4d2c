"""CPU tests of the multi-rank (sequence-sharded) path with gloo, world_size 2.

bench.py --gpus N shards sequences across ranks: every rank owns its own
sequences, pool and allocator, and the only collectives are the barrier and
the max-over-ranks timing reduction.  Here two gloo ranks each drive a
bookkeeping-only cache through the bench's own fill plan and decode cycle,
check it bit-exact against an oracle instance of their own shard, and reduce
their step times with bench.reduce_max.
"""
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, out_dir):
    import sys

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import datetime

    import torch.distributed as dist

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    import bench
    from langtrain_studio_b200.kv import KvCache
    from oracle import oracle

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    seed = bench.shard_seed(rank)
    lens = bench.workload(seed)[:16] // 8  # a small shard of the workload
    n_blocks = int(((lens + bench.CYCLE + 1 + 15) // 16).sum()) + 16
    kv = KvCache(1, 8, 128, n_blocks * 16, n_heads=32, max_seqs=16, max_batch=8192, device=-1)
    ok = oracle.OracleKv(1, 8 * 128, n_blocks * 16, max_seqs=16)
    seqs, pos = bench.fill_plan(lens, seed)
    b, s = kv.append_batch(seqs, pos)
    rc, done, bo, so = ok.append_batch(seqs, pos)
    assert rc == 0 and np.array_equal(b, bo) and np.array_equal(s, so)
    # one full decode cycle of the bench (append, then kv_remove back)
    for phase in range(bench.CYCLE):
        p = (lens + phase).astype(np.uint32)
        b, s = kv.append_batch(np.arange(16), p)
        rc, _, bo, so = ok.append_batch(np.arange(16), p)
        assert rc == 0 and np.array_equal(b, bo) and np.array_equal(s, so)
    for i in range(16):
        kv.truncate(i, int(lens[i]))
        ok.truncate(i, int(lens[i]))
    for i in range(16):
        assert np.array_equal(kv.seq_blocks(i), ok.seq_blocks(i))
    assert np.array_equal(kv.free_list(), ok.free_list())
    local_ms = 1.0 + rank * 0.5
    ms_max = bench.reduce_max(local_ms, "cpu", world)
    dist.barrier()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(f"{ms_max} {int(lens.sum())} {seed}\n")
    dist.destroy_process_group()


def test_two_rank_sequence_sharding(tmp_path):
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    rows = [open(tmp_path / f"rank{r}.txt").read().split() for r in range(world)]
    assert all(float(r[0]) == 1.5 for r in rows)  # max over ranks seen by every rank
    assert rows[0][2] != rows[1][2]  # disjoint shards: each rank has its own sequences

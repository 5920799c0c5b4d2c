"""KV-head sharding across 2 GPUs: each rank holds half the KV heads of every
sequence (identical bookkeeping calls on both ranks), attends with its own
q heads, and lt_kv_gather_heads (NCCL all-gather + permute) must reproduce
the unsharded attention of the oracle within the north-star tolerance.  The
gather fused into attention (lt_kv_*_gather) is checked the same way on 2
GPUs, and its set-up rules on one GPU (nranks = 1)."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, out_dir):
    import datetime
    import sys

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from langtrain_studio_b200 import kv as kvm
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(rank)
    hkv, hq, d = 4, 16, 128
    hl, ql = hkv // world, hq // world
    lens = [100, 333, 1000, 17]
    rng = np.random.default_rng(0)  # the same full K/V and q on every rank
    K = [rng.standard_normal((L, hkv * d)).astype(np.float32) for L in lens]
    V = [rng.standard_normal((L, hkv * d)).astype(np.float32) for L in lens]
    q = rng.standard_normal((len(lens), hq * d)).astype(np.float32)
    nb = sum((L + 16) // 16 for L in lens) + 8
    kv = kvm.KvCache(1, hl, d, nb * 16, n_heads=ql, max_seqs=len(lens), max_batch=4096, device=rank)
    cols = slice(rank * hl * d, (rank + 1) * hl * d)
    for s, L in enumerate(lens):
        b, sl = kv.append_batch(np.full(L, s), np.arange(L))
        kv.write(0, b, sl, torch.from_numpy(np.ascontiguousarray(K[s][:, cols])).cuda(),
                 torch.from_numpy(np.ascontiguousarray(V[s][:, cols])).cuda())
    qcols = slice(rank * ql * d, (rank + 1) * ql * d)
    local = kv.attend(0, torch.from_numpy(np.ascontiguousarray(q[:, qcols])).cuda(), np.arange(len(lens)),
                      np.array(lens) - 1, out_dtype=torch.float32)
    uid = [kvm.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = kvm.NcclComm(world, uid[0], rank, rank)
    full = kvm.gather_heads(kv, local, comm).cpu().numpy()
    ok = oracle.OracleKv(1, hkv * d, nb * 16, max_seqs=len(lens))
    for s, L in enumerate(lens):
        rc, _, b, sl = ok.append_batch(np.full(L, s), np.arange(L))
        ok.write_batch(0, b, sl, K[s], V[s])
    ref = ok.attend(0, q, np.arange(len(lens)), np.array(lens) - 1, hq, hkv, d)
    err = float(np.abs(full - ref).max())
    np.save(os.path.join(out_dir, f"err{rank}.npy"), np.array([err]))
    comm.close()
    kv.close()
    dist.destroy_process_group()


def test_head_sharded_attention_matches_unsharded(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_rank, args=(2, _port(), str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        err = float(np.load(tmp_path / f"err{r}.npy")[0])
        assert err < 2e-5, err  # f32 outputs; the north-star bar is 2e-3


# ---- the gather fused into attention: NVLink peer stores, no collective ----

def _peer_rank(rank, world, port, out_dir, skip_rank):
    import datetime
    import sys

    import torch
    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200 import kv as kvm
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(rank)
    hkv, hq, d = 4, 16, 128
    hl, ql = hkv // world, hq // world
    lens = [100, 333, 1000, 17]
    n = len(lens)
    rng = np.random.default_rng(0)  # the same full K/V and q on every rank
    K = [rng.standard_normal((L, hkv * d)).astype(np.float32) for L in lens]
    V = [rng.standard_normal((L, hkv * d)).astype(np.float32) for L in lens]
    steps = 3
    q = rng.standard_normal((steps + 2, n, hq * d)).astype(np.float32)
    Kn = rng.standard_normal((steps, n, hkv * d)).astype(np.float32)
    Vn = rng.standard_normal((steps, n, hkv * d)).astype(np.float32)
    nb = sum((L + steps + 16) // 16 for L in lens) + 8
    kv = kvm.KvCache(1, hl, d, nb * 16, n_heads=ql, max_seqs=n, max_batch=4096, device=rank)
    ok = oracle.OracleKv(1, hkv * d, nb * 16, max_seqs=n)
    cols = slice(rank * hl * d, (rank + 1) * hl * d)
    qcols = slice(rank * ql * d, (rank + 1) * ql * d)
    for s, L in enumerate(lens):
        b, sl = kv.append_batch(np.full(L, s), np.arange(L))
        kv.write(0, b, sl, torch.from_numpy(np.ascontiguousarray(K[s][:, cols])).cuda(),
                 torch.from_numpy(np.ascontiguousarray(V[s][:, cols])).cuda())
        rc, _, bo, so = ok.append_batch(np.full(L, s), np.arange(L))
        ok.write_batch(0, bo, so, K[s], V[s])
    kvm.setup_peer_gather(kv, rank, world, max_tokens=16)
    seqs = np.arange(n)
    errs = []

    def local_q(i):
        return torch.from_numpy(np.ascontiguousarray(q[i][:, qcols])).cuda()

    if skip_rank is None:
        # attend only: f32 out, then f16 out (the other half of the gather buffer)
        pos = np.array(lens) - 1
        ref = ok.attend(0, q[0], seqs, pos, hq, hkv, d)
        full = kv.attend_gather(0, local_q(0), seqs, pos, out_dtype=torch.float32)
        kv.check()
        errs.append(float(np.abs(full.cpu().numpy() - ref).max()))
        ref = ok.attend(0, q[1], seqs, pos, hq, hkv, d)
        full = kv.attend_gather(0, local_q(1).half(), seqs, pos, out_dtype=torch.float16)
        kv.check()
        np.testing.assert_allclose(full.float().cpu().numpy(), ref, rtol=1e-3, atol=2e-3)
        # decode steps: append + fused K/V write + attention + gather, one call each
        for t in range(steps):
            pos = np.array(lens) + t
            b, sl = kv.append_batch(seqs, pos)
            rc, _, bo, so = ok.append_batch(seqs, pos)
            full = kv.write_attend_gather(0, b, sl, torch.from_numpy(np.ascontiguousarray(Kn[t][:, cols])).cuda(),
                                          torch.from_numpy(np.ascontiguousarray(Vn[t][:, cols])).cuda(),
                                          local_q(t + 2), seqs, pos, out_dtype=torch.float32)
            kv.check()
            ok.write_batch(0, bo, so, Kn[t], Vn[t])
            ref = ok.attend(0, q[t + 2], seqs, pos, hq, hkv, d)
            errs.append(float(np.abs(full.cpu().numpy() - ref).max()))
        np.save(os.path.join(out_dir, f"err{rank}.npy"), np.array(errs))
    else:
        # One rank misses a call: the others' bounded wait runs out and the
        # handle reports LT_E_TIMEOUT; nothing hangs.  The missing rank stays
        # alive (its buffer mapped) until they are done.
        pos = np.array(lens) - 1
        status = "skipped"
        if rank != skip_rank:
            kv.attend_gather(0, local_q(0), seqs, pos, out_dtype=torch.float32)
            try:
                kv.check()
                status = "no error"
            except kvm.KvError as e:
                status = "timeout" if e.code == N.LT_E_TIMEOUT else f"code {e.code}"
        np.save(os.path.join(out_dir, f"status{rank}.npy"), np.array([status]))
    torch.cuda.synchronize()
    kv.peer_close()
    dist.barrier()
    kv.close()
    dist.destroy_process_group()


def test_peer_gather_matches_unsharded(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_peer_rank, args=(2, _port(), str(tmp_path), None), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        errs = np.load(tmp_path / f"err{r}.npy")
        assert errs.size == 4 and float(errs.max()) < 2e-5, errs  # f32 outputs


def test_peer_gather_rank_missing_a_call_times_out(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_peer_rank, args=(2, _port(), str(tmp_path), 1), nprocs=2, join=True, start_method="spawn")
    assert str(np.load(tmp_path / "status0.npy")[0]) == "timeout"
    assert str(np.load(tmp_path / "status1.npy")[0]) == "skipped"


def test_peer_gather_single_rank_and_reimport():
    """One rank (nranks = 1): the fused gather returns attend()'s rows through
    its own buffer and flag, on both halves.  A second import of the same
    buffers is refused (their flags hold the epochs of the calls made so far);
    close + a new export + import make the gather usable again."""
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200 import kv as kvm

    hkv, hq, d = 2, 8, 128
    lens = [40, 300, 17]
    n = len(lens)
    g = torch.Generator(device="cuda").manual_seed(3)
    nb = sum((L + 15) // 16 for L in lens) + 4
    kv = kvm.KvCache(1, hkv, d, nb * 16, n_heads=hq, max_seqs=n, max_batch=512, device=0)
    try:
        for s, L in enumerate(lens):
            b, sl = kv.append_batch(np.full(L, s), np.arange(L))
            kv.write(0, b, sl, torch.randn(L, hkv * d, device="cuda", generator=g),
                     torch.randn(L, hkv * d, device="cuda", generator=g))
        seqs, pos = np.arange(n), np.array(lens) - 1
        q = torch.randn(n, hq * d, device="cuda", generator=g)
        ref = kv.attend(0, q, seqs, pos, out_dtype=torch.float32)
        h = kv.peer_export(0, 1, max_tokens=8)
        kv.peer_import([h])
        for _ in range(3):  # halves 1, 0, 1
            out = kv.attend_gather(0, q, seqs, pos, out_dtype=torch.float32)
            kv.check()
            torch.testing.assert_close(out, ref, rtol=0, atol=1e-6)
        with pytest.raises(kvm.KvError) as e:
            kv.peer_import([h])
        assert e.value.code == N.LT_E_ARG
        kv.peer_close()
        h = kv.peer_export(0, 1, max_tokens=8)
        kv.peer_import([h])
        out = kv.attend_gather(0, q, seqs, pos, out_dtype=torch.float32)
        kv.check()
        torch.testing.assert_close(out, ref, rtol=0, atol=1e-6)
        kv.peer_close()
    finally:
        kv.close()


# ---- the sharded data path on one GPU: every rank's handle in one process ----

@pytest.mark.parametrize("world,hkv,hq", [(2, 4, 16), (8, 8, 64)])
def test_head_shards_on_one_gpu_match_unsharded(world, hkv, hq):
    """The KV-head-sharded mode without its collective: `world` handles, each
    holding KV heads [r*hl, (r+1)*hl) of every sequence, all on cuda:0, get
    the same bookkeeping calls (replicated tables), a prefill, then three
    fused append + attention decode steps.  Every rank's block tables and free
    list equal rank 0's, and the rank outputs laid side by side in rank order
    (the gathered layout, [token][rank][local q heads][D]) match the
    unsharded oracle within the f32 bar.  (8, 8, 64) is config 4's 70B
    attention shape at its 8-GPU sharding: one KV head and 8 q heads a rank."""
    from langtrain_studio_b200 import kv as kvm
    from oracle import oracle

    d = 128
    hl, ql = hkv // world, hq // world
    lens = [100, 333, 1000, 17, 2049]
    n, steps = len(lens), 3
    rng = np.random.default_rng(world)
    K = [rng.standard_normal((L, hkv * d)).astype(np.float32) for L in lens]
    V = [rng.standard_normal((L, hkv * d)).astype(np.float32) for L in lens]
    nb = sum((L + steps + 16) // 16 for L in lens) + 8
    kvs = [kvm.KvCache(1, hl, d, nb * 16, n_heads=ql, max_seqs=n, max_batch=4096, device=0) for _ in range(world)]
    ok = oracle.OracleKv(1, hkv * d, nb * 16, max_seqs=n)
    col = lambda r, h: slice(r * h * d, (r + 1) * h * d)  # noqa: E731
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    for s, L in enumerate(lens):
        for r, kv in enumerate(kvs):
            b, sl = kv.append_batch(np.full(L, s), np.arange(L))
            kv.write(0, b, sl, dev(K[s][:, col(r, hl)]), dev(V[s][:, col(r, hl)]))
        rc, _, b, sl = ok.append_batch(np.full(L, s), np.arange(L))
        assert rc == 0
        ok.write_batch(0, b, sl, K[s], V[s])
    seqs = np.arange(n)
    for step in range(steps):
        pos = np.array(lens) + step
        kn = rng.standard_normal((n, hkv * d)).astype(np.float32)
        vn = rng.standard_normal((n, hkv * d)).astype(np.float32)
        q = rng.standard_normal((n, hq * d)).astype(np.float32)
        outs = []
        for r, kv in enumerate(kvs):
            b, sl = kv.append_batch(seqs, pos)
            outs.append(kv.write_attend(0, b, sl, dev(kn[:, col(r, hl)]), dev(vn[:, col(r, hl)]), dev(q[:, col(r, ql)]),
                                        seqs, pos).cpu().numpy())
        rc, _, b, sl = ok.append_batch(seqs, pos)
        assert rc == 0
        ok.write_batch(0, b, sl, kn, vn)
        ref = ok.attend(0, q, seqs, pos, hq, hkv, d)
        full = np.concatenate([o.reshape(n, ql * d) for o in outs], axis=1)
        np.testing.assert_allclose(full, ref, rtol=1e-4, atol=2e-5, err_msg=f"step {step}")
    for kv in kvs:
        kv.check()
        assert np.array_equal(kv.free_list(), kvs[0].free_list())
        for s in range(n):
            assert np.array_equal(kv.seq_blocks(s), kvs[0].seq_blocks(s))
            assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s))
    for kv in kvs:
        kv.close()

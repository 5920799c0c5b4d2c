"""GPU parity at the benchmarked configurations, against the oracle.

The bench's numbers come from steps whose outputs are checked here on the
same workloads, built by the same code (bench.py's `workload`, `fill_plan`,
seeds and call order): the cache, filled through the C ABI exactly as the
bench fills it, and the oracle (the CPU restatement of kv.rs and of the
attention closure model.rs:431-476) receive identical appends and rows; each
decode step's attention is compared within the north-star tolerance, and
block tables, refcounts, free list and pool bytes bit-exact.

  C2  configs[1]: 64 sequences, lengths U[512, 4096], 16-token pieces of all
      sequences interleaved (scattered block ids), 32/8/128, decode steps of
      fused append + attention (lt_kv_write_attend) with f16 q/out as the
      bench runs them, and one with f32 q/out (the model runner's types,
      model.rs:393).
  C3  configs[2]: 256 sequences made by share(src, s, 2047) of a 2048-token
      prefix, 256 copy-on-write copies on the first divergent append, 256
      distinct suffix tokens each, then decode steps with the tensor-core
      shared-prefix pass on.
  C4  configs[3]: 16 x 32768 at 64/8/128 (one GPU), plus the per-rank shapes
      of its 8-GPU runs on one GPU -- head-sharded (1 KV head, 8 q heads,
      16 x 32768: each (token, head) cut over ~74 warps, the two-level
      stream-K merge) and batch-sharded (2 x 32768, 8 KV heads) -- each with
      the default launch sizing and with one tile per warp minimum.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

ATOL, RTOL = 2e-3, 1e-3          # f16 outputs vs the oracle's f32 result
ATOL32, RTOL32 = 2e-5, 1e-4      # f32 outputs (tests/test_gpu_parity.py)
BLOCK = 16


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


class BigTwin:
    """A GPU cache and the oracle with identical calls; rows are drawn on the
    GPU (the bench's generator and call order) and copied to the oracle."""

    def __init__(self, oracle_mod, hkv, hq, d, n_blocks, max_seqs):
        from langtrain_studio_b200.kv import KvCache

        self.kv = KvCache(1, hkv, d, n_blocks * BLOCK, n_heads=hq, max_seqs=max_seqs, max_batch=8192, device=0)
        self.ok = oracle_mod.OracleKv(1, hkv * d, n_blocks * BLOCK, max_seqs=max_seqs)
        self.hkv, self.hq, self.d, self.kvd = hkv, hq, d, hkv * d
        self.max_seqs = max_seqs

    def append(self, seqs, pos):
        b, s = self.kv.append_batch(seqs, pos)
        rc, done, bo, so = self.ok.append_batch(seqs, pos)
        assert rc == 0 and done == len(seqs)
        assert np.array_equal(b, bo) and np.array_equal(s, so)
        return b, s

    def write(self, b, s, k, v):
        """k, v: device f16 [n, kvd]."""
        self.kv.write(0, b, s, k, v)
        self.ok.write_batch(0, b, s, k.cpu().numpy(), v.cpu().numpy())

    def truncate(self, seq, frm):
        self.kv.truncate(seq, frm)
        self.ok.truncate(seq, frm)

    def share(self, src, dst, n):
        self.kv.share(src, dst, n)
        self.ok.share(src, dst, n)

    def decode_step(self, seqs, pos, k, v, q, out_dtype=torch.float16):
        """One bench step: append one token per sequence, then the fused
        write + attention launch; returns (GPU out as f32, oracle out)."""
        b, s = self.append(seqs, pos)
        out = self.kv.write_attend(0, b, s, k, v, q, seqs, pos, out_dtype=out_dtype)
        self.ok.write_batch(0, b, s, k.cpu().numpy(), v.cpu().numpy())
        ref = self.ok.attend(0, q.float().cpu().numpy(), seqs, pos, self.hq, self.hkv, self.d)
        torch.cuda.synchronize()
        self.kv.check()
        return out.float().cpu().numpy(), ref

    def check_tables(self):
        assert np.array_equal(self.kv.free_list(), self.ok.free_list())
        assert np.array_equal(self.kv.refs(), self.ok.refs())
        for s in range(self.max_seqs):
            assert self.kv.len(s) == self.ok.len(s), s
            assert np.array_equal(self.kv.seq_blocks(s), self.ok.seq_blocks(s)), s

    def check_pool(self, chunk=2048):
        """Every pool byte, in the reference layout, a chunk of blocks at a time."""
        torch.cuda.synchronize()
        ko, vo = self.ok.pool()
        nb = self.kv.n_blocks
        for b0 in range(0, nb, chunk):
            n = min(chunk, nb - b0)
            k, v = self.kv.pool_reference_layout(0, b0, n)
            assert np.array_equal(k, ko[0, b0:b0 + n]), f"K pool differs in blocks [{b0}, {b0 + n})"
            assert np.array_equal(v, vo[0, b0:b0 + n]), f"V pool differs in blocks [{b0}, {b0 + n})"

    def close(self):
        self.kv.close()


def _close(got, ref, atol, rtol, what):
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} outside atol {atol} / rtol {rtol}; "
                           f"max abs err {err.max():.3g}")


def test_c2_headline_steps_match_oracle(oracle_mod):
    import bench

    seed = bench.shard_seed(0)
    lens = bench.workload(seed)
    hq, hkv, d, B = bench.N_HEADS, bench.N_KV_HEADS, bench.HEAD_DIM, bench.BATCH
    n_blocks = int(((lens + bench.CYCLE + 1 + BLOCK - 1) // BLOCK).sum()) + B  # bench.build_cache's pool
    t = BigTwin(oracle_mod, hkv, hq, d, n_blocks, B)
    seqs, pos = bench.fill_plan(lens, seed)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(seed)
    for i in range(0, seqs.size, 8192):
        b, s = t.append(seqs[i:i + 8192], pos[i:i + 8192])
        k = torch.randn((b.size, hkv * d), generator=gen, device="cuda", dtype=torch.float16)
        v = torch.randn((b.size, hkv * d), generator=gen, device="cuda", dtype=torch.float16)
        t.write(b, s, k, v)
    ids = np.concatenate([t.kv.seq_blocks(i) for i in range(B)])
    assert not np.all(np.diff(ids) == 1), "block ids should be interleaved across sequences"
    g = torch.Generator(device="cuda")
    g.manual_seed(seed + 7)
    sq = np.arange(B, dtype=np.uint32)
    crossed = 0
    for phase in range(4):
        pos_now = (lens + phase).astype(np.uint32)
        crossed += int((pos_now % BLOCK == 0).sum())  # appends that take a new block
        packed = torch.randn((B, 2 * hkv * d + hq * d), generator=g, device="cuda", dtype=torch.float16)
        k, v, q = packed[:, :hkv * d], packed[:, hkv * d:2 * hkv * d], packed[:, 2 * hkv * d:]
        k, v, q = k.contiguous(), v.contiguous(), q.contiguous()
        if phase < 3:  # the bench's step: f16 q and out
            got, ref = t.decode_step(sq, pos_now, k, v, q)
            _close(got, ref, ATOL, RTOL, f"C2 step {phase} (f16 q/out)")
        else:  # the model runner's types: f32 q and out
            got, ref = t.decode_step(sq, pos_now, k, v, q.float())
            _close(got, ref, ATOL, RTOL, "C2 step 3 (f32 q, f16 out)")
    assert crossed > 0, "no step took a new block"
    got, ref = t.decode_step(sq, (lens + 4).astype(np.uint32), k, v, q.float(), out_dtype=torch.float32)
    _close(got, ref, ATOL32, RTOL32, "C2 step 4 (f32 q/out)")
    t.check_tables()
    t.check_pool()
    # the bench's cycle end: kv_remove back to the starting lengths
    for i in range(B):
        t.truncate(i, int(lens[i]))
    t.kv.flush()
    t.check_tables()
    t.close()


def test_c3_prefix_stress_matches_oracle(oracle_mod):
    """configs[2] as bench.run_c3 builds it, with the shared-prefix pass."""
    n_seq, prefix, suffix = 256, 2048, 256
    hq, hkv, d = 32, 8, 128
    kvd = hkv * d
    steps = 3
    per_seq_blocks = 1 + (suffix + steps + 2 + BLOCK - 1) // BLOCK
    n_blocks = prefix // BLOCK + n_seq * per_seq_blocks + 8
    t = BigTwin(oracle_mod, hkv, hq, d, n_blocks, n_seq + 1)
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    rnd = lambda n, w=kvd: torch.randn((n, w), generator=g, device="cuda", dtype=torch.float16)  # noqa: E731
    b, s = t.append(np.zeros(prefix, np.uint32), np.arange(prefix))
    t.write(b, s, rnd(prefix), rnd(prefix))
    seqs = np.arange(1, n_seq + 1, dtype=np.uint32)
    for i in seqs:
        t.share(0, int(i), prefix - 1)  # the scheduler's cap = len - 1 (prefix.rs:60)
    free0 = t.kv.free_blocks()
    b, s = t.append(seqs, np.full(n_seq, prefix - 1))  # every member copies the shared partial block
    assert free0 - t.kv.free_blocks() == n_seq
    t.write(b, s, rnd(n_seq), rnd(n_seq))
    t.check_tables()
    t.check_pool()  # 256 copy-on-write copies, bit-exact
    pos = np.arange(prefix, prefix + suffix)
    for i0 in range(0, n_seq, 32):
        ss = np.repeat(seqs[i0:i0 + 32], suffix)
        pp = np.tile(pos, len(seqs[i0:i0 + 32]))
        b, s = t.append(ss, pp)
        t.write(b, s, rnd(ss.size), rnd(ss.size))
    lens = np.full(n_seq, prefix + suffix, np.int64)
    c0 = t.kv.cascade_launches()
    for step in range(steps):
        k, v, q = rnd(n_seq), rnd(n_seq), rnd(n_seq, hq * d)
        got, ref = t.decode_step(seqs, lens.astype(np.uint32), k, v, q)
        _close(got, ref, ATOL, RTOL, f"C3 step {step}")
        lens += 1
    assert t.kv.cascade_launches() > c0, "the shared-prefix pass did not run"
    t.check_tables()
    t.check_pool()
    t.close()


C4_SHAPES = {
    # name: (sequences, KV heads, q heads) on one GPU
    "1gpu": (16, 8, 64),
    "head-x8-rank": (16, 1, 8),
    "batch-x8-rank": (2, 8, 64),
}


@pytest.mark.parametrize("shape", list(C4_SHAPES))
def test_c4_long_context_matches_oracle(oracle_mod, shape):
    """configs[3] as bench.run_c4 fills it (32768 tokens per sequence in
    8192-token appends), then decode steps under both launch sizings."""
    n_seq, hkv, hq = C4_SHAPES[shape]
    L, d = 32768, 128
    kvd = hkv * d
    n_blocks = n_seq * ((L + 16 + 1 + BLOCK - 1) // BLOCK) + 8
    t = BigTwin(oracle_mod, hkv, hq, d, n_blocks, n_seq)
    g = torch.Generator(device="cuda")
    g.manual_seed(1234)
    for sq in range(n_seq):
        for p0 in range(0, L, 8192):
            b, s = t.append(np.full(8192, sq), np.arange(p0, p0 + 8192))
            t.write(b, s, torch.randn((8192, kvd), generator=g, device="cuda", dtype=torch.float16),
                    torch.randn((8192, kvd), generator=g, device="cuda", dtype=torch.float16))
    seqs = np.arange(n_seq, dtype=np.uint32)
    for min_tiles in (8, 1):  # 8 is the handle's default
        t.kv.set_min_tiles_per_warp(min_tiles)
        for step in range(2):
            k = torch.randn((n_seq, kvd), generator=g, device="cuda", dtype=torch.float16)
            v = torch.randn((n_seq, kvd), generator=g, device="cuda", dtype=torch.float16)
            q = torch.randn((n_seq, hq * d), generator=g, device="cuda", dtype=torch.float16)
            got, ref = t.decode_step(seqs, np.full(n_seq, L + step, np.uint32), k, v, q)
            _close(got, ref, ATOL, RTOL, f"C4 {shape} min_tiles {min_tiles} step {step}")
        for sq in range(n_seq):
            t.truncate(sq, L)  # the bench's kv_remove back to 32768
    got, ref = t.decode_step(seqs, np.full(n_seq, L, np.uint32), k, v, q.float(), out_dtype=torch.float32)
    _close(got, ref, ATOL32, RTOL32, f"C4 {shape} f32 q/out")
    t.check_tables()
    t.check_pool()
    t.close()

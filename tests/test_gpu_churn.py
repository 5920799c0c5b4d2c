"""GPU tests of the continuous-batching churn workload
at small scale.

1. The Python restatement of the reference scheduler's KV policy
   (oracle/churn.py: admit, LRU eviction, preemption, retire, compaction
   every step) drives the C ABI while an oracle twin replays every call.
2. The native driver (include/lt_sched.h) runs the same policy in C++ on the
   GPU cache; the restatement runs beside it on the oracle with the same
   arrivals and the same K/V and q rows.
Either way the bookkeeping must match bit for bit after every step, the pool
bytes at the end, and the decode attention stays within the north-star
tolerance."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


class TwinKv:
    """KvCache facade that mirrors every call onto the oracle."""

    def __init__(self, kv, ok, hq, hkv, d):
        self.kv, self.ok = kv, ok
        self.hq, self.hkv, self.d = hq, hkv, d
        self.attn = []

    def free_blocks(self):
        assert self.kv.free_blocks() == self.ok.free_blocks()
        return self.kv.free_blocks()

    def truncate(self, s, frm):
        self.kv.truncate(s, frm)
        self.ok.truncate(s, frm)

    def append_batch(self, seqs, pos):
        b, sl = self.kv.append_batch(seqs, pos)
        rc, done, bo, so = self.ok.append_batch(seqs, pos)
        assert rc == 0 and np.array_equal(b, bo) and np.array_equal(sl, so)
        return b, sl

    def write(self, layer, b, sl, k, v):
        self.kv.write(layer, b, sl, k, v)
        self.ok.write_batch(layer, b, sl, k.cpu().numpy(), v.cpu().numpy())

    def write_attend(self, layer, b, sl, k, v, q, seqs, pos, out):
        self.kv.write_attend(layer, b, sl, k, v, q, seqs, pos, out=out)
        self.ok.write_batch(layer, b, sl, k.cpu().numpy(), v.cpu().numpy())
        ref = self.ok.attend(layer, q.float().cpu().numpy(), seqs, pos, self.hq, self.hkv, self.d)
        self.attn.append((out.float().cpu().numpy(), ref))

    def compact(self):
        moved = self.kv.compact()
        assert moved == len(self.ok.compact())
        return moved


def test_churn_driver_matches_oracle(oracle_mod):
    import bench
    from langtrain_studio_b200.kv import KvCache
    from oracle import churn

    hq, hkv, d = 8, 2, 128
    n_slots, pool = 24, 96
    kv = KvCache(1, hkv, d, pool * 16, n_heads=hq, max_seqs=n_slots, max_batch=4096, max_blocks_per_seq=64,
                 device=0)
    ok = oracle_mod.OracleKv(1, hkv * d, pool * 16, max_seqs=n_slots)
    twin = TwinKv(kv, ok, hq, hkv, d)
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    kv_src = torch.randn((4096, hkv * d), generator=g, device="cuda", dtype=torch.float16)
    q_src = torch.randn((n_slots, hq * d), generator=g, device="cuda", dtype=torch.float16)
    out = torch.empty((n_slots, hq * d), device="cuda", dtype=torch.float16)
    drv = churn.ChurnDriver(twin, n_slots, kv_src, q_src)
    arr = bench.Arrivals(1.5, 7, lo=8, hi=300, olo=4, ohi=40)
    for step in range(60):
        for p, o in arr.step():
            drv.submit(p, o)
        drv.step(out)
        assert np.array_equal(kv.free_list(), ok.free_list())
        assert np.array_equal(kv.refs(), ok.refs())
        for s in range(n_slots):
            assert kv.len(s) == ok.len(s)
            assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s))
    st = drv.stats
    assert st["evicted"] > 0 and st["moved"] > 0 and st["decode"] > 0 and st["prefill"] > 0, st
    torch.cuda.synchronize()
    kref, vref = ok.pool()
    kd, vd = kv.pool_reference_layout(0)
    assert np.array_equal(kd, kref[0]) and np.array_equal(vd, vref[0])
    for got, ref in twin.attn:
        np.testing.assert_allclose(got, ref, rtol=1e-3, atol=2e-3)
    kv.check()
    kv.close()


class _OracleData:
    """KvCache facade over the oracle with the data path (K/V writes, attention)."""

    def __init__(self, ok, hq, hkv, d):
        self.ok, self.hq, self.hkv, self.d = ok, hq, hkv, d
        self.last_attn = None

    def free_blocks(self):
        return self.ok.free_blocks()

    def truncate(self, s, frm):
        self.ok.truncate(s, frm)

    def append_batch(self, seqs, pos):
        rc, done, b, sl = self.ok.append_batch(seqs, pos)
        assert rc == 0
        return b, sl

    def write(self, layer, b, sl, k, v):
        self.ok.write_batch(layer, b, sl, k, v)

    def write_attend(self, layer, b, sl, k, v, q, seqs, pos, out):
        self.ok.write_batch(layer, b, sl, k, v)
        self.last_attn = self.ok.attend(layer, q.astype(np.float32), seqs, pos, self.hq, self.hkv, self.d)

    def compact(self):
        return len(self.ok.compact())

    def share(self, src, dst, n):
        self.ok.share(src, dst, n)

    def seq_blocks(self, s):
        return self.ok.seq_blocks(s)

    def refs(self):
        return self.ok.refs()


def test_native_scheduler_on_gpu_matches_oracle(oracle_mod):
    import bench
    from langtrain_studio_b200.kv import KvCache
    from langtrain_studio_b200.sched import Scheduler
    from oracle import churn

    hq, hkv, d = 8, 2, 128
    n_slots, pool = 32, 128
    kv = KvCache(1, hkv, d, pool * 16, n_heads=hq, max_seqs=n_slots, max_batch=8192, max_blocks_per_seq=64,
                 device=0)
    sched = Scheduler(kv, n_slots)
    ok = oracle_mod.OracleKv(1, hkv * d, pool * 16, max_seqs=n_slots)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    kv_src = torch.randn((4096, hkv * d), generator=g, device="cuda", dtype=torch.float16)
    q_src = torch.randn((n_slots, hq * d), generator=g, device="cuda", dtype=torch.float16)
    out = torch.empty((n_slots, hq * d), device="cuda", dtype=torch.float16)
    facade = _OracleData(ok, hq, hkv, d)
    drv = churn.ChurnDriver(facade, n_slots, kv_src.cpu().numpy(), q_src.cpu().numpy())
    arr = bench.Arrivals(2.0, 11, lo=8, hi=300, olo=4, ohi=40)
    worst = 0.0
    for step in range(80):
        for p, o in arr.step():
            sched.submit(p, o)
            drv.submit(p, o)
        nd = sched.step(kv_src, q_src, out)
        facade.last_attn = None
        drv.step(np.zeros((n_slots, hq * d), np.float16))
        assert np.array_equal(kv.free_list(), ok.free_list()), step
        assert np.array_equal(kv.refs(), ok.refs()), step
        for s in range(n_slots):
            assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s)), (step, s)
        if nd:
            got = out[:nd].float().cpu().numpy()
            np.testing.assert_allclose(got, facade.last_attn, rtol=1e-3, atol=2e-3)
            worst = max(worst, float(np.abs(got - facade.last_attn).max()))
    st = sched.stats
    assert st["evicted"] > 0 and st["moved_blocks"] > 0 and st["decode_tokens"] > 0 and st["prefill_tokens"] > 0
    torch.cuda.synchronize()
    kref, vref = ok.pool()
    kd, vd = kv.pool_reference_layout(0)
    assert np.array_equal(kd, kref[0]) and np.array_equal(vd, vref[0])
    kv.check()
    sched.close()
    kv.close()


def test_token_requests_with_prefix_reuse_on_gpu(oracle_mod):
    """Token requests (lt_sched_submit_tokens): shared system prompts are
    placed on or copied from the slots that hold them (kv_copy, then
    copy-on-write of the shared partial block on the GPU), only the suffix is
    written, decode tokens run the fused append + attention.  The Python
    restatement (oracle/prefix.py) drives the oracle with the same rows."""
    from langtrain_studio_b200.kv import KvCache
    from langtrain_studio_b200.sched import Scheduler
    from oracle import prefix as pref

    hq, hkv, d = 8, 2, 128
    n_slots, pool = 8, 160
    kv = KvCache(1, hkv, d, pool * 16, n_heads=hq, max_seqs=n_slots, max_batch=8192, max_blocks_per_seq=pool,
                 device=0)
    sched = Scheduler(kv, n_slots)
    ok = oracle_mod.OracleKv(1, hkv * d, pool * 16, max_seqs=n_slots)
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    kv_src = torch.randn((4096, hkv * d), generator=g, device="cuda", dtype=torch.float16)
    q_src = torch.randn((n_slots, hq * d), generator=g, device="cuda", dtype=torch.float16)
    out = torch.empty((n_slots, hq * d), device="cuda", dtype=torch.float16)
    facade = _OracleData(ok, hq, hkv, d)
    drv = pref.PrefixDriver(facade, n_slots, kv_src=kv_src.cpu().numpy(), q_src=q_src.cpu().numpy())
    rng = np.random.default_rng(4)
    worst = 0.0
    for step in range(90):
        if step < 70:
            for _ in range(int(rng.poisson(0.8))):
                k = int(rng.integers(0, 2))
                prompt = np.concatenate([(np.arange(40 + 37 * k) * 5 + k) % 997,
                                         rng.integers(1000, 9000, int(rng.integers(3, 60)))]).astype(np.int32)
                o = int(rng.integers(3, 30))
                sched.submit_tokens(prompt, o)
                drv.submit(prompt, o)
        nd = sched.step(kv_src, q_src, out)
        facade.last_attn = None
        assert drv.step() == nd, step
        assert np.array_equal(kv.free_list(), ok.free_list()), step
        assert np.array_equal(kv.refs(), ok.refs()), step
        for s in range(n_slots):
            assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s)), (step, s)
        if nd:
            got = out[:nd].float().cpu().numpy()
            np.testing.assert_allclose(got, facade.last_attn, rtol=1e-3, atol=2e-3)
            worst = max(worst, float(np.abs(got - facade.last_attn).max()))
    st = sched.stats
    assert st["copies"] > 0 and st["cached_tokens"] > 0 and st["decode_tokens"] > 0, st
    torch.cuda.synchronize()
    kref, vref = ok.pool()
    kd, vd = kv.pool_reference_layout(0)
    assert np.array_equal(kd, kref[0]) and np.array_equal(vd, vref[0])
    kv.check()
    sched.close()
    kv.close()

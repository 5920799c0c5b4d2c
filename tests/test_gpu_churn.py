"""GPU test of the continuous-batching churn workload at
small scale: bench.ChurnDriver drives the C ABI with the reference
scheduler's KV policy (admit, LRU eviction, preemption, retire, compaction
every step) while an oracle twin replays every call; bookkeeping must match
bit for bit after every step, the pool bytes at the end, and the attention of
the decode tokens stays within the north-star tolerance."""
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
    drv = bench.ChurnDriver(twin, n_slots, 1.5, 7, kv_src, q_src, prompt_lo=8, prompt_hi=300, out_lo=4, out_hi=40)
    for step in range(60):
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

"""GPU parity tests of the Q8_0 KV cache (include/lt_kv.h, LT_KV_Q8_0) through the C ABI.

Bar: pool bytes (int8 values and f16 scales) bit-exact against the oracle's
quantiser (quant.rs:785-795 on Q8_0 blocks) for every write path -- lt_kv_write
from f32 and f16, the fused append of lt_kv_write_attend, copy-on-write and
compaction moves; lt_kv_rows bit-exact; attention over q * d within the
north-star tolerance of the oracle's f32 attention (tighter for f32 outputs).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from test_gpu_parity import ATOL, RTOL, Twin  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def q8_twin(oracle_mod, *a, **kw):
    return Twin(oracle_mod, *a, kv_format="q8_0", **kw)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_write_is_bit_exact(oracle_mod, hd, dtype):
    rng = np.random.default_rng(hd)
    t = q8_twin(oracle_mod, 2, 4, hd, 16 * 20, n_heads=8, max_seqs=4)
    for s, L in enumerate([1, 17, 40, 100]):
        t.fill(s, L, rng, dtype=dtype)
    # magnitudes from tiny to large, exact zeros and one all-zero group
    b, sl = t.append(np.array([0, 0]), np.array([1, 2]))
    k = (rng.standard_normal((2, 4 * hd)) * np.logspace(-6, 4, 4 * hd)).astype(dtype)
    v = rng.standard_normal((2, 4 * hd)).astype(dtype)
    k[0, 5] = 0
    v[1, :32] = 0
    t.write(1, b, sl, k, v)
    t.check_pool()
    t.check_tables()
    for s, L in enumerate([3, 17, 40, 100]):
        for layer in range(2):
            kr, vr = t.kv.rows(layer, s, L)
            ko, vo = t.ok.rows(layer, s, L)
            assert np.array_equal(kr.cpu().numpy().view(np.uint16), ko)
            assert np.array_equal(vr.cpu().numpy().view(np.uint16), vo)


ATT_CASES = [
    # (head_dim, n_heads, n_kv_heads, lens)
    (128, 32, 8, [1, 15, 16, 17, 200]),
    (128, 64, 8, [513, 1100]),
    (64, 32, 4, [31, 192, 64]),
    (128, 8, 8, [2049, 3]),     # group 1
    (64, 12, 4, [77, 300]),     # group 3
]


@pytest.mark.parametrize("hd,hq,hkv,lens", ATT_CASES)
@pytest.mark.parametrize("q_dtype,out_dtype,min_tiles", [(torch.float32, torch.float32, 8),
                                                         (torch.float16, torch.float16, 8),
                                                         (torch.float32, torch.float32, 1)])
def test_attention_matches_oracle(oracle_mod, hd, hq, hkv, lens, q_dtype, out_dtype, min_tiles):
    rng = np.random.default_rng(hd + hq + len(lens))
    total = sum((L + 16) // 16 for L in lens) + 8
    t = q8_twin(oracle_mod, 1, hkv, hd, 16 * total, n_heads=hq, max_seqs=len(lens))
    t.kv.set_min_tiles_per_warp(min_tiles)
    for s, L in enumerate(lens):
        t.fill(s, L, rng)
    seqs = np.arange(len(lens))
    pos = np.array(lens) - 1
    q = rng.standard_normal((len(lens), hq * hd)).astype(np.float32)
    out, ref = t.attend_both(0, seqs, pos, q, q_dtype, out_dtype)
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)
    if out_dtype == torch.float32:
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    t.kv.check()


def test_stale_bytes_never_leak(oracle_mod):
    """A reused block keeps the previous sequence's bytes past the new
    sequence's end.  Here they were written from infinities (scale inf, values
    0), so 0 * scale would be NaN: such slots must not reach S or O."""
    rng = np.random.default_rng(9)
    t = q8_twin(oracle_mod, 1, 2, 64, 16 * 6, n_heads=4, max_seqs=3)
    b, sl = t.append(np.zeros(48, np.int64), np.arange(48))
    inf = np.full((48, 128), np.inf, np.float32)
    t.write(0, b, sl, inf, inf)
    t.check_pool()
    t.truncate(0, 0)
    t.fill(2, 5, rng)  # takes the last freed block: slots 5..15 keep scale inf
    q = rng.standard_normal((1, 4 * 64)).astype(np.float32)
    out, ref = t.attend_both(0, np.array([2]), np.array([4]), q)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("kv_dtype", [np.float32, np.float16])
def test_fused_write_attend_equals_write_then_attend(oracle_mod, kv_dtype):
    rng = np.random.default_rng(6)
    hkv, hd, hq = 8, 128, 32
    lens = [16, 33, 700, 1, 95]
    tot = sum((L + 17) // 16 for L in lens) * 2 + 16
    a = q8_twin(oracle_mod, 1, hkv, hd, 16 * tot, n_heads=hq, max_seqs=8)
    for s, L in enumerate(lens):
        a.fill(s, L, rng)
    seqs = np.arange(len(lens))
    pos = np.array(lens)
    b_, s_ = a.append(seqs, pos)
    k = rng.standard_normal((len(lens), hkv * hd)).astype(kv_dtype)
    v = rng.standard_normal((len(lens), hkv * hd)).astype(kv_dtype)
    q = rng.standard_normal((len(lens), hq * hd)).astype(np.float32)
    kd, vd, qd = (torch.from_numpy(x).cuda() for x in (k, v, q))
    out_f = a.kv.write_attend(0, b_, s_, kd, vd, qd, seqs, pos)
    a.ok.write_batch(0, b_, s_, k, v)
    a.check_pool()
    ref = a.ok.attend(0, q, seqs, pos, hq, hkv, hd)
    np.testing.assert_allclose(out_f.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)
    out_u = a.kv.attend(0, qd, seqs, pos)
    assert torch.equal(out_f, out_u)


@pytest.mark.parametrize("hd", [64, 128])
def test_fused_append_d64_and_d128(oracle_mod, hd):
    """The fused append's lane mapping differs with head_dim (half the lanes
    idle at 64): decode steps of several tokens keep the pool bit-exact."""
    rng = np.random.default_rng(hd + 1)
    hkv, hq = 4, 16
    t = q8_twin(oracle_mod, 1, hkv, hd, 16 * 40, n_heads=hq, max_seqs=4)
    lens = [3, 30, 64, 100]
    for s, L in enumerate(lens):
        t.fill(s, L, rng)
    for step in range(20):
        seqs = np.arange(4)
        pos = np.array([t.kv.len(s) for s in seqs])
        b, sl = t.append(seqs, pos)
        k = rng.standard_normal((4, hkv * hd)).astype(np.float32)
        v = rng.standard_normal((4, hkv * hd)).astype(np.float32)
        q = rng.standard_normal((4, hq * hd)).astype(np.float32)
        out = t.kv.write_attend(0, b, sl, *(torch.from_numpy(x).cuda() for x in (k, v, q)), seqs, pos)
        t.ok.write_batch(0, b, sl, k, v)
        ref = t.ok.attend(0, q, seqs, pos, hq, hkv, hd)
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)
    t.check_pool()


def test_cow_compaction_and_no_cascade(oracle_mod):
    """Copy-on-write copies and compaction moves carry the Q8_0 tiles
    byte for byte; shared prefixes never take the (f16-only) prefix pass."""
    rng = np.random.default_rng(7)
    t = q8_twin(oracle_mod, 2, 2, 64, 16 * 90, n_heads=8, max_seqs=12)
    t.fill(0, 200, rng)
    for s in range(1, 10):
        t.share(0, s, 150 + s)
        t.fill(s, 170 + 3 * s, rng)  # first append copies the shared partial block
    t.check_pool()
    seqs = np.arange(1, 10)
    pos = np.array([t.kv.len(s) - 1 for s in seqs])
    q = rng.standard_normal((9, 8 * 64)).astype(np.float32)
    c0 = t.kv.cascade_launches()
    for layer in range(2):
        out, ref = t.attend_both(layer, seqs, pos, q)
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    assert t.kv.cascade_launches() == c0
    t.truncate(0, 0)
    t.truncate(4, 0)
    assert t.compact() > 0
    t.check_tables()
    t.check_pool()
    seqs = np.array([1, 2, 3, 5, 6, 7, 8, 9])
    pos = np.array([t.kv.len(s) - 1 for s in seqs])
    out, ref = t.attend_both(1, seqs, pos, q[:8])
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)


def test_random_ops_full_parity(oracle_mod):
    rng = np.random.default_rng(300)
    max_seqs = 10
    t = q8_twin(oracle_mod, 2, 2, 64, 16 * 60, n_heads=4, max_seqs=max_seqs)
    t.kv.set_min_tiles_per_warp(1)
    for step in range(120):
        r = rng.random()
        if r < 0.5:
            seqs = rng.choice(max_seqs, size=int(rng.integers(1, 5)), replace=False)
            pos = np.array([t.kv.len(int(s)) for s in seqs])
            if (t.kv.free_blocks() - len(seqs)) < 2:
                continue
            b, sl = t.append(seqs, pos)
            layer = int(rng.integers(2))
            k = rng.standard_normal((seqs.size, 128)).astype(np.float32)
            v = rng.standard_normal((seqs.size, 128)).astype(np.float32)
            q = rng.standard_normal((seqs.size, 256)).astype(np.float32)
            out = t.kv.write_attend(layer, b, sl, *(torch.from_numpy(x).cuda() for x in (k, v, q)), seqs, pos)
            t.ok.write_batch(layer, b, sl, k, v)
            ref = t.ok.attend(layer, q, seqs, pos, 4, 2, 64)
            np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)
        elif r < 0.7:
            s = int(rng.integers(max_seqs))
            t.truncate(s, int(rng.integers(0, t.kv.len(s) + 1)))
        elif r < 0.85:
            src, dst = (int(x) for x in rng.choice(max_seqs, size=2, replace=False))
            t.share(src, dst, int(rng.integers(0, t.kv.len(src) + 2)))
        else:
            t.compact()
        if step % 20 == 19:
            t.check_tables()
            t.check_pool()
    t.check_tables()
    t.check_pool()

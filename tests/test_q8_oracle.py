"""CPU tests of the oracle's Q8_0 KV format (include/lt_kv.h, LT_KV_Q8_0).

The group quantiser is the engine's own (quant.rs:785-795): d = max|x| / 127,
id = 1/d (0 when d = 0), q = round(x * id) half away from zero, cast to int8
saturating (NaN -> 0).  The cache keeps d as f16 (the Q8_0 block of
quant.rs:254-275) and reads a value back as q * d.  Pinned here by
hand-worked known answers and by an independent numpy restatement.
"""
import numpy as np
import pytest


def np_q8_group(x):
    """numpy restatement of quant.rs:785-795 (f32 arithmetic, like the Rust)."""
    x = np.asarray(x, np.float32)
    finite_abs = np.abs(x)[~np.isnan(x)]
    amax = np.float32(finite_abs.max()) if finite_abs.size else np.float32(0)
    d = np.float32(amax / np.float32(127.0))
    idv = np.float32(np.float32(1.0) / d) if d > 0 else np.float32(0)
    with np.errstate(invalid="ignore", over="ignore"):
        y = (x * idv).astype(np.float64)  # the f32 product, widened exactly
        r = np.trunc(y + np.copysign(0.5, y))  # half away from zero, exact in f64
        r = np.where(np.isnan(r), 0, np.clip(r, -128, 127))
    return r.astype(np.int8), d


def f16_bits(x):
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def test_group_known_answers(oracle_mod):
    # amax 127 -> d = 1, id = 1: exact half-way cases round away from zero
    x = np.zeros(32, np.float32)
    x[:8] = [127, 0.5, 1.5, -0.5, -2.5, 2.5, 126.5, -127]
    q, d = oracle_mod.q8_group(x)
    assert d == 1.0
    assert q[:8].tolist() == [127, 1, 2, -1, -3, 3, 127, -127]
    assert (q[8:] == 0).all()
    # all zero: d = 0, id = 0
    q, d = oracle_mod.q8_group(np.zeros(32, np.float32))
    assert d == 0.0 and (q == 0).all()
    # a NaN is ignored by the maximum and quantises to 0
    x = np.zeros(32, np.float32)
    x[:3] = [np.nan, 1.0, -0.25]
    q, d = oracle_mod.q8_group(x)
    assert d == np.float32(1.0) / np.float32(127.0)
    assert q[:3].tolist() == [0, 127, -32]
    # an infinity: d = inf, id = 0, every value (inf * 0 = NaN included) -> 0
    x = np.linspace(-3, 3, 32).astype(np.float32)
    x[5] = np.inf
    q, d = oracle_mod.q8_group(x)
    assert np.isinf(d) and (q == 0).all()


def test_group_matches_numpy_restatement(oracle_mod):
    rng = np.random.default_rng(3)
    for scale in (1e-30, 1e-6, 1e-3, 1.0, 7.5, 3e4, 1e30):
        for _ in range(200):
            x = (rng.standard_normal(32) * scale).astype(np.float32)
            if rng.random() < 0.2:
                x[rng.integers(32)] = 0.0
            q, d = oracle_mod.q8_group(x)
            qn, dn = np_q8_group(x)
            assert np.array_equal(q, qn), (scale, x)
            assert np.float32(d) == dn


@pytest.mark.parametrize("kv_dim", [64, 256])
def test_cache_write_rows_and_format(oracle_mod, kv_dim):
    rng = np.random.default_rng(kv_dim)
    kv = oracle_mod.OracleKv(2, kv_dim, 64, 4, kv_format="q8_0")
    assert kv.bytes() == 2 * 4 * 16 * 2 * (kv_dim + kv_dim // 32 * 2)
    n = 20
    _, done, b, s = kv.append_batch(np.zeros(n, np.uint32), np.arange(n))
    assert done == n
    k = (rng.standard_normal((n, kv_dim)) * 3).astype(np.float32)
    v = rng.standard_normal((n, kv_dim)).astype(np.float16)  # f16 input is widened, then quantised
    kv.write_batch(1, b, s, k, v)
    kq, vq, kd, vd = kv.pool_q8()
    for i in range(n):
        for g in range(kv_dim // 32):
            qn, dn = np_q8_group(k[i, 32 * g:32 * g + 32])
            assert np.array_equal(kq[1, b[i], s[i], 32 * g:32 * g + 32], qn)
            assert kd[1, b[i], s[i], g] == f16_bits(dn)
            qn, dn = np_q8_group(v[i, 32 * g:32 * g + 32].astype(np.float32))
            assert np.array_equal(vq[1, b[i], s[i], 32 * g:32 * g + 32], qn)
            assert vd[1, b[i], s[i], g] == f16_bits(dn)
    kr, vr = kv.rows(1, 0, n)
    deq = kq[1, b, s].astype(np.float32) * np.repeat(kd[1, b, s].view(np.float16).astype(np.float32), 32, axis=1)
    assert np.array_equal(kr, f16_bits(deq))
    deq = vq[1, b, s].astype(np.float32) * np.repeat(vd[1, b, s].view(np.float16).astype(np.float32), 32, axis=1)
    assert np.array_equal(vr, f16_bits(deq))


def test_attention_over_dequantised_rows(oracle_mod):
    rng = np.random.default_rng(11)
    hkv, hq, d = 2, 8, 64
    kv = oracle_mod.OracleKv(1, hkv * d, 16 * 20, 3, kv_format="q8_0")
    lens = [5, 33, 70]
    for sq, L in enumerate(lens):
        _, _, b, s = kv.append_batch(np.full(L, sq, np.uint32), np.arange(L))
        kv.write_batch(0, b, s, rng.standard_normal((L, hkv * d)).astype(np.float32),
                       rng.standard_normal((L, hkv * d)).astype(np.float32))
    q = rng.standard_normal((3, hq * d)).astype(np.float32)
    pos = np.array(lens) - 1
    out = kv.attend(0, q, np.arange(3), pos, hq, hkv, d)
    kq, vq, kd, vd = kv.pool_q8()
    scale = 1.0 / np.sqrt(d)
    for i, L in enumerate(lens):
        blocks = kv.seq_blocks(i)
        rows = [(blocks[p // 16], p % 16) for p in range(L)]
        K = np.stack([kq[0, bb, ss].astype(np.float64) * np.repeat(kd[0, bb, ss].view(np.float16), 32)
                      for bb, ss in rows])
        V = np.stack([vq[0, bb, ss].astype(np.float64) * np.repeat(vd[0, bb, ss].view(np.float16), 32)
                      for bb, ss in rows])
        for h in range(hq):
            kh = h // (hq // hkv)
            sc = K[:, kh * d:(kh + 1) * d] @ q[i, h * d:(h + 1) * d].astype(np.float64) * scale
            w = np.exp(sc - sc.max())
            w /= w.sum()
            ref = w @ V[:, kh * d:(kh + 1) * d]
            np.testing.assert_allclose(out[i, h * d:(h + 1) * d], ref, rtol=2e-5, atol=2e-6)


def test_copy_on_write_and_compaction_move_q8_bytes(oracle_mod):
    rng = np.random.default_rng(5)
    kv = oracle_mod.OracleKv(2, 64, 16 * 12, 4, kv_format="q8_0")
    _, _, b, s = kv.append_batch(np.zeros(20, np.uint32), np.arange(20))
    for layer in range(2):
        kv.write_batch(layer, b, s, rng.standard_normal((20, 64)).astype(np.float32),
                       rng.standard_normal((20, 64)).astype(np.float32))
    before = [kv.rows(layer, 0, 20) for layer in range(2)]
    kv.share(0, 1, 20)
    _, _, b1, s1 = kv.append_batch(np.array([1], np.uint32), np.array([20]))  # CoW of the shared last block
    assert b1[0] != kv.seq_blocks(0)[-1]
    for layer in range(2):
        kr, vr = kv.rows(layer, 1, 20)
        assert np.array_equal(kr, before[layer][0]) and np.array_equal(vr, before[layer][1])
    kv.truncate(0, 0)
    assert len(kv.compact()) > 0
    for layer in range(2):
        kr, vr = kv.rows(layer, 1, 20)
        assert np.array_equal(kr, before[layer][0]) and np.array_equal(vr, before[layer][1])

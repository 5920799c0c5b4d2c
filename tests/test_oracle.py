"""CPU tests of the oracle itself: pinned against the reference's known-answer
tests (engine/crates/native/src/kv.rs:202-229, ported verbatim), against the
F16C/numpy golden vectors for f32->f16, and against an independent float64
restatement of the attention closure (engine/crates/native/src/model.rs:431-476).
"""
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"


def fill(kv, seq, n, base):
    """kv.rs:194-200: append positions len..n of seq, row value base + p."""
    for p in range(kv.len(seq), n):
        b, s = kv.append(seq, p)
        x = np.full(kv.kv_dim, base + p, np.float32)
        kv.write(0, b, s, x, x)


def f16(u16):
    return np.asarray(u16, np.uint16).view(np.float16).astype(np.float32)


def test_share_then_diverge_copies_on_write(oracle_mod):
    """kv.rs:202-217."""
    kv = oracle_mod.OracleKv(1, 4, 256, max_seqs=8)
    fill(kv, 0, 20, 0.0)
    kv.share(0, 1, 20)
    free_before = kv.free_blocks()
    b, s = kv.append(1, 20)
    kv.write(0, b, s, np.full(4, 1000.0, np.float32), np.full(4, 1000.0, np.float32))
    assert kv.free_blocks() == free_before - 1
    a = f16(kv.rows(0, 0, 20)[0][:, 0])
    c = f16(kv.rows(0, 1, 21)[0][:, 0])
    assert np.array_equal(a, c[:20])
    assert c[20] == 1000.0
    assert kv.len(0) == 20


def test_truncate_frees_blocks(oracle_mod):
    """kv.rs:219-229."""
    kv = oracle_mod.OracleKv(1, 4, 64, max_seqs=8)
    fill(kv, 3, 40, 0.0)
    assert kv.free_blocks() == 1
    kv.truncate(3, 10)
    assert kv.free_blocks() == 3
    kv.truncate(3, 0)
    assert kv.free_blocks() == 4
    with pytest.raises(oracle_mod.OracleError):
        kv.append(3, 5)


def test_free_list_order_and_errors(oracle_mod):
    """kv.rs:45 (first alloc is block 0), :67-74 (full), :87-92 (non-contiguous)."""
    kv = oracle_mod.OracleKv(2, 8, 48, max_seqs=4)  # 3 blocks
    assert kv.capacity() == 48 and kv.bytes() == 2 * 3 * 16 * 8 * 2 * 2
    assert list(kv.free_list()) == [2, 1, 0]
    assert kv.append(0, 0) == (0, 0)
    assert kv.append(1, 0) == (1, 0)
    with pytest.raises(oracle_mod.OracleError) as e:
        kv.append(0, 5)
    assert e.value.code == oracle_mod.NONCONTIG
    assert kv.append(2, 0) == (2, 0)
    with pytest.raises(oracle_mod.OracleError) as e:
        kv.append(3, 0)
    assert e.value.code == oracle_mod.FULL
    kv.truncate(1, 0)
    assert list(kv.free_list()) == [1]
    assert kv.append(3, 0) == (1, 0)


def test_share_self_removes_sequence(oracle_mod):
    """share(x, x, len) truncates x first and then finds no source (kv.rs:173-174)."""
    kv = oracle_mod.OracleKv(1, 4, 64, max_seqs=4)
    fill(kv, 0, 20, 0.0)
    kv.share(0, 0, 10)
    assert kv.len(0) == 0 and kv.free_blocks() == 4


def test_f16_conversion_golden(oracle_mod):
    g = np.load(GOLDEN / "f16_convert.npz")
    x = g["f32_bits"].view(np.float32)
    got = oracle_mod.f32_to_f16_bits(x)
    bad = np.nonzero(got != g["f16_bits"])[0]
    assert bad.size == 0, f"{bad.size} mismatches, first f32 bits {g['f32_bits'][bad[:5]]}"


def test_compaction_rule(oracle_mod):
    kv = oracle_mod.OracleKv(2, 8, 16 * 10, max_seqs=8)
    for s in range(5):
        fill(kv, s, 16 * 2 - s, float(10 * s))
    kv.truncate(1, 0)
    kv.truncate(3, 5)
    before = {s: kv.rows(1, s, kv.len(s)) for s in range(5) if kv.len(s)}
    before0 = {s: kv.rows(0, s, kv.len(s)) for s in range(5) if kv.len(s)}
    moves = kv.compact()
    live = np.nonzero(kv.refs())[0]
    assert list(live) == list(range(len(live)))  # live blocks packed at the bottom
    assert list(kv.free_list()) == list(range(kv.n_blocks - 1, len(live) - 1, -1))
    assert all(src > dst for src, dst in moves)
    for s, (k, v) in before.items():
        k2, v2 = kv.rows(1, s, kv.len(s))
        assert np.array_equal(k, k2) and np.array_equal(v, v2)
        k0, v0 = kv.rows(0, s, kv.len(s))
        assert np.array_equal(before0[s][0], k0)


def attention_f64(q, krows, vrows, n_heads, n_kv_heads, hd):
    """Independent float64 restatement of model.rs:431-476 for one token."""
    group = n_heads // n_kv_heads
    out = np.zeros(n_heads * hd)
    for h in range(n_kv_heads):
        K = krows[:, h * hd:(h + 1) * hd].astype(np.float64)
        V = vrows[:, h * hd:(h + 1) * hd].astype(np.float64)
        for g in range(group):
            qh = q[(h * group + g) * hd:(h * group + g + 1) * hd].astype(np.float64)
            s = K @ qh / np.sqrt(hd)
            p = np.exp(s - s.max())
            p /= p.sum()
            out[(h * group + g) * hd:(h * group + g + 1) * hd] = p @ V
    return out


@pytest.mark.parametrize("hd,hq,hkv", [(64, 8, 2), (128, 16, 4), (128, 8, 1)])
def test_oracle_attention_matches_float64(oracle_mod, hd, hq, hkv):
    rng = np.random.default_rng(1)
    kv = oracle_mod.OracleKv(1, hkv * hd, 16 * 40, max_seqs=8)
    lens = [1, 17, 200]
    for s, L in enumerate(lens):
        blocks, slots = [], []
        for p in range(L):
            b, sl = kv.append(s, p)
            blocks.append(b)
            slots.append(sl)
        kv.write_batch(0, blocks, slots, rng.standard_normal((L, hkv * hd), np.float32),
                       rng.standard_normal((L, hkv * hd), np.float32))
    q = rng.standard_normal((3, hq * hd)).astype(np.float32)
    pos = np.array([L - 1 for L in lens], np.uint32)
    out = kv.attend(0, q, np.arange(3), pos, hq, hkv, hd, n_threads=2)
    for i, L in enumerate(lens):
        k, v = kv.rows(0, i, L)
        ref = attention_f64(q[i], f16(k), f16(v), hq, hkv, hd)
        np.testing.assert_allclose(out[i], ref, rtol=1e-5, atol=1e-6)


def test_oracle_attention_thread_count_invariant(oracle_mod):
    rng = np.random.default_rng(2)
    kv = oracle_mod.OracleKv(1, 2 * 64, 16 * 64, max_seqs=8)
    for s in range(4):
        L = 100 + 37 * s
        bl = [kv.append(s, p) for p in range(L)]
        kv.write_batch(0, [b for b, _ in bl], [x for _, x in bl], rng.standard_normal((L, 128), np.float32),
                       rng.standard_normal((L, 128), np.float32))
    q = rng.standard_normal((4, 8 * 64)).astype(np.float32)
    pos = np.array([99, 136, 173, 210], np.uint32)
    a = kv.attend(0, q, np.arange(4), pos, 8, 2, 64, n_threads=1)
    b = kv.attend(0, q, np.arange(4), pos, 8, 2, 64, n_threads=4)
    assert np.array_equal(a, b)

"""GPU parity tests: every kernel through the C ABI against the oracle.

Bar (north star): bit-exact for append (pool bytes), block tables, copy-on-
write and compaction; attention within max-abs 2e-3 / rel 1e-3 of the
oracle's f32 result (ATOL / RTOL below).
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3  # north-star attention tolerance (fp16 outputs vs f32 reference)


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


class Twin:
    """The GPU cache and the oracle, driven with identical calls."""

    def __init__(self, oracle_mod, n_layers, n_kv_heads, head_dim, n_tokens, n_heads=None, max_seqs=16,
                 max_batch=4096, kv_format="f16"):
        from langtrain_studio_b200.kv import KvCache

        self.kv = KvCache(n_layers, n_kv_heads, head_dim, n_tokens, n_heads=n_heads or n_kv_heads,
                          max_seqs=max_seqs, max_batch=max_batch, device=0, kv_format=kv_format)
        self.ok = oracle_mod.OracleKv(n_layers, n_kv_heads * head_dim, n_tokens, max_seqs=max_seqs,
                                      kv_format=kv_format)
        self.kv_format = kv_format
        self.om = oracle_mod
        self.L, self.hkv, self.d = n_layers, n_kv_heads, head_dim
        self.hq = n_heads or n_kv_heads
        self.kv_dim = n_kv_heads * head_dim
        self.max_seqs = max_seqs

    def append(self, seqs, pos):
        b, s = self.kv.append_batch(seqs, pos)
        rc, done, bo, so = self.ok.append_batch(seqs, pos)
        assert rc == 0 and np.array_equal(b, bo) and np.array_equal(s, so)
        return b, s

    def write(self, layer, b, s, k, v):
        """k, v: numpy f32 or f16 [n, kv_dim]."""
        self.kv.write(layer, b, s, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        self.ok.write_batch(layer, b, s, k, v)

    def fill(self, seq, n, rng, layers=None, dtype=np.float32):
        start = self.kv.len(seq)
        if n <= start:
            return
        pos = np.arange(start, n)
        b, s = self.append(np.full(pos.size, seq), pos)
        for layer in (range(self.L) if layers is None else layers):
            k = rng.standard_normal((pos.size, self.kv_dim)).astype(dtype)
            v = rng.standard_normal((pos.size, self.kv_dim)).astype(dtype)
            self.write(layer, b, s, k, v)

    def truncate(self, seq, frm):
        self.kv.truncate(seq, frm)
        self.ok.truncate(seq, frm)

    def share(self, src, dst, n):
        self.kv.share(src, dst, n)
        self.ok.share(src, dst, n)

    def compact(self):
        moved = self.kv.compact()
        assert moved == len(self.ok.compact())
        return moved

    def check_pool(self):
        torch.cuda.synchronize()
        if self.kv_format == "q8_0":
            ref = self.ok.pool_q8()
            for layer in range(self.L):
                got = self.kv.pool_reference_layout(layer)
                for name, a, r in zip(("Kq", "Vq", "Kd", "Vd"), got, ref):
                    assert np.array_equal(a, r[layer]), f"{name} pool differs in layer {layer}"
            return
        ko, vo = self.ok.pool()
        for layer in range(self.L):
            k, v = self.kv.pool_reference_layout(layer)
            assert np.array_equal(k, ko[layer]), f"K pool differs in layer {layer}"
            assert np.array_equal(v, vo[layer]), f"V pool differs in layer {layer}"

    def check_tables(self):
        assert np.array_equal(self.kv.free_list(), self.ok.free_list())
        assert np.array_equal(self.kv.refs(), self.ok.refs())
        for s in range(self.max_seqs):
            assert self.kv.len(s) == self.ok.len(s)
            assert np.array_equal(self.kv.seq_blocks(s), self.ok.seq_blocks(s))

    def attend_both(self, layer, seqs, pos, q, q_dtype=torch.float32, out_dtype=torch.float32):
        qd = torch.from_numpy(q).cuda().to(q_dtype)
        out = self.kv.attend(layer, qd, seqs, pos, out_dtype=out_dtype)
        q_used = qd.float().cpu().numpy()
        ref = self.ok.attend(layer, q_used, seqs, pos, self.hq, self.hkv, self.d)
        return out.float().cpu().numpy(), ref


def test_known_answer_share_then_diverge(oracle_mod):
    """kv.rs:202-217 with the data path on the GPU."""
    t = Twin(oracle_mod, 1, 1, 64, 256)
    for p in range(20):
        b, s = t.append([0], [p])
        x = np.full((1, 64), float(p), np.float32)
        t.write(0, b, s, x, x)
    t.share(0, 1, 20)
    free_before = t.kv.free_blocks()
    b, s = t.append([1], [20])
    x = np.full((1, 64), 1000.0, np.float32)
    t.write(0, b, s, x, x)
    assert t.kv.free_blocks() == free_before - 1
    a = t.kv.rows(0, 0, 20)[0][:, 0].float().cpu().numpy()
    c = t.kv.rows(0, 1, 21)[0][:, 0].float().cpu().numpy()
    assert np.array_equal(a, c[:20])
    assert c[20] == 1000.0
    assert t.kv.len(0) == 20
    t.check_pool()
    t.check_tables()


def test_known_answer_truncate_frees_blocks(oracle_mod):
    """kv.rs:219-229 through the GPU handle."""
    from langtrain_studio_b200.kv import KvNonContiguous

    t = Twin(oracle_mod, 1, 1, 64, 64)
    t.fill(3, 40, np.random.default_rng(0))
    assert t.kv.free_blocks() == 1
    t.truncate(3, 10)
    assert t.kv.free_blocks() == 3
    t.truncate(3, 0)
    assert t.kv.free_blocks() == 4
    with pytest.raises(KvNonContiguous):
        t.kv.append(3, 5)


@pytest.mark.parametrize("hd", [64, 128])
def test_write_bit_exact_f32_all_classes(oracle_mod, hd):
    """K1: f32 -> f16 in the kernel equals half::f16::from_f32 bit for bit,
    over the golden edge classes (NaN payloads, ties, subnormals, overflow)."""
    from pathlib import Path

    g = np.load(Path(__file__).parent / "golden" / "f16_convert.npz")
    vals = g["f32_bits"].view(np.float32)
    hkv = 2
    kv_dim = hkv * hd
    n_tok = (vals.size + kv_dim - 1) // kv_dim
    vals = np.resize(vals, n_tok * 2 * kv_dim).reshape(2, n_tok, kv_dim)
    t = Twin(oracle_mod, 2, hkv, hd, 16 * (n_tok + 16), max_batch=n_tok + 8)
    b, s = t.append(np.zeros(n_tok, int), np.arange(n_tok))
    t.write(1, b, s, np.ascontiguousarray(vals[0]), np.ascontiguousarray(vals[1]))
    t.check_pool()
    kr, vr = t.kv.rows(1, 0, n_tok)
    ko, vo = t.ok.rows(1, 0, n_tok)
    assert np.array_equal(kr.cpu().numpy().view(np.uint16), ko)
    assert np.array_equal(vr.cpu().numpy().view(np.uint16), vo)


def test_write_f16_stored_unchanged(oracle_mod):
    rng = np.random.default_rng(3)
    t = Twin(oracle_mod, 1, 4, 128, 16 * 20)
    b, s = t.append(np.zeros(50, int), np.arange(50))
    k = rng.standard_normal((50, 512)).astype(np.float16)
    v = rng.standard_normal((50, 512)).astype(np.float16)
    t.write(0, b, s, k, v)
    t.check_pool()


def test_cow_copies_all_layers(oracle_mod):
    """K3: divergence from a shared partial block copies it for every layer."""
    rng = np.random.default_rng(4)
    t = Twin(oracle_mod, 3, 2, 128, 16 * 64)
    t.fill(0, 40, rng)
    for dst in (1, 2, 3):
        t.share(0, dst, 37)
    t.fill(1, 45, rng)  # CoW of block 2 (positions 32..39) at pos 37
    t.fill(0, 41, rng)  # seq 0 writes into its still-shared block: CoW as well
    t.fill(2, 38, rng)
    t.check_tables()
    t.check_pool()


ATT_CASES = [
    # (head_dim, n_heads, n_kv_heads, lens)
    (128, 32, 8, [1, 15, 16, 17, 200]),
    (128, 64, 8, [513, 1100]),          # G=8, multi-chunk split-K
    (64, 32, 4, [31, 192, 64]),         # config-1 shape
    (128, 8, 2, [2049]),
    (128, 16, 2, [131, 149, 160]),      # with min_tiles 1: 8, 9, 10 helper warps (two-level merge from 9)
]


@pytest.mark.parametrize("hd,hq,hkv,lens", ATT_CASES)
@pytest.mark.parametrize("q_dtype,out_dtype,min_tiles", [(torch.float32, torch.float32, 8),
                                                         (torch.float16, torch.float16, 8),
                                                         (torch.float32, torch.float32, 1),
                                                         (torch.float16, torch.float32, 3)])
def test_attention_matches_oracle(oracle_mod, hd, hq, hkv, lens, q_dtype, out_dtype, min_tiles):
    """min_tiles 1 splits every (token, head) over the most warps (the most
    merges); the default 8 is the launch sizing of small steps."""
    rng = np.random.default_rng(hd + hq + len(lens))
    total = sum((L + 16) // 16 for L in lens) + 8
    t = Twin(oracle_mod, 1, hkv, hd, 16 * total, n_heads=hq, max_seqs=len(lens))
    t.kv.set_min_tiles_per_warp(min_tiles)
    for s, L in enumerate(lens):
        t.fill(s, L, rng)
    seqs = np.arange(len(lens))
    pos = np.array(lens) - 1
    q = rng.standard_normal((len(lens), hq * hd)).astype(np.float32)
    out, ref = t.attend_both(0, seqs, pos, q, q_dtype, out_dtype)
    np.testing.assert_allclose(out, ref, rtol=RTOL, atol=ATOL)
    if out_dtype == torch.float32:
        # f32 out: much tighter than the bar (hi/lo split of q and P).
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    t.kv.check()


def test_attention_prefill_positions(oracle_mod):
    """Several tokens of one sequence in one call (chunked prefill): token i
    attends over [0, pos_i] only."""
    rng = np.random.default_rng(9)
    t = Twin(oracle_mod, 1, 2, 128, 16 * 40, n_heads=8)
    t.fill(0, 300, rng)
    pos = np.array([0, 5, 15, 16, 100, 299])
    q = rng.standard_normal((pos.size, 8 * 128)).astype(np.float32)
    out, ref = t.attend_both(0, np.zeros(pos.size, int), pos, q)
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)


def test_stale_rows_never_leak(oracle_mod):
    """Rows past the sequence end hold stale NaN/Inf from an earlier owner;
    attention must not see them (reference reads exactly len rows)."""
    t = Twin(oracle_mod, 1, 1, 128, 16 * 4, n_heads=4)
    b, s = t.append(np.zeros(16, int), np.arange(16))
    bad = np.full((16, 128), np.nan, np.float32)
    bad[::2] = np.inf
    t.write(0, b, s, bad, bad)
    t.truncate(0, 0)
    rng = np.random.default_rng(5)
    t.fill(1, 3, rng)  # same block, slots 0..2 rewritten, 3..15 stale NaN/Inf
    q = rng.standard_normal((1, 4 * 128)).astype(np.float32)
    out, ref = t.attend_both(0, [1], [2], q)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("kv_dtype", [np.float32, np.float16])
def test_fused_write_attend_equals_write_then_attend(oracle_mod, kv_dtype):
    rng = np.random.default_rng(6)
    hkv, hd, hq = 8, 128, 32
    lens = [16, 33, 700, 1, 95]
    tot = sum((L + 17) // 16 for L in lens) * 2 + 16
    a = Twin(oracle_mod, 1, hkv, hd, 16 * tot, n_heads=hq, max_seqs=8)
    for s, L in enumerate(lens):
        a.fill(s, L, rng)
    seqs = np.arange(len(lens))
    pos = np.array(lens)
    b_, s_ = a.append(seqs, pos)
    k = rng.standard_normal((len(lens), hkv * hd)).astype(kv_dtype)
    v = rng.standard_normal((len(lens), hkv * hd)).astype(kv_dtype)
    q = rng.standard_normal((len(lens), hq * hd)).astype(np.float32)
    kd, vd, qd = (torch.from_numpy(x).cuda() for x in (k, v, q))
    launches = a.kv.launch_count()
    out_f = a.kv.write_attend(0, b_, s_, kd, vd, qd, seqs, pos)
    assert a.kv.launch_count() - launches <= 3  # plan + fused attention (+ split-K combine)
    a.ok.write_batch(0, b_, s_, k, v)
    a.check_pool()
    ref = a.ok.attend(0, q, seqs, pos, hq, hkv, hd)
    np.testing.assert_allclose(out_f.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)
    out_u = a.kv.attend(0, qd, seqs, pos)
    assert torch.equal(out_f, out_u)


def test_compaction_moves_data_and_remaps(oracle_mod):
    """K4: after compaction pool, tables, refs and attention all match."""
    rng = np.random.default_rng(7)
    t = Twin(oracle_mod, 2, 2, 64, 16 * 80, n_heads=8, max_seqs=8)
    for s in range(6):
        t.fill(s, 30 + 41 * s, rng)
    t.share(5, 6, 100)
    t.truncate(1, 0)
    t.truncate(3, 7)
    t.fill(6, 130, rng)
    t.truncate(0, 0)
    moved = t.compact()
    assert moved > 0
    t.check_tables()
    t.check_pool()
    seqs = np.array([2, 3, 4, 5, 6])
    pos = np.array([t.kv.len(s) - 1 for s in seqs])
    q = rng.standard_normal((5, 8 * 64)).astype(np.float32)
    for layer in range(2):
        out, ref = t.attend_both(layer, seqs, pos, q)
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    # keep working after compaction: new appends take the lowest free ids
    t.fill(0, 20, rng)
    t.check_tables()
    t.check_pool()


@pytest.mark.parametrize("seed", [0, 1])
def test_random_ops_full_parity(oracle_mod, seed):
    """Long random mixes of the scheduler's calls with data on the GPU."""
    rng = np.random.default_rng(100 + seed)
    max_seqs = 10
    t = Twin(oracle_mod, 2, 2, 64, 16 * 60, n_heads=4, max_seqs=max_seqs)
    t.kv.set_min_tiles_per_warp([1, 8, 2][seed % 3])
    for step in range(120):
        r = rng.random()
        if r < 0.5:
            seqs = rng.choice(max_seqs, size=int(rng.integers(1, 5)), replace=False)
            pos = np.array([t.kv.len(int(s)) for s in seqs])
            if (t.kv.free_blocks() - len(seqs)) < 2:
                continue
            b, s = t.append(seqs, pos)
            for layer in range(2):
                k = rng.standard_normal((len(seqs), 128)).astype(np.float32)
                v = rng.standard_normal((len(seqs), 128)).astype(np.float32)
                t.write(layer, b, s, k, v)
        elif r < 0.7:
            s = int(rng.integers(0, max_seqs))
            t.truncate(s, int(rng.integers(0, t.kv.len(s) + 2)))
        elif r < 0.9:
            src, dst = (int(x) for x in rng.choice(max_seqs, 2, replace=False))
            t.share(src, dst, int(rng.integers(0, t.kv.len(src) + 3)))
        else:
            t.compact()
        if step % 20 == 19:
            t.check_tables()
            t.check_pool()
            live = [s for s in range(max_seqs) if t.kv.len(s) > 0]
            if live:
                pos = np.array([t.kv.len(s) - 1 for s in live])
                q = rng.standard_normal((len(live), 4 * 64)).astype(np.float32)
                out, ref = t.attend_both(1, np.array(live), pos, q)
                np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    t.kv.check()


def test_bad_arguments_are_rejected_without_launch(oracle_mod):
    from langtrain_studio_b200.kv import KvError

    t = Twin(oracle_mod, 1, 1, 64, 16 * 4, n_heads=2)
    t.fill(0, 10, np.random.default_rng(0))
    q = torch.zeros((1, 128), device="cuda")
    n0 = t.kv.launch_count()
    with pytest.raises(KvError):
        t.kv.attend(0, q, [0], [10])  # position not in the cache
    with pytest.raises(KvError):
        t.kv.attend(1, q, [0], [5])  # layer out of range
    with pytest.raises(KvError):
        t.kv.write(0, [99], [0], torch.zeros((1, 64), device="cuda"), torch.zeros((1, 64), device="cuda"))
    assert t.kv.launch_count() == n0


CASCADE_CASES = [
    (128, 32, 8, 40, 700, 37),    # Llama-3-8B shape, group 4
    (64, 32, 4, 24, 1024, 5),     # config-1 shape, group 8
    (128, 8, 8, 16, 333, 90),     # group 1
    (64, 12, 4, 10, 200, 17),     # group 3
]


@pytest.mark.parametrize("hd,hq,hkv,n_seq,prefix,suffix", CASCADE_CASES)
@pytest.mark.parametrize("fused", [False, True])
def test_cascade_shared_prefix_matches_oracle(oracle_mod, hd, hq, hkv, n_seq, prefix, suffix, fused):
    """Sequences made with share(0, s, prefix) and their own suffixes: the
    shared blocks go through the prefix pass (one extra launch), the rest
    through the decode launch, and the merged outputs match the oracle."""
    rng = np.random.default_rng(hd + n_seq + prefix)
    per = (prefix + suffix + 16) // 16 + 2
    t = Twin(oracle_mod, 1, hkv, hd, 16 * (prefix // 16 + 2 + n_seq * per), n_heads=hq, max_seqs=n_seq + 1)
    t.fill(0, prefix, rng)
    lens = []
    for s in range(1, n_seq + 1):
        t.share(0, s, prefix)
        L = prefix + suffix + s % 7
        t.fill(s, L, rng)
        lens.append(L)
    seqs = np.arange(1, n_seq + 1)
    pos = np.array(lens)
    b, sl = t.append(seqs, pos)
    k = rng.standard_normal((n_seq, hkv * hd)).astype(np.float32)
    v = rng.standard_normal((n_seq, hkv * hd)).astype(np.float32)
    q = rng.standard_normal((n_seq, hq * hd)).astype(np.float32)
    c0 = t.kv.cascade_launches()
    if fused:
        out = t.kv.write_attend(0, b, sl, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(),
                                torch.from_numpy(q).cuda(), seqs, pos).cpu().numpy()
        t.ok.write_batch(0, b, sl, k, v)
        ref = t.ok.attend(0, q, seqs, pos, hq, hkv, hd)
    else:
        t.write(0, b, sl, k, v)
        out, ref = t.attend_both(0, seqs, pos, q)
    assert t.kv.cascade_launches() == c0 + 1
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    t.check_pool()
    t.check_tables()
    t.kv.check()


@pytest.mark.parametrize("hd,hq,hkv,cached,chunk", [(128, 32, 8, 700, 64), (64, 32, 4, 2048, 256),
                                                   (128, 8, 8, 333, 21), (128, 16, 2, 1000, 97)])
def test_cascade_prefill_chunk_matches_oracle(oracle_mod, hd, hq, hkv, cached, chunk):
    """A prefill chunk: `chunk` tokens of one sequence over `cached` cached
    positions, written first, then attended in one call.  Every token's
    blocks before its own go through the prefix pass with the token's causal
    limit (the chunk's blocks included), its own block through the decode
    launch; outputs match the oracle, and a second chunk of two sequences in
    one call (two such groups) does too."""
    rng = np.random.default_rng(hd + cached + chunk)
    per = (cached + 2 * chunk + 16) // 16 + 2
    t = Twin(oracle_mod, 1, hkv, hd, 16 * 2 * per, n_heads=hq, max_seqs=2)
    for s in range(2):
        t.fill(s, cached + s * 5, rng)
    for round_ in range(2):
        seqs, pos = [], []
        for s in range(2 if round_ else 1):
            start = t.kv.len(s)
            p = np.arange(start, start + chunk)
            t.fill(s, start + chunk, rng)  # the chunk's rows are written before the attention call
            seqs.append(np.full(chunk, s))
            pos.append(p)
        seqs, pos = np.concatenate(seqs), np.concatenate(pos)
        q = rng.standard_normal((seqs.size, hq * hd)).astype(np.float32)
        c0 = t.kv.cascade_launches()
        out, ref = t.attend_both(0, seqs, pos, q)
        assert t.kv.cascade_launches() == c0 + 1, "the prefix pass did not run"
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5, err_msg=f"round {round_}")
    t.kv.check()


def test_cascade_groups_mixed_with_private_sequences(oracle_mod):
    """Two prefix groups, one of them with a member that shares only part of
    the prefix (the group's shared run shortens to it), and sequences with no
    sharing, in one call; also the same call with the pass turned off."""
    rng = np.random.default_rng(77)
    hd, hq, hkv = 128, 16, 4
    t = Twin(oracle_mod, 1, hkv, hd, 16 * 900, n_heads=hq, max_seqs=40)
    t.fill(0, 640, rng)     # group A root
    t.fill(20, 515, rng)    # group B root
    lens = {}
    for s in range(1, 12):
        t.share(0, s, 640 if s != 5 else 300)  # seq 5 shares 300 positions only
        lens[s] = 700 + s
    for s in range(21, 32):
        t.share(20, s, 515)
        lens[s] = 530 + 3 * s
    for s in range(33, 38):
        lens[s] = 100 + 40 * s % 300  # private
    for s, L in lens.items():
        t.fill(s, L, rng)
    seqs = np.array(sorted(lens))
    pos = np.array([lens[s] - 1 for s in seqs])
    q = rng.standard_normal((seqs.size, hq * hd)).astype(np.float32)
    c0 = t.kv.cascade_launches()
    out, ref = t.attend_both(0, seqs, pos, q)
    assert t.kv.cascade_launches() == c0 + 1
    np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5)
    t.kv.set_cascade(0)
    out2, _ = t.attend_both(0, seqs, pos, q)
    assert t.kv.cascade_launches() == c0 + 1
    np.testing.assert_allclose(out2, ref, rtol=1e-4, atol=2e-5)
    t.kv.check()

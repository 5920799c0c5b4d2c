"""The Llama step on the GPU (include/lt_llama.h) against the oracle.

Per op, on identical inputs:
- QMatrix::matmul (quant.rs:405-428): bit-exact, any shape, with the
  residual add;
- QActs::quantize (quant.rs:771-795): bit-exact, including ties, zero
  blocks, NaN and infinity;
- SiLU(gate) * up + quantize (model.rs:492-494): the device rounds exp
  correctly to f32, while the C library's expf that the reference calls is
  off by one ulp on ~0.03 % of inputs; so SiLU equals a correctly-rounded-exp
  restatement everywhere and the oracle within 2 ulps (the divide and the
  multiply can carry one ulp of exp into two), and its quantization is
  bit-exact;
- greedy argmax (sampling.rs:161-163): equal, ties and NaN included;
- rms_norm (model.rs:174-183): within 1e-5 relative (a tree sum of squares
  instead of the reference's sequential one, which is the less exact of the
  two), and its quantization bit-exact on the device's own output.
End to end: the C1 model's forward on the GPU (previous tokens forced to the
all-oracle run's) stays within the oracle's own noise floor (see
test_gpu_c1.py), and its cache bookkeeping equals the oracle's, bit-exact.
"""
import numpy as np
import pytest
import torch

from langtrain_studio_b200 import llama as LL
from oracle import model as M

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _ulps(a, b):
    ai = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    bi = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


def _special_rows(rng, n, cols):
    x = (rng.standard_normal((n, cols)) * rng.choice([1e-3, 1.0, 50.0], (n, 1))).astype(np.float32)
    x[0, :32] = 0.0                                    # zero block: d = 0
    x[0, 32:64] = np.arange(32) - 15.5                 # amax 16.5 -> exact .5 products
    if cols >= 96:
        x[0, 64:96] = np.float32(127.0)                # id = 1
        x[0, 70] = 0.5
        x[0, 71] = -2.5                                # ties away from zero
    if cols >= 160:
        x[0, 96] = np.nan                              # NaN: ignored by amax, quantizes to 0
        x[0, 128] = np.inf                             # inf amax: id = 0
        x[0, 129] = -1e-42                             # subnormal
    return x


@pytest.mark.parametrize("cols", [64, 256, 2048])
def test_quantize_bit_exact(cols):
    rng = np.random.default_rng(cols)
    x = _special_rows(rng, 9, cols)
    qs, sc = LL.q8_quantize(_cuda(x))
    qo, so = M.quantize(x)
    assert np.array_equal(qs.cpu().numpy(), qo)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), so.view(np.uint32))


@pytest.mark.parametrize("rows,cols,n", [(16, 32, 1), (40, 256, 3), (2560, 2048, 4), (48, 5632, 13),
                                         (2048, 2048, 8), (33, 2048, 17)])
def test_q8_matmul_bit_exact(rows, cols, n):
    rng = np.random.default_rng(rows * 7 + n)
    wq = rng.integers(-128, 128, (rows, cols), dtype=np.int8)
    ws = (rng.random((rows, cols // 32)) * 0.01).astype(np.float16)
    ws[0, 0] = np.float16(0.0)
    x = _special_rows(rng, n, cols) if cols >= 160 else rng.standard_normal((n, cols)).astype(np.float32)
    x = np.nan_to_num(x, nan=0.0, posinf=1.0)
    xq, xs = M.quantize(x)
    ref = M.matmul_q8(wq, ws.astype(np.float32), xq, xs)
    out = LL.q8_matmul(_cuda(wq), _cuda(ws.view(np.uint16)), _cuda(xq), _cuda(xs))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), np.argwhere(got != ref)[:5]
    # residual add: x += W . x_q (model.rs:478-481)
    base = rng.standard_normal((n, rows)).astype(np.float32)
    acc = _cuda(base)
    LL.q8_matmul(_cuda(wq), _cuda(ws.view(np.uint16)), _cuda(xq), _cuda(xs), out=acc, accumulate=True)
    assert np.array_equal(acc.cpu().numpy().view(np.uint32), (base + ref).view(np.uint32))


def _silu_cr(g, u):
    """SiLU with a correctly rounded f32 exp (the double-precision exp rounded once)."""
    with np.errstate(over="ignore"):
        e = np.exp(-g.astype(np.float64)).astype(np.float32)
        return (g / (np.float32(1.0) + e)) * u


@pytest.mark.parametrize("ffn,n", [(512, 1), (5632, 4), (5632, 7)])
def test_silu_quantize(ffn, n):
    rng = np.random.default_rng(ffn + n)
    g = (rng.standard_normal((n, ffn)) * 4).astype(np.float32)
    u = rng.standard_normal((n, ffn)).astype(np.float32)
    g[0, :8] = [-100.0, -88.0, -87.0, 0.0, -0.0, 88.0, 1e-30, -1e-30]
    h, qs, sc = LL.silu_q8(_cuda(np.concatenate([g, u], axis=1)), ffn)
    h = h.cpu().numpy()
    assert np.array_equal(h.view(np.uint32), _silu_cr(g, u).view(np.uint32))
    ho = M.silu_mul(g, u)
    d = _ulps(h, ho)
    assert d.max() <= 2 and (d > 0).mean() < 1e-3, (d.max(), (d > 0).sum())
    qo, so = M.quantize(h)  # the quantizer on the device's own SiLU output: bit-exact
    assert np.array_equal(qs.cpu().numpy(), qo)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), so.view(np.uint32))


def test_silu_exp_over_a_million_values():
    rng = np.random.default_rng(11)
    g = np.concatenate([rng.uniform(-90, 90, 1 << 19), rng.standard_normal(1 << 19) * 3]).astype(np.float32)
    g = g.reshape(-1, 1024)
    u = np.ones_like(g)
    h, _, _ = LL.silu_q8(_cuda(np.concatenate([g, u], axis=1)), 1024)
    h = h.cpu().numpy()
    assert np.array_equal(h.view(np.uint32), _silu_cr(g, u).view(np.uint32))
    d = _ulps(h, M.silu_mul(g, u))
    print(f"SiLU vs libm expf: {(d > 0).sum()} of {d.size} values apart, at most {d.max()} ulps")
    assert d.max() <= 2 and (d > 0).mean() < 1e-3


def test_argmax_matches_total_order_last_max():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6, 32000)).astype(np.float32)
    x[1, [5, 900, 31999]] = 50.0              # ties: the last one wins
    x[2, 17] = np.nan                         # positive NaN is the largest under total_cmp
    x[3, :] = -0.0
    x[3, 100] = 0.0                           # +0 > -0
    x[4, :] = -np.inf
    x[5, 7] = np.inf
    got = LL.argmax_rows(_cuda(x)).cpu().numpy()
    assert np.array_equal(got, M.argmax(x))


@pytest.mark.parametrize("dim,n", [(256, 3), (2048, 4)])
def test_rms_norm_quantize_within_ulps(dim, n):
    rng = np.random.default_rng(dim)
    x = (rng.standard_normal((n + 2, dim)) * 3).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(dim)).astype(np.float32)
    rows = np.array([n + 1, 0, 2][: n], np.int32) if n <= 3 else None
    idx = None if rows is None else _cuda(rows)
    normed, qs, sc = LL.rms_norm_q8(_cuda(x if rows is not None else x[:n]), _cuda(w), 1e-5, rows_idx=idx)
    src = x[rows] if rows is not None else x[:n]
    ref = M.rms_norm(src, w, 1e-5)
    got = normed.cpu().numpy()
    # The reference sums the squares sequentially (rounding error up to
    # ~dim * 2^-24 relative); the device sums a tree.  Both sit within 1e-5
    # of the float64 value, the device no farther than the reference.
    s64 = src.astype(np.float64)
    exact = s64 / np.sqrt((s64 * s64).mean(axis=1, keepdims=True) + 1e-5) * w.astype(np.float64)
    e_gpu = np.abs(got - exact) / np.abs(exact).max()
    e_ref = np.abs(ref - exact) / np.abs(exact).max()
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
    assert e_gpu.max() <= e_ref.max() + 2 ** -23
    qo, so = M.quantize(normed.cpu().numpy())  # quantizer on the GPU's own normed rows: bit-exact
    assert np.array_equal(qs.cpu().numpy(), qo)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), so.view(np.uint32))


@pytest.mark.parametrize("pro,rows,cols,n", [(LL.PRO_QUANT, 2048, 2048, 4), (LL.PRO_QUANT, 40, 256, 1),
                                             (LL.PRO_SILU, 2048, 5632, 4), (LL.PRO_SILU, 33, 512, 8),
                                             (LL.PRO_RMSNORM, 2560, 2048, 4), (LL.PRO_RMSNORM, 1000, 2048, 3),
                                             (LL.PRO_RMSNORM, 64, 256, 8), (LL.PRO_QUANT, 2048, 2048, 12)])
def test_fused_projection_equals_two_launches(pro, rows, cols, n):
    """The decode path (prologue fused into the matmul launch) gives the bits
    of the standalone prologue kernel followed by the matmul."""
    rng = np.random.default_rng(rows + cols + n + pro)
    wq = _cuda(rng.integers(-128, 128, (rows, cols), dtype=np.int8))
    ws = _cuda((rng.random((rows, cols // 32)) * 0.01).astype(np.float16).view(np.uint16))
    width = 2 * cols if pro == LL.PRO_SILU else cols
    x = _cuda((rng.standard_normal((n + 3, width)) * 2).astype(np.float32))
    idx = gamma = None
    if pro == LL.PRO_RMSNORM:
        gamma = _cuda((1 + 0.1 * rng.standard_normal(cols)).astype(np.float32))
        idx = _cuda(rng.permutation(n + 3)[:n].astype(np.int32))
    else:
        x = x[:n].contiguous()
    base = rng.standard_normal((n, rows)).astype(np.float32)
    outs = []
    for fused in (True, False):
        for acc in (False, True):
            o = _cuda(base) if acc else None
            outs.append(LL.q8_project(pro, wq, ws, x, rows_idx=idx, gamma=gamma, out=o, accumulate=acc,
                                      fused=fused).cpu().numpy())
    LL.q8_check()
    assert np.array_equal(outs[0].view(np.uint32), outs[2].view(np.uint32))
    assert np.array_equal(outs[1].view(np.uint32), outs[3].view(np.uint32))
    assert np.array_equal(outs[1].view(np.uint32), (base + outs[0]).view(np.uint32))


TINY = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=1000)


def _gpu_model(om, max_batch=256):
    m = LL.Llama(om.n_layers, om.dim, om.n_heads, om.n_kv_heads, om.head_dim, om.ffn_dim, om.vocab,
                 max_batch=max_batch)
    m.load(om.export_tensor)
    return m


def test_tiny_forward_close_to_oracle():
    om = M.OracleModel(**TINY, seed=1)
    gm = _gpu_model(om)
    prompts = M.c1_prompts(om.vocab, 2, 48, 32, seed=2)
    okv = om.oracle_kv(512, 4)
    ref = np.zeros((2, 6, om.vocab), np.float32)
    toks = M.run_c1(om, okv, okv.share, prompts, 32, 6, logits_out=ref)
    kv = gm.kv_cache(512, 4)
    got = np.zeros_like(ref)
    LL.serve_shared_prefix(gm, kv, prompts, 32, 6, teacher=toks, logits_out=got)
    d = np.abs(got - ref).max()
    assert d < 0.05 * ref.std(), (d, ref.std())
    for s in range(4):
        assert np.array_equal(kv.seq_blocks(s), okv.seq_blocks(s))
    assert np.array_equal(kv.free_list(), okv.free_list())
    assert np.array_equal(kv.refs(), okv.refs())


def test_forward_rejects_bad_input_after_claim():
    om = M.OracleModel(**TINY, seed=1)
    gm = _gpu_model(om)
    kv = gm.kv_cache(64, 2)
    with pytest.raises(LL.LlamaError):
        gm.forward(kv, [5, om.vocab], [0, 0], [0, 1], [1])   # token id out of range (model.rs:521-523)
    assert kv.len(0) == 2                                     # cells claimed first, as the reference does
    with pytest.raises(Exception):
        gm.forward(kv, [1], [0], [7], [0])                    # non-contiguous position
    wrong = LL.KvCache(1, 2, 64, 64, n_heads=4, max_seqs=2)
    with pytest.raises(LL.LlamaError):
        gm.forward(wrong, [1], [0], [0], [0])                 # cache shape differs from the model


@pytest.fixture(scope="module")
def c1():
    om = M.OracleModel(**M.C1_SHAPE, seed=0)
    prompts = M.c1_prompts(om.vocab)
    okv = om.oracle_kv(1024, 4)
    logits = np.zeros((4, 64, om.vocab), np.float32)
    ref = M.run_c1(om, okv, okv.share, prompts, 64, 64, logits_out=logits)
    return om, prompts, ref, logits, okv


def test_c1_gpu_forward_within_noise_floor(c1):
    om, prompts, ref, logits, okv = c1
    floor_kv = om.oracle_kv(1024, 4)
    lf = np.zeros_like(logits)

    class Perturbed:  # oracle attention with a relative N(0, 1e-6) error: the noise floor
        rng = np.random.default_rng(1)

        def append(self, seqs, pos):
            rc, done, b, s = floor_kv.append_batch(seqs, pos)
            assert rc == 0
            return b, s

        def write(self, layer, b, s, k, v):
            floor_kv.write_batch(layer, b, s, k, v)

        def attend(self, layer, q, seqs, pos):
            o = floor_kv.attend(layer, q, seqs, pos, om.n_heads, om.n_kv_heads, om.head_dim)
            return o * (1 + 1e-6 * self.rng.standard_normal(o.shape)).astype(np.float32)

    pf = M.run_c1(om, M.PyKv(Perturbed(), om.kv_dim, om.q_dim), floor_kv.share, prompts, 64, 64, teacher=ref,
                  logits_out=lf)
    gm = _gpu_model(om)
    kv = gm.kv_cache(1024, 4)
    lg = np.zeros_like(logits)
    pg = LL.serve_shared_prefix(gm, kv, prompts, 64, 64, teacher=ref, logits_out=lg)
    d_floor, d_gpu = np.abs(lf - logits).max(), np.abs(lg - logits).max()
    n_floor, n_gpu = int((pf != ref).sum()), int((pg != ref).sum())
    print(f"C1 GPU forward: max |dlogit| {d_gpu:.4f} (floor {d_floor:.4f}), picks differing {n_gpu}/{ref.size} "
          f"(floor {n_floor})")
    assert d_gpu <= 2.0 * d_floor
    assert n_gpu <= 2 * n_floor + 4
    for s in range(4):
        assert np.array_equal(kv.seq_blocks(s), okv.seq_blocks(s))
    assert np.array_equal(kv.free_list(), okv.free_list())
    assert np.array_equal(kv.refs(), okv.refs())


def test_c1_gpu_greedy_free_running(c1):
    """The device-only greedy loop (lt_llama_step_greedy): the picks before the
    first near-tie of the reference's logits are the reference's."""
    om, prompts, ref, logits, _ = c1
    gm = _gpu_model(om)
    kv = gm.kv_cache(1024, 4)
    got = LL.serve_shared_prefix(gm, kv, prompts, 64, 64)
    mg = M.top2_margin(logits)
    for s in range(4):
        first_tie = int(np.argmax(mg[s] < 0.4)) if (mg[s] < 0.4).any() else 64
        assert np.array_equal(got[s, :first_tie], ref[s, :first_tie]), (s, first_tie)

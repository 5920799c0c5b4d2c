"""The persistent decode step of lt_llama_forward against the multi-launch path.

A forward of up to 8 tokens, one per sequence, runs as one cooperative
launch (langtrain_studio_b200/csrc/lt_llama_decode.cu).  Its matmuls (the
reference's row_dot order, quant.rs:418-421), norms, quantiser, RoPE and K/V
append are the multi-launch path's arithmetic, so:

- when attention is exact (every token at position 0: softmax over one
  position is 1, the output is the cached V row) the two paths give
  bit-identical logits and pools;
- otherwise the K/V rows appended at layer 0 are bit-identical (they depend
  only on the embeddings) and the logits agree within the noise that int8
  re-quantisation puts on a last-bit attention difference (the bar the
  oracle comparison of tests/test_gpu_llama.py uses).

The step also picks the greedy token in the same launch; that pick equals the
argmax of the logits it computes.  The C1 tests of tests/test_gpu_llama.py and
tests/test_gpu_c1.py run their decode steps through this kernel too.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from langtrain_studio_b200 import llama as LL  # noqa: E402
from oracle import model as M  # noqa: E402

pytestmark = pytest.mark.gpu

TINY = dict(dim=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, ffn_dim=512, vocab=1000)
C1_3L = dict(M.C1_SHAPE, n_layers=3)  # the C1 shape, three layers


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _pair(shape, seed, n_tokens=1024, max_seqs=8):
    """Two handles with the same weights: persistent step on / off."""
    om = M.OracleModel(**shape, seed=seed)
    out = []
    for persistent in (True, False):
        gm = LL.Llama(om.n_layers, om.dim, om.n_heads, om.n_kv_heads, om.head_dim, om.ffn_dim, om.vocab,
                      max_batch=256)
        gm.load(om.export_tensor)
        gm.set_persistent(persistent)
        out.append((gm, gm.kv_cache(n_tokens, max_seqs)))
    assert out[0][0].persistent_available(), "the persistent step should take this shape"
    return om, out


def _pool(kv, layer):
    torch.cuda.synchronize()
    return kv.read_pool(layer)


@pytest.mark.parametrize("shape", ["tiny", "c1_3l"])
def test_first_tokens_bit_identical(shape):
    """Four new sequences, first token each: attention is exact on both paths."""
    om, ((gp, kp), (gm, km)) = _pair(TINY if shape == "tiny" else C1_3L, seed=3)
    rng = np.random.default_rng(4)
    tokens = rng.integers(0, om.vocab, 4)
    seqs, pos = np.arange(4), np.zeros(4)
    l0 = gp.launch_count()
    a = gp.forward(kp, tokens, seqs, pos, np.arange(4)).cpu().numpy()
    assert gp.launch_count() - l0 == 1, "one launch for the whole step"
    b = gm.forward(km, tokens, seqs, pos, np.arange(4)).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    for layer in range(om.n_layers):
        assert np.array_equal(_pool(kp, layer), _pool(km, layer)), f"pool differs in layer {layer}"


def test_decode_steps_match_multi_launch_path():
    """Prefill (multi-launch, more than 8 tokens), then teacher-forced decode
    steps of 4 sequences sharing a 32-token prefix on both paths."""
    om, ((gp, kp), (gm, km)) = _pair(TINY, seed=1, n_tokens=2048)
    prompts = M.c1_prompts(om.vocab, 4, 48, 32, seed=2)
    teacher = np.random.default_rng(5).integers(0, om.vocab, (4, 8))
    outs = []
    for g, kv in ((gp, kp), (gm, km)):
        lg = np.zeros((4, 8, om.vocab), np.float32)
        LL.serve_shared_prefix(g, kv, prompts, 32, 8, teacher=teacher, logits_out=lg)
        outs.append(lg)
    d = np.abs(outs[0] - outs[1]).max()
    assert d < 0.05 * outs[1].std(), (d, outs[1].std())
    # layer 0's appended rows depend only on the embeddings: bit-identical
    assert np.array_equal(_pool(kp, 0), _pool(km, 0))
    for s in range(4):
        assert np.array_equal(kp.seq_blocks(s), km.seq_blocks(s))
    assert np.array_equal(kp.free_list(), km.free_list())


def test_long_contexts_match_multi_launch_path():
    """Contexts of up to 700 positions: a (token, KV head)'s 44 blocks are
    dealt over the 16 warps of one CTA (up to three each) and merged in
    shared memory; the short ones leave warps without blocks."""
    om, ((gp, kp), (gm, km)) = _pair(TINY, seed=9, n_tokens=4096)
    rng = np.random.default_rng(10)
    lens = [700, 33, 512, 129]
    prompts = [rng.integers(0, om.vocab, L) for L in lens]
    for g, kv in ((gp, kp), (gm, km)):
        for s, L in enumerate(lens):  # prefill in chunks of up to 200 tokens (multi-launch: one sequence, > 8 tokens)
            for p0 in range(0, L, 200):
                p1 = min(L, p0 + 200)
                g.forward(kv, prompts[s][p0:p1], np.full(p1 - p0, s), np.arange(p0, p1), [p1 - p0 - 1])
    outs = []
    for g, kv in ((gp, kp), (gm, km)):
        r2 = np.random.default_rng(12)
        lg = []
        for step in range(3):
            tok = r2.integers(0, om.vocab, 4)
            lg.append(g.forward(kv, tok, np.arange(4), np.array(lens) + step, np.arange(4)).cpu().numpy())
        outs.append(np.stack(lg))
    d = np.abs(outs[0] - outs[1]).max()
    assert d < 0.05 * outs[1].std(), (d, outs[1].std())
    assert np.array_equal(_pool(kp, 0), _pool(km, 0))


def test_in_kernel_greedy_pick_is_the_argmax_of_the_logits():
    om, ((g1, k1), _) = _pair(TINY, seed=6)
    g2 = LL.Llama(om.n_layers, om.dim, om.n_heads, om.n_kv_heads, om.head_dim, om.ffn_dim, om.vocab, max_batch=256)
    g2.load(om.export_tensor)
    k2 = g2.kv_cache(1024, 8)
    rng = np.random.default_rng(7)
    cur = rng.integers(0, om.vocab, 6)
    seqs = np.arange(6)
    for step in range(5):
        pos = np.full(6, step)
        picks = g1.step_greedy(k1, cur, seqs, pos, np.arange(6))          # pick inside the persistent launch
        lg = g2.forward(k2, cur, seqs, pos, np.arange(6))                  # the same step, logits out
        ref = LL.argmax_rows(lg).cpu().numpy()
        assert np.array_equal(picks, ref), step
        cur = picks


def test_batches_the_persistent_step_does_not_take_fall_back():
    """Two tokens of one sequence, or more than 8 tokens, take the multi-launch
    path (one launch per kernel)."""
    om, ((gp, kp), _) = _pair(TINY, seed=8)
    l0 = gp.launch_count()
    gp.forward(kp, [1, 2], [0, 0], [0, 1], [1])
    assert gp.launch_count() - l0 > 1
    l0 = gp.launch_count()
    gp.forward(kp, np.arange(9), np.arange(1, 8).tolist() + [1, 2], [0] * 7 + [1, 1], [0])
    assert gp.launch_count() - l0 > 1
    assert kp.len(0) == 2 and kp.len(1) == 2 and kp.len(7) == 1

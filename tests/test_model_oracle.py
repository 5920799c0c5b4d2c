"""CPU tests of the C1 end-to-end forward (oracle/lt_model.c).

The forward restates model.rs:366-518 over Q8_0 weights; the reference is
Rust and not built here, so these tests pin the properties the reference's
design guarantees instead (quant.rs:405-407: "a request's output never
depends on how many other requests share the batch"):
- batch invariance: logits of a token are bit-identical whether it runs
  alone or inside a batch;
- prefix sharing is transparent: share(0, s, 64) + suffix prefill gives the
  same logits as prefilling the whole prompt;
- the callback adapter the GPU test uses returns exactly what the direct
  oracle adapter does.
"""
import numpy as np
import pytest

from oracle import model as M
from oracle import oracle as O

TINY = dict(dim=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=32, ffn_dim=512, vocab=1000)


@pytest.fixture(scope="module")
def tiny():
    return M.OracleModel(**TINY, seed=0)


class _OracleViaCallbacks:
    def __init__(self, m, n_tokens, max_seqs):
        self.kv = m.oracle_kv(n_tokens, max_seqs)
        self.m = m

    def append(self, seqs, pos):
        rc, done, b, s = self.kv.append_batch(seqs, pos)
        if rc:
            raise O.OracleError(rc, "append")
        return b, s

    def write(self, layer, b, s, k, v):
        self.kv.write_batch(layer, b, s, k, v)

    def attend(self, layer, q, seqs, pos):
        return self.kv.attend(layer, q, seqs, pos, self.m.n_heads, self.m.n_kv_heads, self.m.head_dim)


def test_batch_invariance(tiny):
    pr = M.c1_prompts(tiny.vocab, 1, 40, 0, seed=3)[0]
    full = tiny.forward(tiny.oracle_kv(256, 2), pr, np.zeros(40), np.arange(40), np.arange(40))
    kv = tiny.oracle_kv(256, 2)
    rows = np.stack([tiny.forward(kv, pr[i:i + 1], [0], [i], [0])[0] for i in range(40)])
    assert np.array_equal(full, rows)
    assert np.isfinite(full).all() and np.abs(full).max() > 0


def test_shared_prefix_equals_full_prefill(tiny):
    pr = M.c1_prompts(tiny.vocab, 2, 48, 32, seed=5)
    kv = tiny.oracle_kv(512, 4)
    tiny.forward(kv, pr[0], np.zeros(48), np.arange(48), [47])
    kv.share(0, 1, 32)
    got = tiny.forward(kv, pr[1, 32:], np.ones(16), np.arange(32, 48), [15])
    ref = tiny.forward(tiny.oracle_kv(512, 4), pr[1], np.zeros(48), np.arange(48), [47])
    assert np.array_equal(got, ref)


def test_callback_adapter_matches_direct(tiny):
    pr = M.c1_prompts(tiny.vocab, 4, 48, 32, seed=0)
    kv = tiny.oracle_kv(1024, 4)
    ref = M.run_c1(tiny, kv, kv.share, pr, 32, 6)
    cb = _OracleViaCallbacks(tiny, 1024, 4)
    got = M.run_c1(tiny, M.PyKv(cb, tiny.kv_dim, tiny.q_dim), cb.kv.share, pr, 32, 6)
    assert np.array_equal(got, ref)
    ko, vo = kv.pool()
    k2, v2 = cb.kv.pool()
    assert np.array_equal(ko, k2) and np.array_equal(vo, v2)


def test_full_cache_surfaces_as_error(tiny):
    kv = tiny.oracle_kv(32, 2)  # two blocks: a 40-token prompt does not fit
    pr = M.c1_prompts(tiny.vocab, 1, 40, 0)[0]
    with pytest.raises(O.OracleError):
        tiny.forward(kv, pr, np.zeros(40), np.arange(40), [39])
    cb = _OracleViaCallbacks(tiny, 32, 2)
    with pytest.raises(O.OracleError):
        tiny.forward(M.PyKv(cb, tiny.kv_dim, tiny.q_dim), pr, np.zeros(40), np.arange(40), [39])


def test_argmax_takes_last_of_equal_maxima(tiny):
    """sampling.rs:161-163: max_by(total_cmp) keeps the last maximum."""
    x = np.array([[1.0, 3.0, 3.0, -1.0], [np.nan, 2.0, 1.0, 2.0], [-0.0, 0.0, -1.0, 0.0]], np.float32)
    assert list(tiny.argmax(x)) == [2, 0, 3]

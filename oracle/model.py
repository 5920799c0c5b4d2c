"""TEST INFRASTRUCTURE ONLY: the C1 end-to-end workload.

``OracleModel`` drives ``oracle/lt_model.c``, the CPU restatement of the
reference engine's Llama forward pass (``engine/crates/native/src/model.rs:366-518``)
over Q8_0 weights (``engine/crates/native/src/quant.rs``).  The KV cache under
the forward is pluggable: the oracle's own KvCache, or any Python object with
``append``/``write``/``attend`` (the GPU cache through the C ABI, in the GPU
tests).  ``run_c1`` is BASELINE configs[0]: 4 sequences of 128 prompt tokens
whose first 64 are shared (seq 0 prefilled, then ``share(0, s, 64)``), greedy
decode.  Only tests/ use this module.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import oracle as O

_u32p, _i32p, _f32p = C.POINTER(C.c_uint32), C.POINTER(C.c_int32), C.POINTER(C.c_float)
APPEND_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, _u32p, _u32p, C.c_uint32, _i32p, _i32p)
WRITE_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, _i32p, _i32p, C.c_uint32, _f32p, _f32p)
ATTEND_FN = C.CFUNCTYPE(None, C.c_void_p, C.c_uint32, _f32p, _u32p, _u32p, C.c_uint32, _f32p)


class _OmKv(C.Structure):
    _fields_ = [("ctx", C.c_void_p), ("append", APPEND_FN), ("write", WRITE_FN), ("attend", ATTEND_FN)]


# Llama-1.1B-style shape of BASELINE configs[0].
C1_SHAPE = dict(dim=2048, n_layers=22, n_heads=32, n_kv_heads=4, head_dim=64, ffn_dim=5632, vocab=32000)


def _lib():
    L = O.lib()
    if not getattr(L, "_om_ready", False):
        p = C.c_void_p
        L.om_new_random.restype = p
        L.om_new_random.argtypes = [C.c_int] * 7 + [C.c_uint64]
        L.om_delete.argtypes = [p]
        L.om_forward.restype = C.c_int
        L.om_forward.argtypes = [p, p, p, p, p, C.c_uint32, p, C.c_uint32, p, C.c_int]
        L.om_argmax.restype = C.c_int32
        L.om_argmax.argtypes = [p, C.c_int]
        L.om_kv_oracle.restype = p
        L.om_kv_oracle.argtypes = [p, C.c_int, C.c_int, C.c_int, C.c_int]
        L.om_kv_free.argtypes = [p]
        L.om_export_tensor.restype = C.c_size_t
        L.om_export_tensor.argtypes = [p, C.c_int, C.c_int, p]
        L.om_quantize.argtypes = [p, C.c_uint32, C.c_uint32, p, p]
        L.om_matmul_q8.argtypes = [p, p, C.c_uint32, C.c_uint32, p, p, C.c_uint32, p, C.c_int]
        L.om_rms_norm.argtypes = [p, p, C.c_uint32, C.c_uint32, C.c_float, p]
        L.om_silu_mul.argtypes = [p, p, C.c_size_t]
        L._om_ready = True
    return L


def _view(ptr, n, dtype):
    return np.ctypeslib.as_array(ptr, shape=(n,)).view(dtype) if n else np.zeros(0, dtype)


class PyKv:
    """Adapts a Python KV object to the C forward's om_kv callbacks.

    The object provides ``append(seqs, pos) -> (blocks, slots)`` (raising on
    a full cache), ``write(layer, blocks, slots, k, v)`` with f32 arrays
    [n, kv_dim] and ``attend(layer, q, seqs, pos) -> out`` f32 [n, q_dim].
    An exception inside a callback is kept and re-raised after the forward.
    """

    def __init__(self, obj, kv_dim: int, q_dim: int):
        self.obj, self.kv_dim, self.q_dim = obj, kv_dim, q_dim
        self.error: BaseException | None = None
        self._cb = (APPEND_FN(self._append), WRITE_FN(self._write), ATTEND_FN(self._attend))
        self.struct = _OmKv(None, *self._cb)

    def _append(self, ctx, seq, pos, n, block, slot):
        try:
            b, s = self.obj.append(_view(seq, n, np.uint32).copy(), _view(pos, n, np.uint32).copy())
            _view(block, n, np.int32)[:] = b
            _view(slot, n, np.int32)[:] = s
            return 0
        except BaseException as e:  # noqa: BLE001 -- surfaced after the forward
            self.error = self.error or e
            return 1

    def _write(self, ctx, layer, block, slot, n, k, v):
        if self.error:
            return
        try:
            m = n * self.kv_dim
            self.obj.write(layer, _view(block, n, np.int32).copy(), _view(slot, n, np.int32).copy(),
                           _view(k, m, np.float32).reshape(n, self.kv_dim).copy(),
                           _view(v, m, np.float32).reshape(n, self.kv_dim).copy())
        except BaseException as e:  # noqa: BLE001
            self.error = e

    def _attend(self, ctx, layer, q, seq, pos, n, out):
        if self.error:
            return
        try:
            m = n * self.q_dim
            res = self.obj.attend(layer, _view(q, m, np.float32).reshape(n, self.q_dim).copy(),
                                  _view(seq, n, np.uint32).copy(), _view(pos, n, np.uint32).copy())
            _view(out, m, np.float32)[:] = np.asarray(res, dtype=np.float32).reshape(-1)
        except BaseException as e:  # noqa: BLE001
            self.error = e


class OracleModel:
    """Random-init Q8_0 Llama (seeded), forward restated from model.rs."""

    def __init__(self, dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, seed=0):
        self._L = _lib()
        self._h = self._L.om_new_random(dim, n_layers, n_heads, n_kv_heads, head_dim, ffn_dim, vocab, seed)
        if not self._h:
            raise MemoryError("om_new_random failed")
        self.dim, self.n_layers, self.n_heads, self.n_kv_heads = dim, n_layers, n_heads, n_kv_heads
        self.head_dim, self.ffn_dim, self.vocab = head_dim, ffn_dim, vocab
        self.kv_dim, self.q_dim = n_kv_heads * head_dim, n_heads * head_dim

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._L.om_delete(h)
            self._h = None

    def oracle_kv(self, n_tokens: int, max_seqs: int) -> O.OracleKv:
        return O.OracleKv(self.n_layers, self.kv_dim, n_tokens, max_seqs=max_seqs)

    def forward(self, kv, tokens, seqs, pos, want, n_threads: int = 0) -> np.ndarray:
        """Model::forward over `kv` (an OracleKv or a PyKv); logits [len(want), vocab]."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        seqs = np.ascontiguousarray(seqs, np.uint32)
        pos = np.ascontiguousarray(pos, np.uint32)
        want = np.ascontiguousarray(want, np.uint32)
        logits = np.zeros((max(want.size, 1), self.vocab), np.float32)
        if isinstance(kv, O.OracleKv):
            w = self._L.om_kv_oracle(kv._h, self.n_heads, self.n_kv_heads, self.head_dim, n_threads)
            try:
                rc = self._L.om_forward(self._h, w, O._ptr(tokens), O._ptr(seqs), O._ptr(pos), tokens.size,
                                        O._ptr(want), want.size, O._ptr(logits), n_threads)
            finally:
                self._L.om_kv_free(w)
        else:
            kv.error = None
            rc = self._L.om_forward(self._h, C.byref(kv.struct), O._ptr(tokens), O._ptr(seqs), O._ptr(pos),
                                    tokens.size, O._ptr(want), want.size, O._ptr(logits), n_threads)
            if kv.error is not None:
                raise kv.error
        if rc:
            raise O.OracleError(rc, f"KV append failed with status {rc}")
        return logits[: want.size]

    def export_tensor(self, which: int, layer: int) -> bytes:
        """One tensor in its GGUF encoding (Q8_0 blocks or F32)."""
        n = self._L.om_export_tensor(self._h, which, layer, None)
        if n == 0:
            raise ValueError(f"no tensor {which} in layer {layer}")
        buf = np.zeros(n, np.uint8)
        self._L.om_export_tensor(self._h, which, layer, O._ptr(buf))
        return buf.tobytes()

    def argmax(self, logits: np.ndarray) -> np.ndarray:
        logits = np.ascontiguousarray(logits, np.float32)
        return np.array([self._L.om_argmax(O._ptr(row), row.size) for row in logits], np.int32)


# ---- op-level restatements (per-op parity checks) ----

def quantize(x: np.ndarray):
    """QActs::quantize (quant.rs:771-795): x f32 [n, cols] -> (qs int8, scales f32)."""
    x = np.ascontiguousarray(x, np.float32)
    n, cols = x.shape
    qs = np.zeros((n, cols), np.int8)
    sc = np.zeros((n, cols // 32), np.float32)
    _lib().om_quantize(O._ptr(x), n, cols, O._ptr(qs), O._ptr(sc))
    return qs, sc


def matmul_q8(wq: np.ndarray, ws: np.ndarray, xq: np.ndarray, xs: np.ndarray, n_threads: int = 0) -> np.ndarray:
    """QMatrix::matmul (quant.rs:405-428, 492-533): out [n, rows]."""
    wq, xq = np.ascontiguousarray(wq, np.int8), np.ascontiguousarray(xq, np.int8)
    ws, xs = np.ascontiguousarray(ws, np.float32), np.ascontiguousarray(xs, np.float32)
    rows, cols = wq.shape
    n = xq.shape[0]
    out = np.zeros((n, rows), np.float32)
    _lib().om_matmul_q8(O._ptr(wq), O._ptr(ws), rows, cols, O._ptr(xq), O._ptr(xs), n, O._ptr(out), n_threads)
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """rms_norm (model.rs:174-183)."""
    x, w = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    _lib().om_rms_norm(O._ptr(x), O._ptr(w), x.shape[1], x.shape[0], eps, O._ptr(out))
    return out


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """g / (1 + exp(-g)) * u (model.rs:492-494)."""
    g = np.array(g, np.float32, copy=True, order="C")
    u = np.ascontiguousarray(u, np.float32)
    _lib().om_silu_mul(O._ptr(g), O._ptr(u), g.size)
    return g


def argmax(x: np.ndarray) -> np.ndarray:
    """Greedy pick per row (sampling.rs:161-163)."""
    x = np.ascontiguousarray(x, np.float32)
    return np.array([_lib().om_argmax(O._ptr(r), r.size) for r in x], np.int32)


def c1_prompts(vocab: int, n_seqs: int = 4, prompt: int = 128, shared: int = 64, seed: int = 0) -> np.ndarray:
    """n_seqs uniform-random prompts whose first `shared` tokens are common."""
    rng = np.random.default_rng(seed)
    common = rng.integers(0, vocab, shared)
    return np.stack([np.concatenate([common, rng.integers(0, vocab, prompt - shared)]) for _ in range(n_seqs)]
                    ).astype(np.int32)


def run_c1(model: OracleModel, kv, share, prompts: np.ndarray, shared: int, n_gen: int, n_threads: int = 0,
           teacher: np.ndarray | None = None, logits_out: np.ndarray | None = None):
    """The C1 serving sequence: prefill seq 0, share its first `shared`
    positions into every other sequence (kv.rs:172-183), prefill their
    suffixes in one batch, then greedy decode with every sequence in each
    step.  `share(src, dst, n)` acts on the cache under `kv`.  Returns the
    generated ids [n_seqs, n_gen].

    With `teacher` [n_seqs, n_gen], step j feeds teacher[:, j-1] instead of
    the model's own previous pick (teacher forcing), so two runs whose
    numerics differ slightly still see the same inputs.  `logits_out`
    [n_seqs, n_gen, vocab] receives the logits of every pick."""
    n_seqs, plen = prompts.shape
    gen = np.zeros((n_seqs, n_gen), np.int32)

    def pick(lg, rows, j):
        if logits_out is not None:
            logits_out[rows, j] = lg
        gen[rows, j] = model.argmax(lg)

    lg = model.forward(kv, prompts[0], np.zeros(plen, np.uint32), np.arange(plen), [plen - 1], n_threads)
    pick(lg, [0], 0)
    for s in range(1, n_seqs):
        share(0, s, shared)
    m = plen - shared
    toks = prompts[1:, shared:].reshape(-1)
    seqs = np.repeat(np.arange(1, n_seqs), m)
    pos = np.tile(np.arange(shared, plen), n_seqs - 1)
    lg = model.forward(kv, toks, seqs, pos, [(i + 1) * m - 1 for i in range(n_seqs - 1)], n_threads)
    pick(lg, list(range(1, n_seqs)), 0)
    for j in range(1, n_gen):
        p = np.full(n_seqs, plen + j - 1, np.uint32)
        feed = gen[:, j - 1] if teacher is None else teacher[:, j - 1]
        lg = model.forward(kv, feed, np.arange(n_seqs), p, np.arange(n_seqs), n_threads)
        pick(lg, list(range(n_seqs)), j)
    return gen


def top2_margin(logits: np.ndarray) -> np.ndarray:
    """Gap between the largest and second-largest logit of each row."""
    part = np.partition(logits, -2, axis=-1)
    return part[..., -1] - part[..., -2]

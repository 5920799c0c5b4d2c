"""Host front end of the Llama step around the paged KV cache (include/lt_llama.h).

``Llama`` is the reference's ``Model`` (engine/crates/native/src/model.rs)
with its weights on one CUDA device: ``forward`` is ``Model::forward``
(model.rs:366-518) running Q8_0 matmuls, the int8 activation quantizer,
RMSNorm, RoPE and SiLU as sm_100a kernels, and the attention path through a
``KvCache``.  The op-level functions below call the same kernels one at a
time (``QMatrix::matmul``, ``QActs::quantize``, ...) for per-op checks.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _native as N
from .kv import KvCache, KvError, _dptr, _ptr, _stream, _u32

# lt_tensor ids (GGUF names per model.rs:236-262)
EMBED, OUTPUT, OUTPUT_NORM, ATTN_NORM, FFN_NORM, Q, K, V, O, GATE, UP, DOWN = range(12)
LAYER_TENSORS = (ATTN_NORM, FFN_NORM, Q, K, V, O, GATE, UP, DOWN)


class LlamaError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


def _check_op(rc: int, what: str):
    if rc != N.LT_OK:
        raise LlamaError(rc, f"{what} failed with status {rc}")


class Llama:
    """A llama-architecture model (Q8_0 weights) on one CUDA device."""

    def __init__(self, n_layers: int, dim: int, n_heads: int, n_kv_heads: int, head_dim: int, ffn_dim: int,
                 vocab: int, *, rope_dim: int = 0, rope_neox: bool = False, eps: float = 1e-5,
                 rope_base: float = 10000.0, max_batch: int = 512, device: int = 0):
        self._lib = N.lib()
        cfg = N.lt_llama_config(n_layers=n_layers, dim=dim, n_heads=n_heads, n_kv_heads=n_kv_heads,
                                head_dim=head_dim, ffn_dim=ffn_dim, vocab=vocab, rope_dim=rope_dim,
                                rope_neox=int(rope_neox), eps=eps, rope_base=rope_base, max_batch=max_batch,
                                device=device)
        h = C.c_void_p()
        rc = self._lib.lt_llama_create(C.byref(cfg), C.byref(h))
        if rc != N.LT_OK:
            raise LlamaError(rc, f"lt_llama_create failed with status {rc}")
        self._h = h
        self.n_layers, self.dim, self.n_heads, self.n_kv_heads = n_layers, dim, n_heads, n_kv_heads
        self.head_dim, self.ffn_dim, self.vocab = head_dim, ffn_dim, vocab
        self.max_batch, self.device = max_batch, device
        self.q_dim, self.kv_dim = n_heads * head_dim, n_kv_heads * head_dim

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.lt_llama_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _err(self, rc: int) -> Exception:
        msg = self._lib.lt_llama_last_error(self._h).decode()
        if rc in (N.LT_E_FULL, N.LT_E_NONCONTIG):
            return KvError(rc, msg)
        return LlamaError(rc, msg)

    def set_tensor(self, which: int, layer: int, data):
        """Copy one tensor in its GGUF encoding (Q8_0 blocks or F32) to the device."""
        buf = np.ascontiguousarray(np.frombuffer(memoryview(data), dtype=np.uint8))
        rc = self._lib.lt_llama_set_tensor(self._h, which, layer, _ptr(buf), buf.size)
        if rc != N.LT_OK:
            raise self._err(rc)

    def load(self, tensor):
        """Set every tensor from `tensor(which, layer) -> bytes`."""
        for which in (EMBED, OUTPUT, OUTPUT_NORM):
            self.set_tensor(which, 0, tensor(which, 0))
        for layer in range(self.n_layers):
            for which in LAYER_TENSORS:
                self.set_tensor(which, layer, tensor(which, layer))

    def kv_cache(self, n_tokens: int, max_seqs: int, **kw) -> KvCache:
        """A KvCache shaped for this model (KvCache::new, model.rs / native/src/lib.rs:94-98)."""
        return KvCache(self.n_layers, self.n_kv_heads, self.head_dim, n_tokens, n_heads=self.n_heads,
                       max_seqs=max_seqs, max_batch=kw.pop("max_batch", self.max_batch), device=self.device, **kw)

    def forward(self, kv: KvCache, tokens, seqs, positions, want, logits=None, stream=None):
        """Model::forward: logits [len(want), vocab] f32 on the device."""
        import torch

        tokens = np.ascontiguousarray(tokens, np.int32)
        seqs, positions, want = _u32(seqs), _u32(positions), _u32(want)
        n, m = tokens.size, want.size
        if logits is None:
            logits = torch.empty((max(m, 1), self.vocab), dtype=torch.float32, device=f"cuda:{self.device}")
        rc = self._lib.lt_llama_forward(self._h, kv._h, _ptr(tokens), _ptr(seqs), _ptr(positions), n, _ptr(want), m,
                                        _dptr(logits) if m else None, _stream(stream))
        if rc != N.LT_OK:
            raise self._err(rc)
        return logits[:m]

    def step_greedy(self, kv: KvCache, tokens, seqs, positions, want, stream=None) -> np.ndarray:
        """forward + argmax of each wanted token (sampling.rs:161-163); synchronises."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        seqs, positions, want = _u32(seqs), _u32(positions), _u32(want)
        nxt = np.zeros(max(want.size, 1), np.int32)
        rc = self._lib.lt_llama_step_greedy(self._h, kv._h, _ptr(tokens), _ptr(seqs), _ptr(positions), tokens.size,
                                            _ptr(want), want.size, _ptr(nxt), _stream(stream))
        if rc != N.LT_OK:
            raise self._err(rc)
        return nxt[: want.size]

    def set_persistent(self, enable: bool = True):
        """Run decode forwards (up to 8 tokens, one per sequence) as one
        persistent launch (default) or on the multi-launch path."""
        rc = self._lib.lt_llama_set_persistent(self._h, int(enable))
        if rc != N.LT_OK:
            raise self._err(rc)

    def persistent_available(self) -> bool:
        return bool(self._lib.lt_llama_persistent_available(self._h))

    def launch_count(self) -> int:
        return self._lib.lt_llama_launch_count(self._h)

    def profile(self, enable: bool = True):
        _check_op(self._lib.lt_llama_profile(self._h, int(enable)), "lt_llama_profile")

    def profile_read(self):
        """(matmul device ms, launches, algorithmic bytes) since the last read."""
        ms, n, b = C.c_double(), C.c_uint64(), C.c_uint64()
        rc = self._lib.lt_llama_profile_read(self._h, C.byref(ms), C.byref(n), C.byref(b))
        if rc != N.LT_OK:
            raise self._err(rc)
        return ms.value, n.value, b.value


def random_q8_0(rows: int, cols: int, sigma: float, rng: np.random.Generator) -> bytes:
    """A synthetic Q8_0 tensor in its GGUF encoding (34-byte blocks {f16 d;
    int8 qs[32]}): int8 values uniform in [-127, 127] and per-block scales
    around sigma * sqrt(3) / 127, so entries have standard deviation ~sigma."""
    nb = rows * cols // 32
    out = np.empty((nb, 34), np.uint8)
    d = (sigma * np.sqrt(3.0) / 127.0 * rng.uniform(0.5, 1.5, nb)).astype(np.float16)
    out[:, :2] = d.view(np.uint8).reshape(nb, 2)
    out[:, 2:] = rng.integers(-127, 128, (nb, 32), dtype=np.int8).view(np.uint8)
    return out.tobytes()


def random_weights(model: "Llama", seed: int = 0):
    """tensor(which, layer) -> bytes for a random-init model of model's shape:
    matrices ~ 0.02 (embedding ~ 1), norm vectors of ones."""
    rng = np.random.default_rng(seed)
    qd, kvd = model.q_dim, model.kv_dim
    shapes = {EMBED: (model.vocab, model.dim, 1.0), OUTPUT: (model.vocab, model.dim, 0.02),
              Q: (qd, model.dim, 0.02), K: (kvd, model.dim, 0.02), V: (kvd, model.dim, 0.02),
              O: (model.dim, qd, 0.02), GATE: (model.ffn_dim, model.dim, 0.02), UP: (model.ffn_dim, model.dim, 0.02),
              DOWN: (model.dim, model.ffn_dim, 0.02)}
    ones = np.ones(model.dim, np.float32).tobytes()

    def tensor(which, layer):
        if which in (OUTPUT_NORM, ATTN_NORM, FFN_NORM):
            return ones
        rows, cols, sigma = shapes[which]
        return random_q8_0(rows, cols, sigma, rng)

    return tensor


def serve_shared_prefix(model: Llama, kv: KvCache, prompts: np.ndarray, shared: int, n_gen: int,
                        teacher: np.ndarray | None = None, logits_out=None, stream=None) -> np.ndarray:
    """The C1 serving sequence on the device: prefill sequence 0, share its
    first `shared` positions into every other sequence (kv.rs:172-183),
    prefill their suffixes in one batch, then greedy decode with every
    sequence in each step.  `teacher` [n_seqs, n_gen] feeds fixed previous
    tokens instead of the model's picks; `logits_out` (host array
    [n_seqs, n_gen, vocab]) receives the logits behind every pick."""
    n_seqs, plen = prompts.shape
    gen = np.zeros((n_seqs, n_gen), np.int32)

    def run(tokens, seqs, pos, want, rows, j):
        if logits_out is None:
            gen[rows, j] = model.step_greedy(kv, tokens, seqs, pos, want, stream=stream)
        else:
            lg = model.forward(kv, tokens, seqs, pos, want, stream=stream)
            logits_out[rows, j] = lg.cpu().numpy()
            gen[rows, j] = argmax_rows(lg).cpu().numpy()

    run(prompts[0], np.zeros(plen), np.arange(plen), [plen - 1], [0], 0)
    for s in range(1, n_seqs):
        kv.share(0, s, shared)
    m = plen - shared
    run(prompts[1:, shared:].reshape(-1), np.repeat(np.arange(1, n_seqs), m), np.tile(np.arange(shared, plen),
        n_seqs - 1), [(i + 1) * m - 1 for i in range(n_seqs - 1)], list(range(1, n_seqs)), 0)
    for j in range(1, n_gen):
        feed = gen[:, j - 1] if teacher is None else teacher[:, j - 1]
        run(feed, np.arange(n_seqs), np.full(n_seqs, plen + j - 1), np.arange(n_seqs), list(range(n_seqs)), j)
    return gen


# ---------------------------------------------------------------- op level

def q8_quantize(x, stream=None):
    """QActs::quantize (quant.rs:771-795): x CUDA f32 [n, cols] -> (qs int8, scales f32)."""
    import torch

    n, cols = x.shape
    qs = torch.empty((n, cols), dtype=torch.int8, device=x.device)
    sc = torch.empty((n, cols // 32), dtype=torch.float32, device=x.device)
    _check_op(N.lib().lt_q8_quantize(_dptr(x), n, cols, _dptr(qs), _dptr(sc), _stream(stream)), "lt_q8_quantize")
    return qs, sc


def q8_matmul(w_qs, w_scales_f16, x_qs, x_scales, out=None, accumulate=False, stream=None):
    """QMatrix::matmul (quant.rs:492-533): out [n, rows] f32 (+)= W . x."""
    import torch

    rows, cols = w_qs.shape
    n = x_qs.shape[0]
    if out is None:
        out = torch.empty((n, rows), dtype=torch.float32, device=w_qs.device)
    _check_op(N.lib().lt_q8_matmul(_dptr(w_qs), _dptr(w_scales_f16), rows, cols, _dptr(x_qs), _dptr(x_scales), n,
                                   _dptr(out), out.stride(0), int(accumulate), _stream(stream)), "lt_q8_matmul")
    return out


PRO_QUANT, PRO_SILU, PRO_RMSNORM = 1, 2, 3


def q8_project(prologue: int, w_qs, w_scales_f16, x, rows_idx=None, gamma=None, eps: float = 1e-5, out=None,
               accumulate=False, fused=True, stream=None):
    """Activation prologue (quantize / SiLU * up + quantize / RMSNorm +
    quantize of f32 x) and the Q8_0 matmul; one launch when fused and n <= 8."""
    import torch

    rows, cols = w_qs.shape
    n = rows_idx.numel() if rows_idx is not None else x.shape[0]
    if out is None:
        out = torch.empty((n, rows), dtype=torch.float32, device=w_qs.device)
    idx = None if rows_idx is None else _dptr(rows_idx)
    g = None if gamma is None else _dptr(gamma)
    _check_op(N.lib().lt_q8_project(prologue, _dptr(w_qs), _dptr(w_scales_f16), rows, cols, _dptr(x), idx, g, eps, n,
                                    _dptr(out), out.stride(0), int(fused), int(accumulate), _stream(stream)),
              "lt_q8_project")
    return out


def q8_check(stream=None):
    """Raise if an op-level matmul's bounded wait gave up (synchronises)."""
    _check_op(N.lib().lt_q8_check(_stream(stream)), "lt_q8_check")


def rms_norm_q8(x, w, eps: float, rows_idx=None, stream=None):
    """rms_norm (model.rs:174-183) + quantize: -> (normed f32, qs, scales)."""
    import torch

    n = x.shape[0] if rows_idx is None else rows_idx.numel()
    dim = x.shape[1]
    normed = torch.empty((n, dim), dtype=torch.float32, device=x.device)
    qs = torch.empty((n, dim), dtype=torch.int8, device=x.device)
    sc = torch.empty((n, dim // 32), dtype=torch.float32, device=x.device)
    idx = None if rows_idx is None else _dptr(rows_idx)
    _check_op(N.lib().lt_rms_norm_q8(_dptr(x), idx, _dptr(w), dim, n, eps, _dptr(normed), _dptr(qs), _dptr(sc),
                                     _stream(stream)), "lt_rms_norm_q8")
    return normed, qs, sc


def silu_q8(gu, ffn: int, stream=None):
    """SiLU(gate) * up (model.rs:492-494) + quantize; gu [n, 2*ffn]."""
    import torch

    n = gu.shape[0]
    h = torch.empty((n, ffn), dtype=torch.float32, device=gu.device)
    qs = torch.empty((n, ffn), dtype=torch.int8, device=gu.device)
    sc = torch.empty((n, ffn // 32), dtype=torch.float32, device=gu.device)
    _check_op(N.lib().lt_silu_q8(_dptr(gu), n, ffn, _dptr(h), _dptr(qs), _dptr(sc), _stream(stream)), "lt_silu_q8")
    return h, qs, sc


def argmax_rows(x, stream=None):
    """Greedy pick per row (sampling.rs:161-163) -> int32 [n] on the device."""
    import torch

    n, cols = x.shape
    idx = torch.empty(n, dtype=torch.int32, device=x.device)
    _check_op(N.lib().lt_argmax_f32(_dptr(x), n, cols, _dptr(idx), _stream(stream)), "lt_argmax_f32")
    return idx

"""TEST INFRASTRUCTURE ONLY: ctypes/numpy front end of the C oracle.

The oracle (``oracle/lt_oracle.c``) restates the reference engine's paged KV
cache (``engine/crates/native/src/kv.rs``) and attention closure
(``engine/crates/native/src/model.rs:431-476``) on the CPU.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg import this
module, as the checker or the timed CPU baseline.  The product path
(``langtrain_studio_b200``) never imports it.

Parity pins: bookkeeping against the reference's known-answer tests
(``kv.rs:202-229``), f32->f16 against numpy's IEEE round-to-nearest-even.
Attention arithmetic: no golden vectors exist in the reference, so it is
pinned only by this restatement.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "lt_oracle.c"
HDR = HERE / "lt_oracle.h"
# The C1 end-to-end forward (model.rs restated) lives in the same library.
MODEL_SRC = HERE / "lt_model.c"
MODEL_HDR = HERE / "lt_model.h"
SOURCES = (SRC, HDR, MODEL_SRC, MODEL_HDR)
BUILD_DIR = HERE / "_build"
LIB = BUILD_DIR / "liblt_oracle.so"

# x86-64-v3 (AVX2/F16C) rather than -march=native: the built library travels to
# other hosts.  -ffp-contract=off: Rust never fuses a*b+c, neither may we.
CFLAGS = ["-O3", "-march=x86-64-v3", "-mf16c", "-ffp-contract=off", "-fno-fast-math",
          "-std=c11", "-fPIC", "-shared", "-pthread", "-fopenmp", "-Wall"]

BLOCK = 16
OK, FULL, NONCONTIG, ARG = 0, 1, 2, 3


def build(force: bool = False) -> Path:
    """Compile the oracle with gcc into oracle/_build/ (idempotent)."""
    BUILD_DIR.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(f.stat().st_mtime for f in SOURCES):
        return LIB
    tmp = LIB.with_suffix(".so.tmp%d" % os.getpid())
    subprocess.run(["gcc", *CFLAGS, "-o", str(tmp), str(SRC), str(MODEL_SRC), "-lm"], check=True)
    os.replace(tmp, LIB)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(str(LIB))
        u32, i32, u64, p = C.c_uint32, C.c_int32, C.c_uint64, C.c_void_p
        L.okv_new.restype = p
        L.okv_new.argtypes = [u32, u32, u32, u32]
        L.okv_new_q8.restype = p
        L.okv_new_q8.argtypes = [u32, u32, u32, u32]
        L.okv_q8_group.restype = C.c_float
        L.okv_q8_group.argtypes = [p, p]
        for name in ("okv_pool_kq", "okv_pool_vq", "okv_pool_kd", "okv_pool_vd"):
            getattr(L, name).restype = p
            getattr(L, name).argtypes = [p]
        L.okv_delete.argtypes = [p]
        for name in ("okv_capacity", "okv_free_blocks", "okv_n_blocks"):
            getattr(L, name).restype = u32
            getattr(L, name).argtypes = [p]
        L.okv_bytes.restype = u64
        L.okv_bytes.argtypes = [p]
        L.okv_len.restype = u32
        L.okv_len.argtypes = [p, u32]
        L.okv_append.restype = C.c_int
        L.okv_append.argtypes = [p, u32, u32, p, p]
        L.okv_append_batch.restype = C.c_int
        L.okv_append_batch.argtypes = [p, p, p, u32, p, p, p]
        L.okv_write.argtypes = [p, u32, i32, i32, p, p]
        L.okv_write_batch.argtypes = [p, u32, p, p, u32, p, p]
        L.okv_write_batch_f16.argtypes = [p, u32, p, p, u32, p, p]
        L.okv_truncate.argtypes = [p, u32, u32]
        L.okv_share.argtypes = [p, u32, u32, u32]
        L.okv_compact.restype = u32
        L.okv_compact.argtypes = [p, p]
        L.okv_seq_blocks.restype = u32
        L.okv_seq_blocks.argtypes = [p, u32, p, u32]
        L.okv_refs.argtypes = [p, p]
        L.okv_free_list.restype = u32
        L.okv_free_list.argtypes = [p, p, u32]
        L.okv_pool_k.restype = p
        L.okv_pool_k.argtypes = [p]
        L.okv_pool_v.restype = p
        L.okv_pool_v.argtypes = [p]
        L.okv_rows.argtypes = [p, u32, u32, u32, p, p]
        L.okv_attend.argtypes = [p, u32, p, p, p, u32, u32, u32, u32, C.c_float, p, C.c_int]
        L.okv_f32_to_f16.restype = C.c_uint16
        L.okv_f32_to_f16.argtypes = [C.c_float]
        L.okv_f16_to_f32.restype = C.c_float
        L.okv_f16_to_f32.argtypes = [C.c_uint16]
        L.okv_f32_to_f16_array.argtypes = [p, p, C.c_size_t]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


def f32_to_f16_bits(x) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().okv_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
    return out


class OracleError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(msg)
        self.code = code


def q8_group(x) -> tuple[np.ndarray, float]:
    """One 32-value group through the engine's int8 quantiser (quant.rs:785-795):
    (int8 values, f32 scale d)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    assert x.size == 32
    q = np.zeros(32, np.int8)
    d = lib().okv_q8_group(_ptr(x), _ptr(q))
    return q, float(np.float32(d))


class OracleKv:
    """KvCache (kv.rs:15-188) restated: same method names and error behaviour.
    kv_format "q8_0" keeps rows as Q8_0 groups (lt_kv.h LT_KV_Q8_0)."""

    def __init__(self, n_layers: int, kv_dim: int, n_tokens: int, max_seqs: int = 1024,
                 kv_format: str = "f16"):
        assert kv_format in ("f16", "q8_0")
        make = lib().okv_new_q8 if kv_format == "q8_0" else lib().okv_new
        self._h = make(n_layers, kv_dim, n_tokens, max_seqs)
        if not self._h:
            raise MemoryError("okv_new failed")
        self.kv_format = kv_format
        self.n_layers, self.kv_dim, self.max_seqs = n_layers, kv_dim, max_seqs
        self.n_blocks = lib().okv_n_blocks(self._h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().okv_delete(h)
            self._h = None

    # accessors ------------------------------------------------------------
    def capacity(self) -> int:
        return lib().okv_capacity(self._h)

    def bytes(self) -> int:
        return lib().okv_bytes(self._h)

    def len(self, seq: int) -> int:
        return lib().okv_len(self._h, seq)

    def free_blocks(self) -> int:
        return lib().okv_free_blocks(self._h)

    # mutation -------------------------------------------------------------
    def append(self, seq: int, pos: int):
        b, s = C.c_int32(), C.c_int32()
        rc = lib().okv_append(self._h, seq, pos, C.byref(b), C.byref(s))
        if rc == FULL:
            raise OracleError(rc, "KV cache full")
        if rc == NONCONTIG:
            raise OracleError(rc, f"seq {seq}: position {pos} is not contiguous (length {self.len(seq)})")
        if rc:
            raise OracleError(rc, "bad argument")
        return b.value, s.value

    def append_batch(self, seqs, positions):
        seqs = np.ascontiguousarray(seqs, dtype=np.uint32)
        positions = np.ascontiguousarray(positions, dtype=np.uint32)
        n = seqs.size
        blocks = np.zeros(n, np.int32)
        slots = np.zeros(n, np.int32)
        done = C.c_uint32()
        rc = lib().okv_append_batch(self._h, _ptr(seqs), _ptr(positions), n, _ptr(blocks), _ptr(slots),
                                    C.byref(done))
        return rc, done.value, blocks, slots

    def write(self, layer: int, block: int, slot: int, k, v):
        k = np.ascontiguousarray(k, dtype=np.float32)
        v = np.ascontiguousarray(v, dtype=np.float32)
        assert k.size == self.kv_dim and v.size == self.kv_dim
        lib().okv_write(self._h, layer, block, slot, _ptr(k), _ptr(v))

    def write_batch(self, layer: int, blocks, slots, k, v):
        blocks = np.ascontiguousarray(blocks, dtype=np.int32)
        slots = np.ascontiguousarray(slots, dtype=np.int32)
        n = blocks.size
        if np.asarray(k).dtype == np.float16:
            k = np.ascontiguousarray(k, dtype=np.float16).view(np.uint16).reshape(n, self.kv_dim)
            v = np.ascontiguousarray(v, dtype=np.float16).view(np.uint16).reshape(n, self.kv_dim)
            lib().okv_write_batch_f16(self._h, layer, _ptr(blocks), _ptr(slots), n, _ptr(k), _ptr(v))
        else:
            k = np.ascontiguousarray(k, dtype=np.float32).reshape(n, self.kv_dim)
            v = np.ascontiguousarray(v, dtype=np.float32).reshape(n, self.kv_dim)
            lib().okv_write_batch(self._h, layer, _ptr(blocks), _ptr(slots), n, _ptr(k), _ptr(v))

    def truncate(self, seq: int, start: int):
        lib().okv_truncate(self._h, seq, start)

    def share(self, src: int, dst: int, length: int):
        lib().okv_share(self._h, src, dst, length)

    def compact(self):
        moves = np.zeros((max(self.n_blocks, 1), 2), np.int32)
        n = lib().okv_compact(self._h, _ptr(moves))
        return moves[:n].copy()

    # introspection --------------------------------------------------------
    def seq_blocks(self, seq: int) -> np.ndarray:
        n = lib().okv_seq_blocks(self._h, seq, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        lib().okv_seq_blocks(self._h, seq, _ptr(out), n)
        return out[:n]

    def refs(self) -> np.ndarray:
        out = np.zeros(max(self.n_blocks, 1), np.uint32)
        lib().okv_refs(self._h, _ptr(out))
        return out[: self.n_blocks]

    def free_list(self) -> np.ndarray:
        out = np.zeros(max(self.n_blocks, 1), np.int32)
        n = lib().okv_free_list(self._h, _ptr(out), self.n_blocks)
        return out[:n].copy()

    def pool(self):
        """(K, V) as uint16 views [layer][block][slot][kv_dim] (reference layout)."""
        shape = (self.n_layers, self.n_blocks, BLOCK, self.kv_dim)
        n = int(np.prod(shape))
        kp = C.cast(lib().okv_pool_k(self._h), C.POINTER(C.c_uint16))
        vp = C.cast(lib().okv_pool_v(self._h), C.POINTER(C.c_uint16))
        k = np.ctypeslib.as_array(kp, shape=(n,)).reshape(shape)
        v = np.ctypeslib.as_array(vp, shape=(n,)).reshape(shape)
        return k, v

    def pool_q8(self):
        """Q8_0 cache: (Kq, Vq) int8 [layer][block][slot][kv_dim] and (Kd, Vd) f16 bits
        [layer][block][slot][kv_dim/32]."""
        assert self.kv_format == "q8_0"
        shape = (self.n_layers, self.n_blocks, BLOCK, self.kv_dim)
        dshape = shape[:3] + (self.kv_dim // 32,)
        out = []
        for name, ct, shp in (("okv_pool_kq", C.c_int8, shape), ("okv_pool_vq", C.c_int8, shape),
                              ("okv_pool_kd", C.c_uint16, dshape), ("okv_pool_vd", C.c_uint16, dshape)):
            ptr = C.cast(getattr(lib(), name)(self._h), C.POINTER(ct))
            out.append(np.ctypeslib.as_array(ptr, shape=(int(np.prod(shp)),)).reshape(shp))
        return tuple(out)

    def rows(self, layer: int, seq: int, n: int):
        k = np.zeros((n, self.kv_dim), np.uint16)
        v = np.zeros((n, self.kv_dim), np.uint16)
        lib().okv_rows(self._h, layer, seq, n, _ptr(k), _ptr(v))
        return k, v

    def attend(self, layer: int, q, seqs, positions, n_heads: int, n_kv_heads: int, head_dim: int,
               scale: float | None = None, n_threads: int = 0) -> np.ndarray:
        q = np.ascontiguousarray(q, dtype=np.float32)
        seqs = np.ascontiguousarray(seqs, dtype=np.uint32)
        positions = np.ascontiguousarray(positions, dtype=np.uint32)
        n = seqs.size
        assert q.size == n * n_heads * head_dim
        if scale is None:
            scale = float(np.float32(1.0) / np.sqrt(np.float32(head_dim)))  # model.rs:402
        out = np.zeros((n, n_heads * head_dim), np.float32)
        lib().okv_attend(self._h, layer, _ptr(q), _ptr(seqs), _ptr(positions), n, n_heads, n_kv_heads,
                         head_dim, scale, _ptr(out), n_threads)
        return out

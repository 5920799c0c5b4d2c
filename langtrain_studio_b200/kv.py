"""Python host mirror of the reference's paged KV cache over the C ABI.

`KvCache` keeps the method names, argument meaning and error behaviour of
the reference's `KvCache` (engine/crates/native/src/kv.rs:15-188) and of the
attention closure of `Model::forward` (engine/crates/native/src/model.rs:
431-476), batched the way `Model::forward` drives them.  Every call goes
through liblt_kv.so; device arrays are torch CUDA tensors, host arrays are
numpy.  Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _native as N

BLOCK = N.BLOCK


class KvError(RuntimeError):
    """A failed C-ABI call; `code` is the lt_status value."""

    def __init__(self, code: int, message: str, n_done: int | None = None):
        super().__init__(message)
        self.code = code
        self.n_done = n_done


class KvCacheFull(KvError):
    pass


class KvNonContiguous(KvError):
    pass


def _ptr(a: np.ndarray) -> int:
    """Address of a C-contiguous numpy array for a c_void_p parameter (the
    array must outlive the call).  ctypes.from_buffer is ~3x cheaper than
    ndarray.ctypes, which matters on the per-step call path; read-only and
    empty arrays take the general route."""
    try:
        return C.addressof(C.c_char.from_buffer(a))
    except (TypeError, ValueError, BufferError):
        return a.ctypes.data


def _dptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _stream(stream) -> C.c_void_p:
    if isinstance(stream, C.c_void_p):
        return stream
    if stream is None:
        import torch

        stream = torch.cuda.current_stream()
    return C.c_void_p(getattr(stream, "cuda_stream", stream))


def _dtype_code(t) -> int:
    import torch

    if t.dtype == torch.float32:
        return N.LT_F32
    if t.dtype == torch.float16:
        return N.LT_F16
    raise TypeError(f"unsupported dtype {t.dtype} (float32 or float16)")


def _u32(a) -> np.ndarray:
    if isinstance(a, np.ndarray) and a.dtype == np.uint32 and a.flags.c_contiguous:
        return a
    return np.ascontiguousarray(np.asarray(a, dtype=np.int64).astype(np.uint32))


def _i32(a) -> np.ndarray:
    if isinstance(a, np.ndarray) and a.dtype == np.int32 and a.flags.c_contiguous:
        return a
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


KV_FORMATS = {"f16": N.LT_KV_F16, "q8_0": N.LT_KV_Q8_0}


class KvCache:
    """Paged KV cache of 16-token blocks on one CUDA device.

    ``KvCache(n_layers, n_kv_heads, head_dim, n_tokens)`` is the reference's
    ``KvCache::new(n_layers, n_kv_heads * head_dim, n_tokens)``.  ``device=-1``
    builds a bookkeeping-only handle (no GPU), for host-side tests.
    ``kv_format="q8_0"`` stores rows as Q8_0 groups (include/lt_kv.h,
    LT_KV_Q8_0) instead of f16.
    """

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, n_tokens: int, *, n_heads: int | None = None,
                 max_seqs: int = 256, max_batch: int = 512, max_blocks_per_seq: int = 0, device: int = 0,
                 kv_format: str = "f16"):
        self._lib = N.lib()
        if kv_format not in KV_FORMATS:
            raise ValueError(f"kv_format must be one of {sorted(KV_FORMATS)}")
        cfg = N.lt_kv_config(
            n_layers=n_layers, n_kv_heads=n_kv_heads, head_dim=head_dim,
            n_heads=n_heads if n_heads is not None else n_kv_heads, n_tokens=n_tokens, max_seqs=max_seqs,
            max_batch=max_batch, max_blocks_per_seq=max_blocks_per_seq, device=device,
            kv_format=KV_FORMATS[kv_format])
        self.kv_format = kv_format
        h = C.c_void_p()
        rc = self._lib.lt_kv_create(C.byref(cfg), C.byref(h))
        if rc != N.LT_OK:
            raise KvError(rc, f"lt_kv_create failed with status {rc}")
        self._h = h
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        # model.rs:402: 1 / sqrt(head_dim) in f32
        self.default_scale = float(np.float32(1.0) / np.float32(math.sqrt(head_dim)))
        self.n_heads = cfg.n_heads
        self.kv_dim = n_kv_heads * head_dim
        self.max_seqs, self.max_batch, self.device = max_seqs, max_batch, device
        self.n_blocks = self._lib.lt_kv_n_blocks(h)

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.lt_kv_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- errors
    def _err(self, rc: int, n_done: int | None = None) -> KvError:
        msg = self._lib.lt_kv_last_error(self._h).decode()
        cls = {N.LT_E_FULL: KvCacheFull, N.LT_E_NONCONTIG: KvNonContiguous}.get(rc, KvError)
        return cls(rc, msg, n_done)

    def _check(self, rc: int):
        if rc != N.LT_OK:
            raise self._err(rc)

    # ------------------------------------------------------------- accessors
    def capacity(self) -> int:
        """Tokens the pool holds (kv.rs:50; Backend::n_ctx)."""
        return self._lib.lt_kv_capacity(self._h)

    def bytes(self) -> int:
        return self._lib.lt_kv_bytes(self._h)

    def len(self, seq: int) -> int:
        return self._lib.lt_kv_len(self._h, seq)

    def free_blocks(self) -> int:
        return self._lib.lt_kv_free_blocks(self._h)

    # -------------------------------------------------------------- mutation
    def append(self, seq: int, pos: int, stream=None):
        """Claim the cell for `pos` of `seq` (kv.rs:85-121) -> (block, slot)."""
        blocks, slots = self.append_batch([seq], [pos], stream=stream)
        return int(blocks[0]), int(slots[0])

    def append_batch(self, seqs, positions, stream=None):
        """Claim cells for a batch in order (model.rs:380-383).  On error the
        raised KvError carries `n_done`: the tokens claimed before it."""
        seqs, positions = _u32(seqs), _u32(positions)
        n = seqs.size
        blocks = np.zeros(max(n, 1), np.int32)
        slots = np.zeros(max(n, 1), np.int32)
        done = C.c_uint32()
        st = _stream(stream) if self.device >= 0 else C.c_void_p(0)
        rc = self._lib.lt_kv_append(self._h, _ptr(seqs), _ptr(positions), n, _ptr(blocks), _ptr(slots),
                                    C.byref(done), st)
        if rc != N.LT_OK:
            raise self._err(rc, done.value)
        return blocks[:n], slots[:n]

    def write(self, layer: int, blocks, slots, k, v, stream=None):
        """KvCache::write for n cells (kv.rs:123-131): k, v CUDA [n, kv_dim]."""
        blocks, slots = _i32(blocks), _i32(slots)
        n = blocks.size
        assert k.is_cuda and k.is_contiguous() and v.is_contiguous() and k.dtype == v.dtype
        assert k.numel() == n * self.kv_dim and v.numel() == n * self.kv_dim
        self._check(self._lib.lt_kv_write(self._h, layer, _ptr(blocks), _ptr(slots), n, _dptr(k), _dptr(v),
                                          _dtype_code(k), _stream(stream)))

    def attend(self, layer: int, q, seqs, positions, out=None, out_dtype=None, scale: float | None = None,
               stream=None):
        """Attention closure (model.rs:431-476): q CUDA [n, n_heads*head_dim]."""
        import torch

        seqs, positions = _u32(seqs), _u32(positions)
        n = seqs.size
        assert q.is_cuda and q.is_contiguous() and q.numel() == n * self.n_heads * self.head_dim
        if out is None:
            out = torch.empty((n, self.n_heads * self.head_dim), dtype=out_dtype or torch.float32, device=q.device)
        if scale is None:
            scale = self.default_scale
        self._check(self._lib.lt_kv_attend(self._h, layer, _dptr(q), _dtype_code(q), _ptr(seqs), _ptr(positions), n,
                                           _dptr(out), _dtype_code(out), scale, _stream(stream)))
        return out

    def write_attend(self, layer: int, blocks, slots, k, v, q, seqs, positions, out=None, out_dtype=None,
                     scale: float | None = None, stream=None):
        """write() then attend() for the same tokens, in one kernel when legal."""
        import torch

        blocks, slots = _i32(blocks), _i32(slots)
        seqs, positions = _u32(seqs), _u32(positions)
        n = seqs.size
        if out is None:
            out = torch.empty((n, self.n_heads * self.head_dim), dtype=out_dtype or torch.float32, device=q.device)
        if scale is None:
            scale = self.default_scale
        self._check(self._lib.lt_kv_write_attend(
            self._h, layer, _ptr(blocks), _ptr(slots), _dptr(k), _dptr(v), _dtype_code(k), _dptr(q), _dtype_code(q),
            _ptr(seqs), _ptr(positions), n, _dptr(out), _dtype_code(out), scale, _stream(stream)))
        return out

    # ------------------------------------------- head-sharded peer gather
    def peer_export(self, rank: int, nranks: int, max_tokens: int) -> bytes:
        """Allocate this rank's gather buffer; returns its 64-byte IPC handle."""
        buf = C.create_string_buffer(N.LT_IPC_HANDLE_BYTES)
        self._check(self._lib.lt_kv_peer_export(self._h, rank, nranks, max_tokens, buf))
        self.peer_ranks = nranks
        return buf.raw

    def peer_import(self, handles):
        """Map every rank's gather buffer (handles in rank order)."""
        blob = b"".join(bytes(h) for h in handles)
        assert len(blob) == N.LT_IPC_HANDLE_BYTES * self.peer_ranks
        self._check(self._lib.lt_kv_peer_import(self._h, C.create_string_buffer(blob, len(blob))))

    def peer_close(self):
        self._check(self._lib.lt_kv_peer_close(self._h))

    def attend_gather(self, layer: int, q, seqs, positions, out=None, out_dtype=None, scale: float | None = None,
                      stream=None):
        """attend() of this rank's heads, gathered over NVLink into
        [n, nranks * n_heads * head_dim] (lt_kv_attend_gather)."""
        import torch

        seqs, positions = _u32(seqs), _u32(positions)
        n = seqs.size
        assert q.is_cuda and q.is_contiguous() and q.numel() == n * self.n_heads * self.head_dim
        if out is None:
            out = torch.empty((n, self.peer_ranks * self.n_heads * self.head_dim), dtype=out_dtype or torch.float32,
                              device=q.device)
        if scale is None:
            scale = self.default_scale
        self._check(self._lib.lt_kv_attend_gather(self._h, layer, _dptr(q), _dtype_code(q), _ptr(seqs),
                                                  _ptr(positions), n, _dptr(out), _dtype_code(out), scale,
                                                  _stream(stream)))
        return out

    def write_attend_gather(self, layer: int, blocks, slots, k, v, q, seqs, positions, out=None, out_dtype=None,
                            scale: float | None = None, stream=None):
        """write_attend() with the gather fused in (lt_kv_write_attend_gather)."""
        import torch

        blocks, slots = _i32(blocks), _i32(slots)
        seqs, positions = _u32(seqs), _u32(positions)
        n = seqs.size
        if out is None:
            out = torch.empty((n, self.peer_ranks * self.n_heads * self.head_dim), dtype=out_dtype or torch.float32,
                              device=q.device)
        if scale is None:
            scale = self.default_scale
        self._check(self._lib.lt_kv_write_attend_gather(
            self._h, layer, _ptr(blocks), _ptr(slots), _dptr(k), _dptr(v), _dtype_code(k), _dptr(q), _dtype_code(q),
            _ptr(seqs), _ptr(positions), n, _dptr(out), _dtype_code(out), scale, _stream(stream)))
        return out

    def truncate(self, seq: int, start: int):
        """Drop positions start.. of seq (kv.rs:153-169; Backend::kv_remove)."""
        self._lib.lt_kv_truncate(self._h, seq, start)

    def share(self, src: int, dst: int, length: int):
        """dst starts with the first `length` tokens of src (kv.rs:172-183)."""
        self._lib.lt_kv_share(self._h, src, dst, length)

    def compact(self, stream=None) -> int:
        moved = C.c_uint32()
        st = _stream(stream) if self.device >= 0 else C.c_void_p(0)
        self._check(self._lib.lt_kv_compact(self._h, C.byref(moved), st))
        return moved.value

    def flush(self, stream=None):
        st = _stream(stream) if self.device >= 0 else C.c_void_p(0)
        self._check(self._lib.lt_kv_flush(self._h, st))

    def check(self, stream=None):
        st = _stream(stream) if self.device >= 0 else C.c_void_p(0)
        self._check(self._lib.lt_kv_check(self._h, st))

    def selftest_wait(self, limit_us: int, stream=None):
        """Make one bounded device wait run out (a flag nothing sets, limit
        `limit_us`); the next check() raises KvError(LT_E_TIMEOUT)."""
        self._check(self._lib.lt_kv_selftest_wait(self._h, int(limit_us), _stream(stream)))

    def rows(self, layer: int, seq: int, n: int, stream=None):
        """K and V rows 0..n of seq (kv.rs:135-150) as f16 CUDA [n, kv_dim]."""
        import torch

        k = torch.empty((n, self.kv_dim), dtype=torch.float16, device=f"cuda:{self.device}")
        v = torch.empty_like(k)
        self._check(self._lib.lt_kv_rows(self._h, layer, seq, n, _dptr(k), _dptr(v), _stream(stream)))
        return k, v

    # --------------------------------------------------------- introspection
    def seq_blocks(self, seq: int) -> np.ndarray:
        n = self._lib.lt_kv_seq_blocks(self._h, seq, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self._lib.lt_kv_seq_blocks(self._h, seq, _ptr(out), n)
        return out[:n]

    def refs(self) -> np.ndarray:
        out = np.zeros(max(self.n_blocks, 1), np.uint32)
        self._lib.lt_kv_refs(self._h, _ptr(out), self.n_blocks)
        return out[: self.n_blocks]

    def free_list(self) -> np.ndarray:
        out = np.zeros(max(self.n_blocks, 1), np.int32)
        n = self._lib.lt_kv_free_list(self._h, _ptr(out), self.n_blocks)
        return out[:n]

    def profile(self, enable: bool = True):
        """Bracket every attention launch with CUDA events (resets totals)."""
        self._check(self._lib.lt_kv_profile(self._h, int(enable)))

    def profile_read(self):
        """(total ms, launches) of the attention launches timed so far."""
        ms, n = C.c_double(), C.c_uint64()
        self._check(self._lib.lt_kv_profile_read(self._h, C.byref(ms), C.byref(n)))
        return ms.value, n.value

    def profile_read_plan(self):
        """(total ms, launches, copied blocks, table entries) of the plan
        launches (copy-on-write copies, compaction moves, table entries)
        timed so far."""
        ms, n, blocks, entries = C.c_double(), C.c_uint64(), C.c_uint64(), C.c_uint64()
        self._check(self._lib.lt_kv_profile_read_plan(self._h, C.byref(ms), C.byref(n), C.byref(blocks),
                                                      C.byref(entries)))
        return ms.value, n.value, blocks.value, entries.value

    def profile_read_write(self):
        """(total ms, launches, rows, input bytes) of the K/V write launches
        (lt_kv_write) timed so far."""
        ms, n, rows, nbytes = C.c_double(), C.c_uint64(), C.c_uint64(), C.c_uint64()
        self._check(self._lib.lt_kv_profile_read_write(self._h, C.byref(ms), C.byref(n), C.byref(rows),
                                                       C.byref(nbytes)))
        return ms.value, n.value, rows.value, nbytes.value

    def set_min_tiles_per_warp(self, tiles: int):
        """Attention launch sizing: at least `tiles` tiles per warp (default 8)."""
        self._check(self._lib.lt_kv_set_min_tiles_per_warp(self._h, tiles))

    def set_cascade(self, min_group_tokens: int):
        """Shared-prefix attention pass for groups of >= min_group_tokens tokens (0: off)."""
        self._check(self._lib.lt_kv_set_cascade(self._h, min_group_tokens))

    def cascade_launches(self) -> int:
        return self._lib.lt_kv_cascade_launches(self._h)

    def launch_count(self) -> int:
        return self._lib.lt_kv_launch_count(self._h)

    def read_pool(self, layer: int, block0: int = 0, count: int | None = None) -> np.ndarray:
        """Raw device pool of blocks [block0, block0 + count) of one layer
        (default: all): f16 caches give uint16 [block][kv_head][2][16][head_dim]
        with the chunk swizzle of include/lt_kv.h still applied; Q8_0 caches
        give the uint8 tiles [block][kv_head][34 * head_dim]."""
        if count is None:
            count = self.n_blocks - block0
        if self.kv_format == "q8_0":
            out = np.zeros((count, self.n_kv_heads, 34 * self.head_dim), np.uint8)
        else:
            out = np.zeros((count, self.n_kv_heads, 2, BLOCK, self.head_dim), np.uint16)
        self._check(self._lib.lt_kv_read_pool(self._h, layer, block0, count, _ptr(out)))
        return out

    def pool_reference_layout(self, layer: int, block0: int = 0, count: int | None = None):
        """Blocks [block0, block0 + count) of this layer's pool as the
        reference lays it out (kv.rs:20): (K, V) uint16 [block][slot][kv_dim];
        for Q8_0 (Kq, Vq) int8 [block][slot][kv_dim] and (Kd, Vd) f16 bits
        [block][slot][kv_dim/32]."""
        if self.kv_format == "q8_0":
            return unswizzle_pool_q8(self.read_pool(layer, block0, count), self.head_dim)
        return unswizzle_pool(self.read_pool(layer, block0, count))


class NcclComm:
    """NCCL communicator for KV-head sharding (lt_kv_nccl_init).  Every rank
    builds it with the same 128-byte id from `nccl_unique_id()` on rank 0."""

    def __init__(self, nranks: int, uid: bytes, rank: int, device: int):
        lib = N.lib()
        buf = C.create_string_buffer(bytes(uid), 128)
        h = C.c_void_p()
        rc = lib.lt_kv_nccl_init(C.byref(h), nranks, buf, rank, device)
        if rc != N.LT_OK:
            raise KvError(rc, f"lt_kv_nccl_init failed with status {rc}")
        self.handle, self.nranks, self.rank = h, nranks, rank

    def close(self):
        if self.handle:
            N.lib().lt_kv_nccl_destroy(self.handle)
            self.handle = None


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    rc = N.lib().lt_kv_nccl_unique_id(buf)
    if rc != N.LT_OK:
        raise KvError(rc, "NCCL is not available (libnccl.so.2)")
    return buf.raw


def setup_peer_gather(kv: "KvCache", rank: int, nranks: int, max_tokens: int):
    """Export this rank's gather buffer, exchange IPC handles over the
    default torch.distributed group, and map every rank's buffer."""
    import torch.distributed as dist

    mine = kv.peer_export(rank, nranks, max_tokens)
    handles = [None] * nranks
    dist.all_gather_object(handles, mine)
    kv.peer_import(handles)


def gather_heads(kv: "KvCache", local, comm: NcclComm, out=None, gathered=None, stream=None):
    """All-gather head-sharded attention outputs into the unsharded layout
    [n][nranks * n_heads * head_dim] (lt_kv_gather_heads)."""
    import torch

    n = local.shape[0]
    w = comm.nranks
    if gathered is None:
        gathered = torch.empty((w, n, local.shape[1]), dtype=local.dtype, device=local.device)
    if out is None:
        out = torch.empty((n, w * local.shape[1]), dtype=local.dtype, device=local.device)
    kv._check(kv._lib.lt_kv_gather_heads(kv._h, _dptr(local), _dptr(gathered), _dptr(out), n, _dtype_code(local),
                                         comm.handle, w, _stream(stream)))
    return out


def unswizzle_pool(raw: np.ndarray):
    """Invert the device pool layout -> reference (K, V) [block][16][head*D].

    Device layout: [block][head][2 (K, V)][D/64][16 slots][64]; inside each
    16 x 64 sub-tile the 16-byte chunk c of slot s is stored at chunk
    position c ^ (s & 7)."""
    nb, hkv, _, blk, d = raw.shape
    hs = d // 64
    sub = raw.reshape(nb, hkv, 2, hs, blk, 8, 8)  # [.., half, slot, physical chunk, 8]
    slot = np.arange(blk)[:, None]
    c = np.arange(8)[None, :]
    phys = c ^ (slot & 7)  # logical chunk c of slot s lives at physical chunk phys
    logical = sub[:, :, :, :, np.arange(blk)[:, None], phys, :]  # [nb, hkv, 2, hs, blk, 8, 8]
    logical = logical.transpose(0, 1, 2, 4, 3, 5, 6).reshape(nb, hkv, 2, blk, d)
    k = logical[:, :, 0].transpose(0, 2, 1, 3).reshape(nb, blk, hkv * d)
    v = logical[:, :, 1].transpose(0, 2, 1, 3).reshape(nb, blk, hkv * d)
    return np.ascontiguousarray(k), np.ascontiguousarray(v)


def _q8_pos(i):
    """Place of entry i (0..15) inside a 16-byte run of a Q8_0 tile."""
    return ((i & 7) >> 1) * 4 + ((i >> 3) << 1) + (i & 1)


def unswizzle_pool_q8(raw: np.ndarray, head_dim: int):
    """Invert the Q8_0 tile layout of include/lt_kv.h -> (Kq, Vq) int8
    [block][16][kv_heads*D] and (Kd, Vd) f16 bits [block][16][kv_heads*D/32]."""
    nb, hkv, tb = raw.shape
    d = head_dim
    assert tb == 34 * d
    pos = np.array([_q8_pos(i) for i in range(16)])
    s = np.arange(BLOCK)[:, None]
    e = np.arange(d)[None, :]
    run = s * (d // 16) + e // 16
    koff = (run // 8) * 128 + ((run % 8) ^ ((run // 8) & 7)) * 16 + pos[e % 16]  # [16, D]
    voff = 16 * d + e * 16 + pos[s]  # [16, D]
    kq = raw[:, :, koff].view(np.int8)  # [nb, hkv, 16, D]
    vq = raw[:, :, voff].view(np.int8)
    g = np.arange(d // 32)[None, :]
    soff = g * 16 + pos[s]  # [16, D/32] in f16 entries
    kd = raw[:, :, 32 * d:33 * d].copy().view(np.uint16)[:, :, soff]
    vd = raw[:, :, 33 * d:34 * d].copy().view(np.uint16)[:, :, soff]
    def rows(a):
        return np.ascontiguousarray(a.transpose(0, 2, 1, 3).reshape(nb, BLOCK, -1))
    return rows(kq), rows(vq), rows(kd), rows(vd)


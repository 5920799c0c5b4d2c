"""ctypes binding of the C ABI in include/lt_kv.h (liblt_kv.so).

This is the same binding a Python host of the reference would write; the
Rust host binds the same symbols through an `extern "C"` block.
There is no fallback: if the library cannot be loaded or built, import fails.
LT_KV_VARIANT=checked|asan loads a debug build of the same sources instead
(see build.py).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

from . import build as _build

(LT_OK, LT_E_FULL, LT_E_NONCONTIG, LT_E_ARG, LT_E_CUDA, LT_E_NCCL, LT_E_TIMEOUT, LT_E_UNSUPPORTED, LT_E_SCRATCH,
 LT_E_BOUNDS) = range(10)
LT_FEATURE_BOUNDS_CHECK = 1
LT_IPC_HANDLE_BYTES = 64
LT_NOALLOC_SCRATCH_BYTES = 8 << 20
LT_NOALLOC_MAX_TOKENS = 1024
LT_F32, LT_F16 = 0, 1
LT_KV_F16, LT_KV_Q8_0 = 0, 1
BLOCK = 16

# Every function include/lt_kv.h declares (tests check the export table).
EXPORTS = (
    "lt_kv_create", "lt_kv_destroy", "lt_kv_last_error", "lt_kv_capacity", "lt_kv_bytes", "lt_kv_len",
    "lt_kv_free_blocks", "lt_kv_append", "lt_kv_write", "lt_kv_attend", "lt_kv_write_attend",
    "lt_kv_truncate", "lt_kv_share", "lt_kv_compact", "lt_kv_flush", "lt_kv_rows", "lt_kv_check",
    "lt_kv_seq_blocks", "lt_kv_refs", "lt_kv_free_list", "lt_kv_n_blocks", "lt_kv_device_pool",
    "lt_kv_device_tables", "lt_kv_read_pool", "lt_kv_launch_count", "lt_kv_profile", "lt_kv_profile_read", "lt_kv_profile_read_plan",
    "lt_kv_profile_read_write",
    "lt_kv_nccl_unique_id", "lt_kv_nccl_init", "lt_kv_nccl_destroy", "lt_kv_gather_heads",
    "lt_paged_attend_noalloc", "lt_paged_attend_noalloc_check", "lt_kv_peer_export", "lt_kv_peer_import", "lt_kv_peer_close",
    "lt_kv_attend_gather", "lt_kv_write_attend_gather", "lt_kv_selftest_wait", "lt_kv_build_features", "lt_kv_set_min_tiles_per_warp", "lt_kv_set_cascade", "lt_kv_cascade_launches",
    "lt_llama_create", "lt_llama_destroy", "lt_llama_last_error", "lt_llama_set_tensor", "lt_llama_forward",
    "lt_llama_step_greedy", "lt_llama_launch_count", "lt_llama_set_persistent", "lt_llama_persistent_available", "lt_llama_profile", "lt_llama_profile_read", "lt_q8_quantize", "lt_q8_matmul", "lt_rms_norm_q8",
    "lt_silu_q8", "lt_argmax_f32", "lt_q8_project", "lt_q8_check",
    "lt_sched_create", "lt_sched_destroy", "lt_sched_last_error", "lt_sched_submit", "lt_sched_step",
    "lt_sched_get_stats", "lt_sched_submit_tokens",
    "lt_slot_cache_create", "lt_slot_cache_destroy", "lt_slot_cache_place", "lt_slot_cache_acquire",
    "lt_slot_cache_release", "lt_slot_cache_evict_lru", "lt_slot_cache_idle_cells", "lt_slot_cache_has_free",
    "lt_slot_cache_tokens", "lt_slot_cache_slot_state", "lt_slot_cache_set_slot",
)


class lt_kv_config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32),
        ("n_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("n_heads", C.c_uint32),
        ("n_tokens", C.c_uint32),
        ("max_seqs", C.c_uint32),
        ("max_batch", C.c_uint32),
        ("max_blocks_per_seq", C.c_uint32),
        ("device", C.c_int32),
        ("kv_format", C.c_uint32),
    ]


class lt_llama_config(C.Structure):
    _fields_ = [
        ("n_layers", C.c_uint32),
        ("dim", C.c_uint32),
        ("n_heads", C.c_uint32),
        ("n_kv_heads", C.c_uint32),
        ("head_dim", C.c_uint32),
        ("ffn_dim", C.c_uint32),
        ("vocab", C.c_uint32),
        ("rope_dim", C.c_uint32),
        ("rope_neox", C.c_int32),
        ("eps", C.c_float),
        ("rope_base", C.c_float),
        ("max_batch", C.c_uint32),
        ("device", C.c_int32),
    ]


class lt_sched_config(C.Structure):
    _fields_ = [
        ("n_slots", C.c_uint32),
        ("decode_headroom", C.c_uint32),
        ("prefill_chunk", C.c_uint32),
        ("compact", C.c_int32),
        ("data", C.c_int32),
    ]


class lt_placement(C.Structure):
    _fields_ = [("slot", C.c_uint32), ("reuse", C.c_uint32), ("copy_src", C.c_int32), ("copy_len", C.c_uint32)]


class lt_sched_stats(C.Structure):
    _fields_ = [(name, C.c_uint64) for name in ("steps", "admitted", "finished", "evicted", "preempted",
                                                 "decode_tokens", "prefill_tokens", "moved_blocks")] + \
               [("running", C.c_uint32), ("queued", C.c_uint32), ("attended_positions", C.c_uint64),
                ("copies", C.c_uint64), ("prompt_tokens", C.c_uint64), ("cached_tokens", C.c_uint64)]


_lock = threading.Lock()
_lib = None


def _declare(L):
    u32, i32, u64, p, st = C.c_uint32, C.c_int32, C.c_uint64, C.c_void_p, C.c_int
    sig = {
        "lt_kv_create": (st, [C.POINTER(lt_kv_config), C.POINTER(p)]),
        "lt_kv_destroy": (None, [p]),
        "lt_kv_last_error": (C.c_char_p, [p]),
        "lt_kv_capacity": (u32, [p]),
        "lt_kv_bytes": (u64, [p]),
        "lt_kv_len": (u32, [p, u32]),
        "lt_kv_free_blocks": (u32, [p]),
        "lt_kv_n_blocks": (u32, [p]),
        "lt_kv_append": (st, [p, p, p, u32, p, p, C.POINTER(u32), p]),
        "lt_kv_write": (st, [p, u32, p, p, u32, p, p, C.c_int, p]),
        "lt_kv_attend": (st, [p, u32, p, C.c_int, p, p, u32, p, C.c_int, C.c_float, p]),
        "lt_kv_write_attend": (st, [p, u32, p, p, p, p, C.c_int, p, C.c_int, p, p, u32, p, C.c_int,
                                    C.c_float, p]),
        "lt_kv_truncate": (None, [p, u32, u32]),
        "lt_kv_share": (None, [p, u32, u32, u32]),
        "lt_kv_compact": (st, [p, C.POINTER(u32), p]),
        "lt_kv_flush": (st, [p, p]),
        "lt_kv_rows": (st, [p, u32, u32, u32, p, p, p]),
        "lt_kv_check": (st, [p, p]),
        "lt_kv_selftest_wait": (st, [p, u32, p]),
        "lt_kv_peer_export": (st, [p, C.c_int, C.c_int, u32, p]),
        "lt_kv_peer_import": (st, [p, p]),
        "lt_kv_peer_close": (st, [p]),
        "lt_kv_attend_gather": (st, [p, u32, p, C.c_int, p, p, u32, p, C.c_int, C.c_float, p]),
        "lt_kv_write_attend_gather": (st, [p, u32, p, p, p, p, C.c_int, p, C.c_int, p, p, u32, p, C.c_int,
                                           C.c_float, p]),
        "lt_kv_build_features": (u32, []),
        "lt_kv_seq_blocks": (u32, [p, u32, p, u32]),
        "lt_kv_refs": (u32, [p, p, u32]),
        "lt_kv_free_list": (u32, [p, p, u32]),
        "lt_kv_device_pool": (p, [p]),
        "lt_kv_device_tables": (p, [p, C.POINTER(u32)]),
        "lt_kv_read_pool": (st, [p, u32, u32, u32, p]),
        "lt_kv_launch_count": (u64, [p]),
        "lt_kv_set_min_tiles_per_warp": (st, [p, u32]),
        "lt_kv_set_cascade": (st, [p, u32]),
        "lt_kv_cascade_launches": (u64, [p]),
        "lt_kv_profile": (st, [p, C.c_int]),
        "lt_kv_profile_read": (st, [p, C.POINTER(C.c_double), C.POINTER(u64)]),
        "lt_kv_profile_read_plan": (st, [p, C.POINTER(C.c_double), C.POINTER(u64), C.POINTER(u64), C.POINTER(u64)]),
        "lt_kv_profile_read_write": (st, [p, C.POINTER(C.c_double), C.POINTER(u64), C.POINTER(u64), C.POINTER(u64)]),
        "lt_kv_nccl_unique_id": (st, [p]),
        "lt_kv_nccl_init": (st, [C.POINTER(p), C.c_int, p, C.c_int, C.c_int]),
        "lt_kv_nccl_destroy": (None, [p]),
        "lt_kv_gather_heads": (st, [p, p, p, p, u32, C.c_int, p, C.c_int, p]),
        "lt_paged_attend_noalloc": (st, [p, u32, u32, u32, u32, u32, p, u32, u32, p, p, u32, p, C.c_int, p,
                                         C.c_int, C.c_float, p]),
        "lt_paged_attend_noalloc_check": (st, [p]),
        "lt_llama_create": (st, [C.POINTER(lt_llama_config), C.POINTER(p)]),
        "lt_llama_destroy": (None, [p]),
        "lt_llama_last_error": (C.c_char_p, [p]),
        "lt_llama_set_tensor": (st, [p, C.c_int, u32, p, C.c_size_t]),
        "lt_llama_forward": (st, [p, p, p, p, p, u32, p, u32, p, p]),
        "lt_llama_step_greedy": (st, [p, p, p, p, p, u32, p, u32, p, p]),
        "lt_llama_launch_count": (u64, [p]),
        "lt_llama_profile": (st, [p, C.c_int]),
        "lt_llama_profile_read": (st, [p, C.POINTER(C.c_double), C.POINTER(u64), C.POINTER(u64)]),
        "lt_llama_set_persistent": (st, [p, C.c_int]),
        "lt_llama_persistent_available": (C.c_int, [p]),
        "lt_q8_quantize": (st, [p, u32, u32, p, p, p]),
        "lt_q8_matmul": (st, [p, p, u32, u32, p, p, u32, p, u32, C.c_int, p]),
        "lt_rms_norm_q8": (st, [p, p, p, u32, u32, C.c_float, p, p, p, p]),
        "lt_silu_q8": (st, [p, u32, u32, p, p, p, p]),
        "lt_argmax_f32": (st, [p, u32, u32, p, p]),
        "lt_q8_project": (st, [C.c_int, p, p, u32, u32, p, p, p, C.c_float, u32, p, u32, C.c_int, C.c_int, p]),
        "lt_q8_check": (st, [p]),
        "lt_sched_create": (st, [p, C.POINTER(lt_sched_config), C.POINTER(p)]),
        "lt_sched_destroy": (None, [p]),
        "lt_sched_last_error": (C.c_char_p, [p]),
        "lt_sched_submit": (st, [p, u32, u32]),
        "lt_sched_step": (st, [p, p, u32, p, p, C.POINTER(u32), p]),
        "lt_sched_get_stats": (st, [p, C.POINTER(lt_sched_stats)]),
        "lt_sched_submit_tokens": (st, [p, p, u32, u32, i32]),
        "lt_slot_cache_create": (st, [u32, C.POINTER(p)]),
        "lt_slot_cache_destroy": (None, [p]),
        "lt_slot_cache_place": (st, [p, p, u32, i32, C.POINTER(lt_placement)]),
        "lt_slot_cache_acquire": (st, [p, C.POINTER(lt_placement), p, u32, i32]),
        "lt_slot_cache_release": (st, [p, u32, p, u32]),
        "lt_slot_cache_evict_lru": (i32, [p]),
        "lt_slot_cache_idle_cells": (u64, [p]),
        "lt_slot_cache_has_free": (C.c_int, [p]),
        "lt_slot_cache_tokens": (u32, [p, u32, p, u32]),
        "lt_slot_cache_slot_state": (st, [p, u32, C.POINTER(i32), C.POINTER(i32), C.POINTER(u64)]),
        "lt_slot_cache_set_slot": (st, [p, u32, p, u32, i32]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def variant() -> str:
    """The library variant this process loads (LT_KV_VARIANT, default release)."""
    return os.environ.get("LT_KV_VARIANT", "release") or "release"


def lib():
    """Load liblt_kv.so (building it with nvcc first if it is missing or stale)."""
    global _lib
    with _lock:
        if _lib is None:
            path = _build.build(variant=variant())
            L = C.CDLL(str(path))
            _declare(L)
            _lib = L
    return _lib


def library_path() -> str:
    return str(_build.library(variant()))

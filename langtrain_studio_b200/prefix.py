"""Host front end of the native slot-level prefix cache (include/lt_prefix.h),
the reference engine's ``SlotCache`` (engine/crates/engine/src/prefix.rs) with
the same method names: ``place``, ``acquire``, ``release``, ``evict_lru``,
``idle_cells``, ``has_free``."""
from __future__ import annotations

import ctypes as C
from typing import NamedTuple

import numpy as np

from . import _native as N
from .kv import KvError

NO_ADAPTER = -1
MIN_COPY_GAIN = 16


class Placement(NamedTuple):
    """prefix.rs:25-31; copy_from is (source slot, length) or None."""
    slot: int
    reuse: int
    copy_from: tuple | None


def _toks(tokens) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))


class SlotCache:
    def __init__(self, n_slots: int):
        self._lib = N.lib()
        h = C.c_void_p()
        rc = self._lib.lt_slot_cache_create(n_slots, C.byref(h))
        if rc != N.LT_OK:
            raise KvError(rc, f"lt_slot_cache_create failed with status {rc}")
        self._h, self.n_slots = h, n_slots

    def close(self):
        if getattr(self, "_h", None):
            self._lib.lt_slot_cache_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def place(self, prompt, adapter: int = NO_ADAPTER) -> Placement | None:
        t = _toks(prompt)
        p = N.lt_placement()
        rc = self._lib.lt_slot_cache_place(self._h, t.ctypes.data, t.size, adapter, C.byref(p))
        if rc == N.LT_E_FULL:
            return None
        if rc != N.LT_OK:
            raise KvError(rc, "lt_slot_cache_place")
        return Placement(p.slot, p.reuse, (p.copy_src, p.copy_len) if p.copy_src >= 0 else None)

    def acquire(self, p: Placement, prompt, adapter: int = NO_ADAPTER):
        t = _toks(prompt)
        src, n = p.copy_from if p.copy_from else (-1, 0)
        pl = N.lt_placement(p.slot, p.reuse, src, n)
        rc = self._lib.lt_slot_cache_acquire(self._h, C.byref(pl), t.ctypes.data, t.size, adapter)
        if rc != N.LT_OK:
            raise KvError(rc, "lt_slot_cache_acquire")

    def release(self, slot: int, kv_tokens):
        t = _toks(kv_tokens)
        rc = self._lib.lt_slot_cache_release(self._h, slot, t.ctypes.data, t.size)
        if rc != N.LT_OK:
            raise KvError(rc, "lt_slot_cache_release")

    def evict_lru(self) -> int | None:
        i = self._lib.lt_slot_cache_evict_lru(self._h)
        return None if i < 0 else i

    def idle_cells(self) -> int:
        return self._lib.lt_slot_cache_idle_cells(self._h)

    def has_free(self) -> bool:
        return bool(self._lib.lt_slot_cache_has_free(self._h))

    def tokens(self, slot: int) -> list:
        n = self._lib.lt_slot_cache_tokens(self._h, slot, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self._lib.lt_slot_cache_tokens(self._h, slot, out.ctypes.data, n)
        return out[:n].tolist()

    def slot_state(self, slot: int):
        """(busy, adapter, last_used)."""
        busy, ad, lu = C.c_int32(), C.c_int32(), C.c_uint64()
        rc = self._lib.lt_slot_cache_slot_state(self._h, slot, C.byref(busy), C.byref(ad), C.byref(lu))
        if rc != N.LT_OK:
            raise KvError(rc, "lt_slot_cache_slot_state")
        return bool(busy.value), ad.value, lu.value

    def set_slot(self, slot: int, tokens, adapter: int = NO_ADAPTER):
        """Test hook: assign a slot's tokens and adapter (prefix.rs tests do)."""
        t = _toks(tokens)
        rc = self._lib.lt_slot_cache_set_slot(self._h, slot, t.ctypes.data, t.size, adapter)
        if rc != N.LT_OK:
            raise KvError(rc, "lt_slot_cache_set_slot")

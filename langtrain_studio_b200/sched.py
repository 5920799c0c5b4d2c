"""Host front end of the native continuous-batching driver (include/lt_sched.h).

``Scheduler`` runs the reference scheduler's KV policy (admission, LRU
eviction, preemption, chunked prefill, retire; engine/crates/engine/src/
scheduler.rs:252-473, prefix.rs:58-125) in C++ over a ``KvCache``: each
``step`` admits, frees room, claims the step's cells, writes its K/V rows,
attends the decode tokens and compacts, with no per-sequence Python work.
"""
from __future__ import annotations

import ctypes as C

from . import _native as N
from .kv import KvCache, KvError, _dptr, _stream


class Scheduler:
    def __init__(self, kv: KvCache, n_slots: int, *, decode_headroom: int = 256, prefill_chunk: int = 256,
                 compact: bool = True, data: bool = True):
        self._lib = N.lib()
        self.kv = kv
        cfg = N.lt_sched_config(n_slots=n_slots, decode_headroom=decode_headroom, prefill_chunk=prefill_chunk,
                                compact=int(compact), data=int(data))
        h = C.c_void_p()
        rc = self._lib.lt_sched_create(kv._h, C.byref(cfg), C.byref(h))
        if rc != N.LT_OK:
            raise KvError(rc, f"lt_sched_create failed with status {rc}")
        self._h = h
        self.n_slots = n_slots

    def close(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.lt_sched_destroy(h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, rc: int):
        if rc != N.LT_OK:
            raise KvError(rc, self._lib.lt_sched_last_error(self._h).decode())

    def submit(self, prompt_len: int, out_len: int):
        self._check(self._lib.lt_sched_submit(self._h, prompt_len, out_len))

    def submit_tokens(self, tokens, out_len: int, adapter: int = -1):
        """A request with its prompt token ids: admitted with prefix reuse
        (lt_sched_submit_tokens)."""
        import numpy as np

        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        self._check(self._lib.lt_sched_submit_tokens(self._h, t.ctypes.data, t.size, out_len, adapter))

    def step(self, kv_src=None, q_src=None, out=None, stream=None) -> int:
        """One scheduler step; returns the number of decode tokens."""
        nd = C.c_uint32()
        rows = kv_src.shape[0] if kv_src is not None else 0
        self._check(self._lib.lt_sched_step(self._h, _dptr(kv_src) if kv_src is not None else None, rows,
                                            _dptr(q_src) if q_src is not None else None,
                                            _dptr(out) if out is not None else None, C.byref(nd),
                                            _stream(stream) if self.kv.device >= 0 else None))
        return nd.value

    @property
    def stats(self) -> dict:
        s = N.lt_sched_stats()
        self._check(self._lib.lt_sched_get_stats(self._h, C.byref(s)))
        return {name: getattr(s, name) for name, _ in N.lt_sched_stats._fields_}

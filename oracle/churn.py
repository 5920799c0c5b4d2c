"""TEST INFRASTRUCTURE ONLY: the reference scheduler's KV policy in Python.

``ChurnDriver`` restates the slot / prefix policy of the reference's
continuous-batching scheduler (engine/crates/engine/src/scheduler.rs:252-473,
prefix.rs:58-125) in blocks, over any object with the KvCache methods it
calls (truncate, free_blocks, append_batch, write, write_attend, compact).
The native driver (include/lt_sched.h) must take exactly the same decisions;
the tests drive both with the same arrivals and compare the caches.
"""
from __future__ import annotations

import numpy as np

BLOCK = 16


class ChurnDriver:
    """The reference scheduler's KV policy restated in Python over a
    KvCache-like object (engine/crates/engine/src/scheduler.rs:252-473,
    prefix.rs:58-125):
      - admit FIFO into the least recently used idle slot while the prompt
        plus min(output, DECODE_HEADROOM=256) tokens fit, evicting idle
        slots' cached KV LRU first (kv_remove(slot, 0));
      - each step: one decode token per sequence past its prompt, prompt
        chunks of at most 256 tokens (EngineConfig.prefill_chunk);
      - before the step, free enough blocks: evict LRU idle, then preempt the
        youngest running sequence (it finishes with Length);
      - retire: a finished slot keeps its KV for prefix reuse (idle);
      - compaction every step (no reference counterpart).
    Prompt ids are random, so no prefix is ever reused; prompt tokens are
    appended and their K/V written, decode tokens run the fused
    append + attention launch (prefill attention is a later addition)."""

    HEADROOM = 256
    CHUNK = 256

    def __init__(self, kv, n_slots, kv_src, q_src):
        self.kv = kv
        self.busy = np.zeros(n_slots, bool)
        self.held = np.zeros(n_slots, np.int64)  # tokens an idle slot keeps
        self.last_used = np.zeros(n_slots, np.int64)
        self.clock = 0
        self.queue = []
        self.active = {}  # slot -> [n_past, prompt, total, admit_step]
        self.step_no = 0
        self.kv_src, self.q_src = kv_src, q_src  # device tensors the K/V/q rows are cut from
        self.stats = dict(decode=0, prefill=0, evicted=0, preempted=0, moved=0, admitted=0, finished=0)

    def _evict_lru_idle(self):
        idle = np.nonzero(~self.busy & (self.held > 0))[0]
        if idle.size == 0:
            return False
        i = int(idle[np.argmin(self.last_used[idle])])
        self.kv.truncate(i, 0)
        self.held[i] = 0
        self.stats["evicted"] += 1
        return True

    def _retire(self, slot, n_past):
        self.busy[slot] = False
        self.held[slot] = n_past
        self.clock += 1
        self.last_used[slot] = self.clock
        del self.active[slot]

    def submit(self, prompt, out):
        self.queue.append((int(prompt), int(out)))

    def _src_off(self, n):
        """The window of kv_src rows a call writes (the native driver's rule)."""
        rows = self.kv_src.shape[0]
        return (self.step_no * 2654435761) % (rows - n + 1) if rows > n else 0

    def admit(self):
        while self.queue:
            idle = np.nonzero(~self.busy)[0]
            if idle.size == 0:
                break
            prompt, out = self.queue[0]
            need = (prompt + min(out, self.HEADROOM) + BLOCK - 1) // BLOCK
            while self.kv.free_blocks() < need and self._evict_lru_idle():
                pass
            if self.kv.free_blocks() < need and self.active:
                break
            self.queue.pop(0)
            idle = np.nonzero(~self.busy)[0]
            slot = int(idle[np.argmin(self.last_used[idle])])
            self.kv.truncate(slot, 0)  # kv_remove(slot, reuse = 0): random prompts share nothing
            self.held[slot] = 0
            self.busy[slot] = True
            self.clock += 1
            self.last_used[slot] = self.clock
            self.active[slot] = [0, prompt, prompt + out, self.step_no]
            self.stats["admitted"] += 1

    def plan(self):
        """(slot, first position, token count) of this step's batch."""
        dec, pre = [], []
        for slot, (n_past, prompt, total, _) in self.active.items():
            if n_past >= prompt:
                dec.append((slot, n_past, 1))
            else:
                pre.append((slot, n_past, min(self.CHUNK, prompt - n_past)))
        return dec, pre

    @staticmethod
    def _new_blocks(items):
        n = 0
        for _, p0, cnt in items:
            n += (p0 + cnt + BLOCK - 1) // BLOCK - (p0 + BLOCK - 1) // BLOCK
        return n

    def ensure_room(self):
        while True:
            dec, pre = self.plan()
            need = self._new_blocks(dec) + self._new_blocks(pre)
            if self.kv.free_blocks() >= need:
                return dec, pre
            if self._evict_lru_idle():
                continue
            youngest = max(self.active, key=lambda s: self.active[s][3])
            self.kv.truncate(youngest, 0)  # preempted: finishes with Length, nothing kept
            self.busy[youngest] = False
            self.held[youngest] = 0
            del self.active[youngest]
            self.stats["preempted"] += 1

    def step(self, out):
        """One scheduler step; returns the number of decode tokens."""
        self.step_no += 1
        self.admit()
        dec, pre = self.ensure_room()
        kv = self.kv
        if pre:
            seqs = np.concatenate([np.full(c, s) for s, _, c in pre])
            pos = np.concatenate([np.arange(p0, p0 + c) for _, p0, c in pre])
            b, sl = kv.append_batch(seqs, pos)
            n = seqs.size
            off = self._src_off(n)
            kv.write(0, b, sl, self.kv_src[off:off + n], self.kv_src[off:off + n])
            self.stats["prefill"] += n
        nd = len(dec)
        if dec:
            seqs = np.array([s for s, _, _ in dec], np.uint32)
            pos = np.array([p for _, p, _ in dec], np.uint32)
            b, sl = kv.append_batch(seqs, pos)
            off = self._src_off(nd)
            kv.write_attend(0, b, sl, self.kv_src[off:off + nd], self.kv_src[off:off + nd], self.q_src[:nd], seqs,
                            pos, out=out[:nd])
            self.stats["decode"] += nd
        for s, p0, c in dec + pre:
            st = self.active[s]
            st[0] = p0 + c
            if st[0] >= st[2]:
                self._retire(s, st[0])
                self.stats["finished"] += 1
        self.stats["moved"] += kv.compact()
        return nd

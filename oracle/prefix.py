"""TEST INFRASTRUCTURE ONLY: the reference's slot-level prefix cache and the
scheduler's token-level admission, restated in Python.

``SlotCache`` restates engine/crates/engine/src/prefix.rs (place :58-92,
acquire :94-102, release :105-112, evict_lru :115-125, idle_cells :53-55)
with the tie-breaks of the Rust iterator adaptors it uses: ``max_by`` and
``max_by_key`` keep the last of equal maxima, ``min_by_key`` the first of
equal minima.

``PrefixDriver`` restates the KV side of the reference scheduler for
requests that carry token ids (engine/crates/engine/src/scheduler.rs:
admit :252-317 with placement and kv_copy, the step's batch :356-413 --
decode tokens first, then prompt chunks, in the order of the active list --,
ensure_kv_room :321-334, sampling's bookkeeping :414-448 and retire
:452-473, with Vec::swap_remove), counting KV room in 16-token blocks: a
step needs the blocks its tokens open plus one copy-on-write block for a
first write into a shared partial block.  Generated tokens get ids that no
prompt uses.  The native driver (lt_sched_submit_tokens) must take exactly
the same decisions.
"""
from __future__ import annotations

import numpy as np

BLOCK = 16
MIN_COPY_GAIN = 16  # prefix.rs:13
NO_ADAPTER = -1


def common_prefix(a, b) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


class SlotCache:
    """prefix.rs:33-126."""

    def __init__(self, n_slots: int):
        self.tokens = [[] for _ in range(n_slots)]
        self.adapter = [NO_ADAPTER] * n_slots
        self.busy = [False] * n_slots
        self.last_used = [0] * n_slots
        self.clock = 0

    def has_free(self) -> bool:
        return not all(self.busy)

    def idle_cells(self) -> int:
        return sum(len(t) for t, b in zip(self.tokens, self.busy) if not b)

    def place(self, prompt, adapter=NO_ADAPTER):
        """(slot, reuse, copy_src, copy_len) or None when every slot is busy."""
        cap = max(len(prompt) - 1, 0)

        def matches(i):
            return min(common_prefix(self.tokens[i], prompt), cap) if self.adapter[i] == adapter else 0

        best = None
        for i in range(len(self.tokens)):  # max_by: longest match, then least recently used; last of ties
            if self.busy[i]:
                continue
            m = matches(i)
            if best is None or m > best[1] or (m == best[1] and self.last_used[i] <= self.last_used[best[0]]):
                best = (i, m)
        if best is None:
            return None
        slot, own = best
        other = None
        for i in range(len(self.tokens)):  # max_by_key over every other slot: last of ties
            if i == slot:
                continue
            m = matches(i)
            if other is None or m >= other[1]:
                other = (i, m)
        if other is not None and other[1] >= own + MIN_COPY_GAIN:
            return slot, other[1], other[0], other[1]
        return slot, own, -1, 0

    def acquire(self, placement, prompt, adapter=NO_ADAPTER):
        slot, reuse, _, _ = placement
        self.clock += 1
        self.busy[slot] = True
        self.last_used[slot] = self.clock
        self.adapter[slot] = adapter
        self.tokens[slot] = list(prompt[:reuse])

    def release(self, slot, kv_tokens):
        self.clock += 1
        self.busy[slot] = False
        self.last_used[slot] = self.clock
        self.tokens[slot] = list(kv_tokens)

    def evict_lru(self):
        best = None
        for i in range(len(self.tokens)):  # min_by_key: the first of equal minima
            if self.busy[i] or not self.tokens[i]:
                continue
            if best is None or self.last_used[i] < self.last_used[best]:
                best = i
        if best is not None:
            self.tokens[best] = []
        return best


def _blocks(n: int) -> int:
    return (n + BLOCK - 1) // BLOCK


class PrefixDriver:
    """Token-level admission with prefix reuse over a KvCache-like object
    exposing truncate, share, free_blocks, append_batch, seq_blocks, refs
    and (optionally) compact."""

    HEADROOM = 256  # scheduler.rs DECODE_HEADROOM
    CHUNK = 256     # EngineConfig::prefill_chunk

    def __init__(self, kv, n_slots: int, compact: bool = True, kv_src=None, q_src=None):
        """kv_src / q_src (host arrays): when given, the K/V rows of the
        step's tokens are written and the decode tokens attended, cut from
        them by the native driver's rule (kv.write / kv.write_attend)."""
        self.kv = kv
        self.kv_src, self.q_src = kv_src, q_src
        self.sc = SlotCache(n_slots)
        self.queue = []
        self.active = []  # dicts: slot, tokens, n_prompt, n_past, max_total, admit, finished
        self.compact_each = compact
        self.step_no = 0
        self.admit_seq = 0
        self.gen_id = -2  # generated tokens: -2, -3, ... (prompt ids are >= 0)
        self.stats = dict(admitted=0, finished=0, evicted=0, preempted=0, copies=0, prompt_tokens=0,
                          cached_tokens=0, decode_tokens=0, prefill_tokens=0, moved_blocks=0)

    def submit(self, tokens, out_len, adapter=NO_ADAPTER):
        self.queue.append((list(tokens), int(out_len), adapter))

    def _evict(self) -> bool:
        i = self.sc.evict_lru()
        if i is None:
            return False
        self.kv.truncate(i, 0)  # Backend::kv_remove(i, 0)
        self.stats["evicted"] += 1
        return True

    def admit(self):
        while self.queue:
            toks, out, ad = self.queue[0]
            pl = self.sc.place(toks, ad)
            if pl is None:
                break
            need = _blocks(len(toks) + min(out, self.HEADROOM)) - pl[1] // BLOCK
            while self.kv.free_blocks() < need and self._evict():
                pass
            if self.kv.free_blocks() < need and self.active:
                break
            self.queue.pop(0)
            slot, reuse, src, n = pl = self.sc.place(toks, ad)  # eviction may have cleared the planned prefix
            if src >= 0:
                self.kv.truncate(slot, 0)
                self.kv.share(src, slot, n)  # Backend::kv_copy
                self.stats["copies"] += 1
            else:
                self.kv.truncate(slot, reuse)
            self.sc.acquire(pl, toks, ad)
            self.admit_seq += 1
            self.active.append(dict(slot=slot, tokens=list(toks), n_prompt=len(toks), n_past=reuse,
                                    max_total=len(toks) + out, admit=self.admit_seq, finished=False))
            self.stats["admitted"] += 1
            self.stats["prompt_tokens"] += len(toks)
            self.stats["cached_tokens"] += reuse

    def _need(self, items) -> int:
        refs = None
        n = 0
        for s, p0, cnt in items:
            n += _blocks(p0 + cnt) - _blocks(p0)
            if p0 % BLOCK:
                if refs is None:
                    refs = self.kv.refs()
                if refs[int(self.kv.seq_blocks(s["slot"])[p0 // BLOCK])] > 1:
                    n += 1  # copy-on-write of a shared partial block (kv.rs:99-110)
        return n

    def _ensure_room(self, need) -> bool:
        while self.kv.free_blocks() < need:
            if self._evict():
                continue
            live = [s for s in self.active if not s["finished"]]
            if live:
                max(live, key=lambda s: s["admit"])["finished"] = True
                self.stats["preempted"] += 1
            return False
        return True

    def _retire(self):
        i = 0
        while i < len(self.active):
            s = self.active[i]
            if not s["finished"]:
                i += 1
                continue
            self.active[i] = self.active[-1]  # Vec::swap_remove
            self.active.pop()
            self.sc.release(s["slot"], s["tokens"][:s["n_past"]])
            if s["n_past"] < len(s["tokens"]):
                self.kv.truncate(s["slot"], s["n_past"])
            self.stats["finished"] += 1

    def step(self) -> int:
        """One engine iteration (admit, step, retire); returns decode tokens."""
        self.step_no += 1
        self.admit()
        nd = 0
        if self.active:
            dec = [(s, s["n_past"], 1) for s in self.active if not s["finished"] and s["n_past"] >= s["n_prompt"]]
            pre = [(s, s["n_past"], min(s["n_prompt"] - s["n_past"], self.CHUNK)) for s in self.active
                   if not s["finished"] and s["n_past"] < s["n_prompt"]]
            if (dec or pre) and self._ensure_room(self._need(dec + pre)):
                seqs = [s["slot"] for s, _, c in dec for _ in range(c)] + \
                       [s["slot"] for s, _, c in pre for _ in range(c)]
                pos = [p0 for _, p0, _ in dec] + [p0 + k for _, p0, c in pre for k in range(c)]
                b, sl = self.kv.append_batch(seqs, pos)
                nd = len(dec)
                if self.kv_src is not None:
                    n, rows = len(pos), self.kv_src.shape[0]
                    off = (self.step_no * 2654435761) % (rows - n + 1) if rows > n else 0
                    src = self.kv_src[off:off + n]
                    if n > nd:
                        self.kv.write(0, b[nd:], sl[nd:], src[nd:], src[nd:])
                    if nd:
                        self.kv.write_attend(0, b[:nd], sl[:nd], src[:nd], src[:nd], self.q_src[:nd],
                                             np.asarray(seqs[:nd], np.uint32), np.asarray(pos[:nd], np.uint32),
                                             None)
                self.stats["decode_tokens"] += nd
                self.stats["prefill_tokens"] += len(pos) - nd
                for s, _, c in pre:
                    s["n_past"] += c
                # sample_at order: the decode tokens, then the prompts whose last chunk ran
                sampled = [s for s, _, _ in dec] + [s for s, _, _ in pre if s["n_past"] == s["n_prompt"]]
                for s in sampled:
                    if s["n_past"] >= s["n_prompt"] and s["n_past"] < len(s["tokens"]):
                        s["n_past"] += 1  # the pending token is now in KV
                    s["tokens"].append(self.gen_id)
                    self.gen_id -= 1
                    if len(s["tokens"]) >= s["max_total"]:
                        s["finished"] = True
        self._retire()
        if self.compact_each and hasattr(self.kv, "compact"):
            self.stats["moved_blocks"] += self.kv.compact()
        return nd

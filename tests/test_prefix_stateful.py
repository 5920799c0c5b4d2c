"""The native slot-level prefix cache (lt_prefix.h) against the restatement
of prefix.rs, as a hypothesis state machine.

Prompts come from a three-token alphabet, so that slots share prefixes of
every length and equal matches are common: the Rust iterator tie-breaks
(max_by / max_by_key keep the last of equal maxima, min_by_key the first of
equal minima), the len - 1 cap and the copy-gain threshold decide most
placements.  After every call both caches must hold the same tokens,
busy flags, adapters and last-used clocks, and every placement and eviction
must agree.  Besides place / acquire / release / evict, a rule assigns slot
fields directly as the reference's tests do, which builds the tied states
the other calls rarely reach.  A divergence is shrunk to a shortest call
sequence.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402
from hypothesis.stateful import RuleBasedStateMachine, invariant, rule  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from langtrain_studio_b200.prefix import Placement, SlotCache  # noqa: E402
from oracle import prefix as ref  # noqa: E402

N_SLOTS = 4
# prompts: a stem of one of two systems in a few lengths (so equal matches,
# and matches 16+ apart, are both common) plus a short tail, alphabet {0, 1, 2}
PROMPTS = st.builds(lambda stem, k, tail: [stem % 2] * k + tail,
                    st.integers(0, 1), st.sampled_from([0, 3, 20, 20, 37, 40]),
                    st.lists(st.integers(0, 2), max_size=6)).filter(len)
ADAPTERS = st.sampled_from([-1, -1, -1, 0, 1])


def _restated_placement(p):
    if p is None:
        return None
    slot, reuse, src, n = p
    return Placement(slot, reuse, (src, n) if src >= 0 else None)


class SlotCaches(RuleBasedStateMachine):
    def __init__(self):
        super().__init__()
        self.nat, self.res = SlotCache(N_SLOTS), ref.SlotCache(N_SLOTS)
        self.held = {}

    def teardown(self):
        self.nat.close()

    @rule(prompt=PROMPTS, adapter=ADAPTERS, take=st.booleans())
    def place(self, prompt, adapter, take):
        pn = self.nat.place(prompt, adapter)
        pr = _restated_placement(self.res.place(prompt, adapter))
        assert pn == pr, (pn, pr)
        if pn is not None and take:
            self.nat.acquire(pn, prompt, adapter)
            self.res.acquire((pn.slot, pn.reuse, pn.copy_from[0] if pn.copy_from else -1,
                              pn.copy_from[1] if pn.copy_from else 0), prompt, adapter)
            self.held[pn.slot] = prompt

    @rule(data=st.data(), extra=st.lists(st.integers(0, 2), max_size=30))
    def release(self, data, extra):
        """A request ends: its slot keeps a prefix of the prompt plus generated tokens."""
        if not self.held:
            return
        slot = data.draw(st.sampled_from(sorted(self.held)))
        prompt = self.held.pop(slot)
        kv = prompt[:data.draw(st.integers(0, len(prompt)))] + extra
        self.nat.release(slot, kv)
        self.res.release(slot, kv)

    @rule(data=st.data(), stem=st.integers(0, 1), k=st.sampled_from([3, 20, 37]), adapter=ADAPTERS)
    def set_slot(self, data, stem, k, adapter):
        """Assign a slot's tokens and adapter without ticking the clock, as the
        reference's own tests do (prefix.rs:159, 169): this makes equal
        matches between slots (busy ones included, half the time), and equal
        last-used clocks among slots that hold tokens, which the tie-breaks
        then decide."""
        if self.held and data.draw(st.booleans()):
            slot = data.draw(st.sampled_from(sorted(self.held)))
        else:
            slot = data.draw(st.integers(0, N_SLOTS - 1))
        tokens = [stem] * k
        self.nat.set_slot(slot, tokens, adapter)
        self.res.tokens[slot], self.res.adapter[slot] = list(tokens), adapter

    @rule()
    def evict(self):
        assert self.nat.evict_lru() == self.res.evict_lru()

    @invariant()
    def same_slots(self):
        assert self.nat.idle_cells() == self.res.idle_cells()
        assert self.nat.has_free() == self.res.has_free()
        for s in range(N_SLOTS):
            assert self.nat.tokens(s) == [int(x) for x in self.res.tokens[s]], s
            assert self.nat.slot_state(s) == (self.res.busy[s], self.res.adapter[s], self.res.last_used[s]), s


SlotCaches.TestCase.settings = settings(max_examples=200, stateful_step_count=50, deadline=None,
                                        suppress_health_check=[HealthCheck.too_slow, HealthCheck.filter_too_much],
                                        database=None)
test_slot_cache_state_machine = SlotCaches.TestCase

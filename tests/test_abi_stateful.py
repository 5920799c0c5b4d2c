"""Host bookkeeping of the C ABI against the oracle, as a hypothesis state
machine.

Rules are the calls the reference scheduler makes through Backend::{decode,
kv_remove, kv_copy} (batched append with the occasional non-contiguous
position, truncate, share) plus compaction.  After every rule the native
handle (bookkeeping only, no GPU) and the oracle restatement of kv.rs must
agree bit for bit: status codes and n_done of failed batches, the (block,
slot) cells, every table, every refcount and the free list in order.  A
divergence is shrunk to a shortest failing call sequence.  The pool is kept
small so that "KV cache full", copy-on-write of shared partial blocks and
compaction moves come up in most runs.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import HealthCheck, settings  # noqa: E402
from hypothesis import strategies as st  # noqa: E402
from hypothesis.stateful import RuleBasedStateMachine, invariant, rule  # noqa: E402

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from langtrain_studio_b200.kv import KvCache, KvError  # noqa: E402
from oracle import oracle  # noqa: E402

MAX_SEQS = 6
POOL_BLOCKS = 24


class Bookkeeping(RuleBasedStateMachine):
    def __init__(self):
        super().__init__()
        oracle.build()
        self.kv = KvCache(2, 1, 64, 16 * POOL_BLOCKS, n_heads=1, max_seqs=MAX_SEQS, max_batch=4096, device=-1)
        self.ok = oracle.OracleKv(2, 64, 16 * POOL_BLOCKS, max_seqs=MAX_SEQS)

    def teardown(self):
        self.kv.close()

    @rule(runs=st.lists(st.tuples(st.integers(0, MAX_SEQS - 1), st.integers(1, 40)), min_size=1, max_size=4),
          gap=st.sampled_from([0, 0, 0, 0, 1, 2]))
    def append_batch(self, runs, gap):
        """One decode/prefill batch: each run is `count` consecutive positions
        of one sequence; a non-zero gap shifts the last run's first position."""
        seqs, pos, lens = [], [], {}
        for i, (s, count) in enumerate(runs):
            start = lens.get(s, self.kv.len(s)) + (gap if i == len(runs) - 1 else 0)
            seqs += [s] * count
            pos += list(range(start, start + count))
            lens[s] = start + count
        rc, done, blocks_o, slots_o = self.ok.append_batch(seqs, pos)
        try:
            blocks, slots = self.kv.append_batch(seqs, pos)
        except KvError as e:
            assert (e.code, e.n_done) == (rc, done), (str(e), rc, done)
            return
        assert rc == 0 and done == len(seqs)
        assert np.array_equal(blocks, blocks_o) and np.array_equal(slots, slots_o)

    @rule(seq=st.integers(0, MAX_SEQS - 1), back=st.integers(-3, 40))
    def truncate(self, seq, back):
        """kv_remove(seq, from): from below, at or past the length."""
        frm = max(self.kv.len(seq) - back, 0)
        self.kv.truncate(seq, frm)
        self.ok.truncate(seq, frm)

    @rule(src=st.integers(0, MAX_SEQS - 1), dst=st.integers(0, MAX_SEQS - 1), cut=st.integers(-5, 60))
    def share(self, src, dst, cut):
        """kv_copy(src, dst, len): len inside, at, or past src's length."""
        length = max(self.kv.len(src) - cut, 0)
        self.kv.share(src, dst, length)
        self.ok.share(src, dst, length)

    @rule()
    def compact(self):
        assert self.kv.compact() == len(self.ok.compact())

    @invariant()
    def same_state(self):
        kv, ok = self.kv, self.ok
        assert kv.free_blocks() == ok.free_blocks()
        assert np.array_equal(kv.free_list(), ok.free_list())
        assert np.array_equal(kv.refs(), ok.refs())
        for s in range(MAX_SEQS):
            assert kv.len(s) == ok.len(s), s
            assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s)), s


Bookkeeping.TestCase.settings = settings(max_examples=150, stateful_step_count=40, deadline=None,
                                         suppress_health_check=[HealthCheck.too_slow], database=None)
test_bookkeeping_state_machine = Bookkeeping.TestCase

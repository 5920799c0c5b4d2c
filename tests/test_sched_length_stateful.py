"""The native driver with length-only requests (lt_sched_submit, the
config 5 churn policy) against its restatement (oracle/churn.py), as a
hypothesis state machine.

Rules: submit a request of a prompt length and an output length, or run a
few steps.  On a small pool admission waits, idle slots' KV is evicted,
steps preempt the youngest sequence and compaction moves blocks.  After every
rule both drivers must agree on every counter and on the running and queued
counts, and both caches on their tables, refcounts and free list.
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
sys.path.insert(0, str(ROOT / "tests"))

from langtrain_studio_b200.kv import KvCache  # noqa: E402
from langtrain_studio_b200.sched import Scheduler  # noqa: E402
from oracle import churn, oracle  # noqa: E402
from test_sched import KEYS, _OracleBookkeeping  # noqa: E402

SLOTS = 6
POOL = 24  # blocks


class LengthRequests(RuleBasedStateMachine):
    def __init__(self):
        super().__init__()
        oracle.build()
        self.kv = KvCache(1, 2, 64, POOL * 16, n_heads=4, max_seqs=SLOTS, max_batch=1 << 14,
                          max_blocks_per_seq=POOL, device=-1)
        self.sched = Scheduler(self.kv, SLOTS, data=False)
        self.ok = oracle.OracleKv(1, 2 * 64, POOL * 16, max_seqs=SLOTS)
        self.drv = churn.ChurnDriver(_OracleBookkeeping(self.ok), SLOTS, np.zeros((4096, 1)), np.zeros((SLOTS, 1)))

    def teardown(self):
        self.sched.close()
        self.kv.close()

    @rule(prompt=st.integers(1, 200), out=st.integers(1, 60))
    def submit(self, prompt, out):
        self.sched.submit(prompt, out)
        self.drv.submit(prompt, out)

    @rule(n=st.integers(1, 10))
    def step(self, n):
        for _ in range(n):
            self.sched.step()
            self.drv.step(np.zeros((SLOTS, 1)))

    @invariant()
    def same_state(self):
        s = self.sched.stats
        for k_py, k_c in KEYS:
            assert self.drv.stats[k_py] == s[k_c], (k_py, self.drv.stats[k_py], s[k_c])
        assert s["running"] == len(self.drv.active) and s["queued"] == len(self.drv.queue)
        assert np.array_equal(self.kv.free_list(), self.ok.free_list())
        assert np.array_equal(self.kv.refs(), self.ok.refs())
        for q in range(SLOTS):
            assert np.array_equal(self.kv.seq_blocks(q), self.ok.seq_blocks(q)), q


LengthRequests.TestCase.settings = settings(max_examples=120, stateful_step_count=40, deadline=None,
                                            suppress_health_check=[HealthCheck.too_slow], database=None)
test_length_requests_state_machine = LengthRequests.TestCase

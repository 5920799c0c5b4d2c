"""Token-level admission of the native scheduler driver (lt_sched with
lt_sched_submit_tokens) against its restatement of scheduler.rs + prefix.rs
(oracle/prefix.py PrefixDriver), as a hypothesis state machine.

Rules: submit a chat-like request (one of two shared system prompts, a user
turn drawn from a small alphabet so turns repeat, an output length, an
adapter id), or run one scheduler step.  The pool is small, so admission
evicts idle prefixes, steps preempt the youngest sequence and prefix copies
(kv_copy) compete for blocks.  After every rule the two drivers must agree
on every counter (admitted, finished, evicted, preempted, copies, prompt and
cached tokens, decode and prefill tokens, moved blocks), on the running and
queued counts, and on the cache's tables, refcounts and free list.
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
from oracle import oracle  # noqa: E402
from oracle import prefix as ref  # noqa: E402
from test_prefix import KEYS, _OracleKv  # noqa: E402

SLOTS = 4
POOL = 16  # blocks: about two prompts with their replies
SYSTEMS = [((np.arange(40 + 24 * k) * 7 + k) % 1000).astype(np.int32) for k in range(2)]


class TokenAdmission(RuleBasedStateMachine):
    def __init__(self):
        super().__init__()
        oracle.build()
        self.kv = KvCache(1, 2, 64, POOL * 16, n_heads=4, max_seqs=SLOTS, max_batch=1 << 14,
                          max_blocks_per_seq=POOL, device=-1)
        self.sched = Scheduler(self.kv, SLOTS, prefill_chunk=32, data=False)
        self.ok = oracle.OracleKv(1, 2 * 64, POOL * 16, max_seqs=SLOTS)
        self.drv = ref.PrefixDriver(_OracleKv(self.ok), SLOTS)
        self.drv.CHUNK = 32  # the same prefill chunk as the native driver

    def teardown(self):
        self.sched.close()
        self.kv.close()

    @rule(system=st.integers(0, 1), user=st.lists(st.integers(1000, 1003), min_size=1, max_size=40),
          out_len=st.integers(1, 30), adapter=st.sampled_from([-1, -1, -1, 0]))
    def submit(self, system, user, out_len, adapter):
        prompt = np.concatenate([SYSTEMS[system], np.asarray(user, np.int32)])
        self.sched.submit_tokens(prompt, out_len, adapter)
        self.drv.submit(prompt, out_len, adapter)

    @rule(n=st.integers(1, 12))
    def step(self, n):
        for _ in range(n):
            self.sched.step()
            self.drv.step()

    @invariant()
    def same_state(self):
        s = self.sched.stats
        for k in KEYS:
            assert self.drv.stats[k] == s[k], (k, self.drv.stats[k], s[k])
        assert s["running"] == len(self.drv.active) and s["queued"] == len(self.drv.queue)
        assert np.array_equal(self.kv.free_list(), self.ok.free_list())
        assert np.array_equal(self.kv.refs(), self.ok.refs())
        for q in range(SLOTS):
            assert np.array_equal(self.kv.seq_blocks(q), self.ok.seq_blocks(q)), q


TokenAdmission.TestCase.settings = settings(max_examples=150, stateful_step_count=40, deadline=None,
                                            suppress_health_check=[HealthCheck.too_slow], database=None)
test_token_admission_state_machine = TokenAdmission.TestCase

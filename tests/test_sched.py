"""CPU test of the native continuous-batching driver (include/lt_sched.h).

The driver runs the reference scheduler's KV policy in C++ over a
bookkeeping-only cache (no device).  The same arrivals go to the Python
restatement of the policy (oracle/churn.py) over the oracle's KvCache.
After every step both caches must hold the same tables, refcounts and free
list, bit for bit, and both drivers the same counts of admissions,
retirements, evictions, preemptions, tokens and moved blocks.
"""
import numpy as np
import pytest

import bench
from langtrain_studio_b200.kv import KvCache
from langtrain_studio_b200.sched import Scheduler
from oracle import churn


class _OracleBookkeeping:
    """KvCache facade over the oracle, bookkeeping only."""

    def __init__(self, ok):
        self.ok = ok

    def free_blocks(self):
        return self.ok.free_blocks()

    def truncate(self, s, frm):
        self.ok.truncate(s, frm)

    def append_batch(self, seqs, pos):
        rc, done, b, sl = self.ok.append_batch(seqs, pos)
        assert rc == 0
        return b, sl

    def write(self, *args, **kw):
        pass

    def write_attend(self, *args, **kw):
        pass

    def compact(self):
        return len(self.ok.compact())


KEYS = [("admitted", "admitted"), ("finished", "finished"), ("evicted", "evicted"), ("preempted", "preempted"),
        ("decode", "decode_tokens"), ("prefill", "prefill_tokens"), ("moved", "moved_blocks")]


@pytest.mark.parametrize("seed,lam,pool,slots", [(1, 1.5, 96, 24), (2, 3.0, 160, 40), (3, 0.7, 64, 12)])
def test_native_scheduler_matches_policy_restatement(oracle_mod, seed, lam, pool, slots):
    kv = KvCache(1, 2, 64, pool * 16, n_heads=4, max_seqs=slots, max_batch=1 << 14, max_blocks_per_seq=64,
                 device=-1)
    sched = Scheduler(kv, slots, data=False)
    ok = oracle_mod.OracleKv(1, 2 * 64, pool * 16, max_seqs=slots)
    drv = churn.ChurnDriver(_OracleBookkeeping(ok), slots, np.zeros((4096, 1)), np.zeros((slots, 1)))
    arr = bench.Arrivals(lam, seed, lo=8, hi=400, olo=4, ohi=60)
    for step in range(150):
        for p, o in arr.step():
            sched.submit(p, o)
            drv.submit(p, o)
        sched.step()
        drv.step(np.zeros((slots, 1)))
        st = sched.stats
        for k_py, k_c in KEYS:
            assert drv.stats[k_py] == st[k_c], (step, k_py, drv.stats[k_py], st[k_c])
        assert st["running"] == len(drv.active) and st["queued"] == len(drv.queue)
        assert np.array_equal(kv.free_list(), ok.free_list()), step
        assert np.array_equal(kv.refs(), ok.refs()), step
        for s in range(slots):
            assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s)), (step, s)
    st = sched.stats
    assert st["evicted"] > 0 and st["finished"] > 0 and st["moved_blocks"] > 0, st
    sched.close()

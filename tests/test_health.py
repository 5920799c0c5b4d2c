"""Host-side failure detection across ranks (langtrain_studio_b200/health.py), on CPU with gloo.

Two ranks beat and check a few steps. Then rank 1 leaves between steps: announced (``leave()``)
in one case, silent in the other (the process exits without a word). Rank 0 must learn of it
on the host before its next step, at once or within the heartbeat timeout, instead of blocking
in its next collective.
"""
import os
import socket
import time

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, out_dir, mode):
    import datetime
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from langtrain_studio_b200.health import PeerLost, RankHealth

    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=30))
    h = RankHealth(store, rank, world, timeout_s=0.5)
    for step in range(3):  # healthy steps
        h.beat(step)
        h.check(step)
    if rank == 1:
        if mode == "announced":
            h.leave()
        store.set("lt_test/rank1_gone", "1")
        return  # silent: no further beat, the process simply ends
    store.wait(["lt_test/rank1_gone"])
    h.beat(3)
    t0 = time.monotonic()
    try:
        h.check(3)
        result = "no error"
    except PeerLost as e:
        result = f"{e.reason}|{e.ranks}"
    waited = time.monotonic() - t0
    with open(os.path.join(out_dir, "rank0.txt"), "w") as f:
        f.write(f"{result}\n{waited}\n")


@pytest.mark.parametrize("mode", ["announced", "silent"])
def test_peer_that_leaves_is_detected_between_steps(tmp_path, mode):
    mp.start_processes(_rank, args=(2, _free_port(), str(tmp_path), mode), nprocs=2, join=True,
                       start_method="spawn")
    result, waited = open(tmp_path / "rank0.txt").read().split("\n")[:2]
    waited = float(waited)
    if mode == "announced":
        assert result == "left|[1]", result
        assert waited < 0.4, waited  # at once, not after the timeout
    else:
        assert result.startswith("sent no heartbeat") and result.endswith("|[1]"), result
        assert 0.5 <= waited < 3.0, waited

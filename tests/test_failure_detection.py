"""Failure detection on the host (gloo ranks on CPU; no GPU is faulted or hung).

* a rank that stops heart-beating (killed between steps) is reported by the
  survivors' watchdog before their next step;
* a rank that never joins is reported;
* a collective whose peer has died ends with an error after the process
  group's (short) timeout instead of hanging.
"""
import os
import time

import torch
import torch.distributed as dist

from dist_util import run_ranks


def _dead_rank_worker(rank, world):
    from mini_megatron_b200.utils.watchdog import Heartbeat, RankFailure
    hb = Heartbeat(interval=0.1, timeout=1.0).start()
    t = torch.ones(4)
    dist.all_reduce(t)          # step 1: everyone alive
    dist.barrier()
    if rank == world - 1:
        os._exit(0)            # dies between steps: no more heartbeats, no exit announcement
    deadline = time.time() + 20
    detected = None
    while time.time() < deadline:
        try:
            hb.check()
        except RankFailure as e:
            detected = e.ranks
            break
        time.sleep(0.1)
    hb.stop()
    os._exit(0 if detected == [world - 1] else 3)


def test_watchdog_detects_dead_rank():
    errs, codes = run_ranks(_dead_rank_worker, 3, timeout_s=60, expect_fail=True)
    assert codes == [0, 0, 0], (codes, errs)


def _announced_exit_worker(rank, world):
    from mini_megatron_b200.utils.watchdog import Heartbeat, RankFailure
    hb = Heartbeat(interval=0.1, timeout=30.0).start()
    dist.barrier()
    if rank == 1:
        hb.announce_exit()
        hb.stop()
        os._exit(0)
    deadline = time.time() + 10
    while time.time() < deadline:
        try:
            hb.check()
        except RankFailure as e:
            hb.stop()
            os._exit(0 if e.ranks == [1] and "announced" in e.reason else 4)
        time.sleep(0.05)
    os._exit(5)


def test_watchdog_reports_announced_exit_quickly():
    errs, codes = run_ranks(_announced_exit_worker, 2, timeout_s=60, expect_fail=True)
    assert codes == [0, 0], (codes, errs)


def _collective_timeout_worker(rank, world):
    dist.barrier()
    if rank == 1:
        os._exit(0)
    t0 = time.time()
    try:
        dist.all_reduce(torch.ones(2))
        code = 6  # should not complete
    except Exception:  # noqa: BLE001 -- gloo raises once the peer is gone / the timeout expires
        code = 0 if time.time() - t0 < 30 else 7
    os._exit(code)


def test_collective_with_dead_peer_errors_instead_of_hanging():
    errs, codes = run_ranks(_collective_timeout_worker, 2, timeout_s=5, expect_fail=True)
    assert codes == [0, 0], (codes, errs)


def test_never_joined_rank_reported():
    from mini_megatron_b200.utils.watchdog import Heartbeat, RankFailure
    store = dist.HashStore()
    hb = Heartbeat(store=store, rank=0, world=2, interval=0.05, timeout=0.3).start()
    time.sleep(1.0)
    try:
        hb.check()
        raise AssertionError("missing rank not reported")
    except RankFailure as e:
        assert e.ranks == [1] and "never joined" in e.reason
    finally:
        hb.stop()

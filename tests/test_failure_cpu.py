"""Failure detection of the multi-rank path, on CPU ranks (gloo), without any GPU.

A rank leaves between steps -- cleanly (it announces it) or abruptly (the process exits with
no clean-up, so its heartbeat stops) -- and the surviving rank must learn of it on the host
through tops.distributed.PeerWatchdog before it launches its next collective, the way
NcclStateExchange checks before every state exchange (it then aborts its NCCL communicator
instead of enqueueing work that would wait for the lost peer).  A collective issued anyway
must end with an error under the process group's short timeout rather than block.
"""
from __future__ import annotations

import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    sys.path[:0] = [str(ROOT), str(ROOT / "pallas-kernel_b200")]
    import datetime

    import torch
    import torch.distributed as dist
    from tops import distributed as TD

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    wd = TD.PeerWatchdog(timeout=1.5, interval=0.05)
    t = torch.ones(4)
    dist.all_reduce(t)  # step 1: every rank takes part
    time.sleep(0.3)
    wd.check()          # nobody is lost yet
    if rank == world - 1:  # the leaving rank: between steps, nothing in flight
        out[rank] = "left"
        if mode == "crash":
            os._exit(0)  # no close(), no destroy: its heartbeat just stops
        wd.close()
        return
    t0 = time.monotonic()
    res = ("not detected",)
    while time.monotonic() - t0 < 15:
        try:
            wd.check()
        except TD.PeerLostError as e:
            res = ("lost", str(e), time.monotonic() - t0)
            break
        time.sleep(0.02)
    if mode == "collective":  # a collective issued anyway ends with an error, it does not block
        t1 = time.monotonic()
        try:
            dist.all_reduce(t)
            res = res + ("collective returned",)
        except Exception as e:  # gloo: connection closed by the peer, or the timeout
            res = res + (f"collective failed: {type(e).__name__}", time.monotonic() - t1)
    out[rank] = res
    wd.close()
    os._exit(0)  # the group cannot be torn down collectively without the lost rank


@pytest.mark.timeout(120)
@pytest.mark.parametrize("mode", ["leave", "crash", "collective"])
def test_lost_peer_is_detected_on_the_host(mode):
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, out)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=90)
        assert pr.exitcode == 0, f"rank exited with {pr.exitcode}"
    assert out[1] == "left"
    res = out[0]
    assert res[0] == "lost", res
    assert "rank 1" in res[1], res
    limit = 1.0 if mode == "leave" else 1.5 + 2.0  # announced: at once; silent: the heartbeat timeout
    assert res[2] < limit, res
    if mode == "collective":
        assert res[3].startswith("collective failed"), res
        assert res[4] < 12.0, res  # within the process group's 10 s timeout (plus slack)


def test_watchdog_without_peers_stays_quiet():
    """A single-rank group has no peers to lose; check() never raises and close() is clean."""
    import datetime

    import torch.distributed as dist
    sys.path[:0] = [str(ROOT / "pallas-kernel_b200")]
    from tops import distributed as TD
    store = dist.HashStore()
    wd = TD.PeerWatchdog(store=store, rank=0, world=1, timeout=0.2, interval=0.02)
    time.sleep(0.3)
    wd.check()
    wd.close()
    assert store.get("tops_gla/heartbeat/0") == b"left"
    del datetime

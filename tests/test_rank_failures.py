"""Rank failures in a multi-process run, made on the host (CPU, `gloo`).

The multi-GPU tests run one process per rank through `ranks.run_workers`.
A rank that raises, or dies without reporting, leaves the others blocked in
a collective it never joins; the runner must report the failed rank and stop
the others within seconds, not wait for the collective's timeout.  No GPU is
involved: the failures are an exception and an early process exit.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist

from ranks import run_workers


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, bad_rank, queue):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
        if rank == bad_rank and mode == "raise":
            raise RuntimeError("planted failure before the collective")
        if rank == bad_rank and mode == "exit":
            os._exit(3)  # dies without reporting
        t = torch.full((4,), float(rank + 1))
        dist.all_reduce(t)
        queue.put((rank, t.tolist(), None))
    except Exception as e:
        queue.put((rank, None, f"{type(e).__name__}: {e}"))


def test_all_ranks_report():
    out = run_workers(_worker, 3, (free_port(), "ok", -1), timeout=120)
    assert out == {r: [6.0] * 4 for r in range(3)}


@pytest.mark.parametrize("mode,expect", [("raise", "planted failure"), ("exit", "exited with code 3")])
def test_a_failed_rank_stops_the_run_quickly(mode, expect):
    t0 = time.monotonic()
    with pytest.raises(AssertionError) as err:
        run_workers(_worker, 3, (free_port(), mode, 1), timeout=120)
    # the other ranks sat in all_reduce; they were stopped, not waited for
    # (a peer may report the broken connection first; the dead rank is named)
    assert time.monotonic() - t0 < 60
    msg = str(err.value)
    assert "rank 1: " in msg and expect in msg, msg


def test_a_silent_hang_is_bounded():
    # no rank fails, but the run exceeds its time limit: every rank is stopped
    t0 = time.monotonic()
    with pytest.raises(AssertionError) as err:
        run_workers(_sleeper, 2, (), timeout=3)
    assert time.monotonic() - t0 < 60 and "no result within 3 s" in str(err.value)


def _sleeper(rank, world, queue):
    time.sleep(300)

"""Failure detection of the data-parallel plumbing, on CPU ranks (gloo).

A rank that dies, raises, or stays alive without joining a collective must
turn the survivors' next collective into an error within the process group's
timeout (``init_from_env(timeout_s=...)``), never into a hang.  The failures
are made on the host: nothing here touches a GPU.
"""

from __future__ import annotations

import os
import socket
import time

import pytest
import torch
import torch.multiprocessing as mp

TIMEOUT_S = 5.0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, port: int, q, mode: str) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    from mround_b200.pipeline.dist import init_from_env

    ctx = init_from_env("gloo", timeout_s=TIMEOUT_S)
    ctx.barrier()  # both ranks are up before the failure
    if rank == 1:
        if mode == "exit":
            os._exit(0)  # dies without leaving the group
        if mode == "raise":
            raise SystemExit(3)  # an exception ends the rank between steps
        if mode == "absent":
            time.sleep(3 * TIMEOUT_S)  # alive, but never joins the collective
            os._exit(0)
    t0 = time.monotonic()
    try:
        ctx.all_reduce_(torch.ones(4))
        q.put(("completed", time.monotonic() - t0))
    except Exception as exc:  # noqa: BLE001 - the error itself is what is observed
        q.put((type(exc).__name__, time.monotonic() - t0))
    q.close()
    q.join_thread()  # the result reaches the parent before the process ends
    os._exit(0)  # without tearing down a group whose peer is gone


@pytest.mark.parametrize("mode", ["exit", "raise", "absent"])
def test_survivor_sees_an_error_not_a_hang(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        outcome, seconds = q.get(timeout=60)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
    assert outcome != "completed", "the collective cannot complete without the peer"
    assert seconds < 4 * TIMEOUT_S, f"the error took {seconds:.1f} s"

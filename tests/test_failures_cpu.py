"""Failure detection of the multi-rank host path, on CPU ranks (gloo).

Failures are made on the host, as the step would meet them: a rank that
leaves without joining the next collective, and a rendezvous that cannot
complete.  Each must end in an exception within the configured bound, never
in a hang (the GPU-side counterpart -- a bounded device wait that runs out --
is ``test_withheld_partial_times_out_and_the_plan_recovers``).
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import time

import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, leave: bool, q):
    import torch

    import __graft_entry__

    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                          WORLD_SIZE=str(world))
        pkg = __graft_entry__.load_package()
        from dflash_mlx_b200.verify_step import init_process_group

        group = init_process_group("gloo", timeout_s=5)
        if leave:
            q.put((rank, "left", 0.0))
            q.close()
            q.join_thread()        # the message is out before the process is
            os._exit(0)            # gone before the exchange, without a word
        keys = torch.arange(8, dtype=torch.int64)
        t0 = time.time()
        try:
            pkg.lm_head.gather_keys(keys, group)
            q.put((rank, "no error", time.time() - t0))
        except Exception as e:  # noqa: BLE001
            q.put((rank, "error: " + type(e).__name__, time.time() - t0))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "setup failed: " + repr(e), 0.0))


def test_a_rank_that_leaves_ends_the_peers_exchange_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, r == 1, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 120
    while len(results) < 2 and time.time() < deadline:
        try:
            r, what, dt = q.get(timeout=5)
            results[r] = (what, dt)
        except Exception:  # noqa: BLE001 - queue poll
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results.get(1, ("?",))[0] == "left", results
    what, dt = results.get(0, ("missing", 0.0))
    assert what.startswith("error"), results
    assert dt < 60


def _init_only(port: int, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK="1", WORLD_SIZE="2")
        import __graft_entry__

        __graft_entry__.load_package()
        from dflash_mlx_b200.verify_step import init_process_group

        t0 = time.time()
        try:
            init_process_group("gloo", timeout_s=3)
            q.put(("started", time.time() - t0, ""))
        except RuntimeError as e:
            q.put(("raised", time.time() - t0, str(e)))
    except Exception as e:  # noqa: BLE001
        q.put(("setup failed", 0.0, repr(e)))


def test_a_rendezvous_that_cannot_complete_raises_within_its_bound():
    # rank 1 of 2 with no rank 0 (no store listening at the port)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_init_only, args=(_free_port(), q))
    p.start()
    try:
        what, dt, msg = q.get(timeout=120)
    finally:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert what == "raised", (what, msg)
    assert "did not start within 3 s" in msg
    assert dt < 60

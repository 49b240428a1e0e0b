"""The N > 1 plumbing of bench.py on CPU ranks (gloo, world size 2): the barrier, the max-over-ranks timing that
`value` is computed from, and that a rank which leaves makes the others' next collective fail after the process
group's timeout instead of hanging (failure detected on the host, no GPU involved)."""

import multiprocessing as mp
import os
import socket
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, mode, q):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    sys.path.insert(0, ROOT)
    import bench

    d = bench.Dist(backend="gloo", timeout_s=5 if mode == "leave" else 60)
    d.init()
    try:
        if mode == "max":
            d.barrier()
            m = d.max(10.0 * (rank + 1))
            q.put((rank, "ok", m))
        elif mode == "leave":
            d.barrier()
            if rank == 1:
                q.put((rank, "left", None))
                q.close()
                q.join_thread()  # the message is sent before the rank disappears
                os._exit(0)  # leaves between steps, with nothing in flight
            t0 = time.time()
            try:
                d.barrier()
                q.put((rank, "no-error", time.time() - t0))
            except Exception as e:  # noqa: BLE001 -- the collective's error is the detection
                q.put((rank, "detected", (time.time() - t0, type(e).__name__)))
    finally:
        if mode != "leave":
            d.close()


def run_ranks(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    deadline = time.time() + timeout
    while len(out) < world and time.time() < deadline:
        try:
            r, status, val = q.get(timeout=1)
            out[r] = (status, val)
        except Exception:  # noqa: BLE001
            pass
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return out


def test_max_over_ranks_and_barrier():
    out = run_ranks("max")
    assert out == {0: ("ok", 20.0), 1: ("ok", 20.0)}


def test_rank_that_leaves_is_detected_by_timeout():
    out = run_ranks("leave")
    assert out[1][0] == "left"
    status, val = out[0]
    assert status == "detected", out
    assert val[0] < 60

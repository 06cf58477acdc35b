"""Host-side failure detection across ranks, on CPU (gloo), without any GPU:
the benchmark's rank plumbing (bench.Dist) runs a step loop of the
expert-parallel exchange pattern (an all-to-all of slabs, then the step's
barrier and max-over-ranks); one rank leaves between steps -- it raises, or it
exits without a word -- and the surviving rank's next collective ends with an
error within the process group's short time-out instead of hanging.  A rank
that never joins makes the others' set-up fail the same way."""
import os
import socket
import sys
import time

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank(rank, world, port, mode, q):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import bench
    t0 = time.time()
    try:
        if mode == "never_joins" and rank == 1:
            time.sleep(30)
            q.put((rank, "absent", 0.0))
            return
        d = bench.Dist(world, rank, "gloo", timeout_s=4.0)
        td = d.td
        for step in range(6):
            if step == 3 and rank == 1:
                if mode == "raises":
                    raise RuntimeError("rank 1 failed between steps")
                os._exit(0)                  # leaves without a word (no process-group shutdown)
            slab = torch.full((world * 16,), float(rank * 100 + step))
            got = torch.empty_like(slab)
            td.all_to_all_single(got, slab)  # the exchange of a step
            d.barrier()
            d.max(float(step))
        q.put((rank, "finished", time.time() - t0))
    except Exception as e:                   # what the surviving rank reports
        q.put((rank, f"error: {type(e).__name__}", time.time() - t0))


@pytest.mark.parametrize("mode", ["raises", "exits", "never_joins"])
def test_survivor_reports_error_not_hang(mode):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {}
    deadline = time.time() + 120
    while len(got) < 2 and time.time() < deadline:
        try:
            r, what, dt = q.get(timeout=5)
            got[r] = (what, dt)
        except Exception:
            if mode == "exits" and 0 in got and not procs[1].is_alive():
                break                        # rank 1 left without reporting, by design
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert 0 in got, f"rank 0 never reported (it hung): {got}"
    what, dt = got[0]
    assert what.startswith("error"), got
    assert dt < 90, f"rank 0 took {dt:.0f} s to notice"
    if mode == "raises":
        assert got.get(1, ("",))[0].startswith("error")

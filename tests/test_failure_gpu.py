"""Failure detection on the device without a fault: a bounded device wait that
cannot be satisfied returns the E4B_ST_TIMEOUT status within its limit, and the
context stays usable afterwards.

The wait is e4b_ep_wait (the expert-parallel peer-memory transport's epoch
wait) on a flag array that no peer writes: one GPU, no peer mapping, nothing
in flight but this one kernel.  The limit is shortened with the context option
"wait_limit_us", so the test spends ~50 ms waiting."""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
E4B_ST_TIMEOUT = 2


def test_ep_wait_times_out_and_context_survives(e4b, dev):
    assert dev.status() == 0
    flags = dev.alloc(8 * 4)                        # two peers' flags, both 0: nobody ever writes them
    ctr = dev.upload(np.array([1], np.uint32))      # this rank's epoch 1: the wait needs flag >= 1
    dev.call("e4b_set_option", b"wait_limit_us", 50_000)
    try:
        t0 = time.time()
        dev.call("e4b_ep_wait", flags.ptr, ctr.ptr, 2)
        dev.sync()
        dt = time.time() - t0
    finally:
        dev.call("e4b_set_option", b"wait_limit_us", 1_000_000)
    assert dev.status() == E4B_ST_TIMEOUT           # reading the word also clears it
    assert dt < 5.0, f"the 50 ms wait took {dt:.2f} s"
    # the context still runs kernels: a satisfied wait (flags raised on the host) ...
    dev.write(flags, np.array([1, 1], np.uint32))
    dev.call("e4b_ep_wait", flags.ptr, ctr.ptr, 2)
    dev.sync()
    assert dev.status() == 0
    # ... and an ordinary operator, checked against numpy
    x = np.linspace(-1, 1, 512, dtype=np.float32)
    w = np.full(512, 1.0, np.float32)
    bx, bw, by = dev.upload(x), dev.upload(w), dev.alloc(512 * 4)
    e4b.ops.rmsnorm(dev, bx, bw, by, None, None, DIM=512)
    dev.sync()
    y = dev.read(by, np.float32, 512)
    ref = x / np.sqrt(np.mean(x.astype(np.float64) ** 2) + 1e-6)
    assert np.max(np.abs(y - ref)) < 1e-5
    assert dev.status() == 0


def test_wait_limit_option_bounds(e4b, dev):
    with pytest.raises(e4b.E4BError):
        dev.call("e4b_set_option", b"wait_limit_us", 10)
    with pytest.raises(e4b.E4BError):
        dev.call("e4b_set_option", b"attn_grid_cap", -1)

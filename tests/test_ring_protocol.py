"""The sliding-window KV ring protocol as property tests (the invariants of the
reference's specs/KVRing.tla, checked over its state machine).

Writer: position p's K/V go to slot p % RING, in order; a prefill chunk of C
positions is written before any of its queries read.  Reader: for query qp with
newest written position mw, slot t holds position
    ps(t) = mw - ((mw + RING - t) % RING)
and is live iff ps <= qp and ps + W > qp (oracle.ops.ring_positions, the
attention kernels' SlotRule).

* SoundRec: ps(t) is the newest position <= mw congruent to t -- the slot's
  true content, so an overwritten position can only drop out of the window,
  never be read as stale K/V.
* Complete: every position of every query's window {qp-W+1 .. qp} is in its
  slot at read time -- holds exactly when RING >= W + C - 1.

This build prefills token by token (C = 1) into rings of window + ring_slack
(512) slots, so Complete holds with 512 slots to spare; a chunked prefill may
use chunks of up to ring_slack + 1 positions.
"""
import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from oracle import ops as O


def rec_ps(t, mw, ring):
    return mw - ((mw + ring - t) % ring)


def states(W, C, ring, nchunks, gen):
    """(mw, queries read at mw) over the spec's behaviour: chunks, then decode steps."""
    total = nchunks * C
    for base in range(0, total, C):
        yield base + C - 1, range(base, base + C)
    for mw in range(total, total + gen):
        yield mw, range(mw, mw + 1)


def sound(mw, ring):
    for t in range(min(ring, mw + 1)):
        r = rec_ps(t, mw, ring)
        if not (r % ring == t and r <= mw and r + ring > mw):
            return False
    return True


def served(qp, mw, W, ring):
    lo = max(0, qp - W + 1)
    return all(rec_ps(p % ring, mw, ring) == p for p in range(lo, qp + 1))


def served_closed(qp, mw, W, ring):
    """served() in closed form: the oldest needed position is still in its slot."""
    return mw - max(0, qp - W + 1) < ring


def complete(W, C, ring, nchunks, gen, fast=False):
    ok = served_closed if fast else served
    return all(ok(qp, mw, W, ring) for mw, qs in states(W, C, ring, nchunks, gen) for qp in qs)


def chunks_to_fill(W, C):
    """Enough chunks that some chunk starts past the first window."""
    return (W - 1) // C + 2


@pytest.mark.parametrize("W", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("C", [1, 2, 4, 7])
def test_sound_recovery_and_completeness_bound_exhaustive(W, C):
    """Every RING up to past the bound, over a behaviour long enough to wrap,
    as a model checker would; the closed form agrees with the slot-by-slot check."""
    n = chunks_to_fill(W, C)
    for ring in range(1, W + C + 4):
        for mw, _ in states(W, C, ring, n, 4):
            assert sound(mw, ring), (W, C, ring, mw)
        ok = complete(W, C, ring, n, 4)
        assert ok == complete(W, C, ring, n, 4, fast=True)
        assert ok == (ring >= W + C - 1), (W, C, ring)


@settings(max_examples=60, deadline=None)
@given(W=st.integers(1, 1100), C=st.integers(1, 600), slack=st.integers(-3, 3), gen=st.integers(0, 6))
def test_completeness_bound_at_production_sizes(W, C, slack, gen):
    ring = max(1, W + C - 1 + slack)
    assert complete(W, C, ring, chunks_to_fill(W, C), gen, fast=True) == (ring >= W + C - 1)


@pytest.mark.parametrize("cfg_name", ["e4b", "a4b", "tiny_ple", "tiny_moe"])
def test_this_builds_rings_are_complete(e4b, cfg_name):
    """Token-by-token prefill (C = 1) into window + ring_slack slots; a chunked
    prefill stays complete up to chunks of ring_slack + 1."""
    cfg = e4b.config.get(cfg_name)
    l = next(i for i in range(cfg.layers) if cfg.is_sliding(i))
    ring, W = cfg.ring(l), cfg.window
    assert ring == W + cfg.ring_slack
    for C in (1, cfg.ring_slack + 1):
        assert complete(W, C, ring, chunks_to_fill(W, C) + 2, 2 * ring, fast=True), C
    assert not complete(W, cfg.ring_slack + 2, ring, chunks_to_fill(W, cfg.ring_slack + 2), 1, fast=True)


@settings(max_examples=80, deadline=None)
@given(W=st.integers(1, 40), ring_extra=st.integers(0, 24), qp=st.integers(0, 400))
def test_oracle_ring_positions_follow_the_protocol(W, ring_extra, qp):
    """oracle.ops.ring_positions (the reader's recovery, checked by the GPU
    attention tests against the kernels) is rec_ps, and the live slots of a
    decode query are exactly its window."""
    ring = W + ring_extra
    ps = O.ring_positions(qp, ring)
    assert [int(x) for x in ps] == [rec_ps(t, qp, ring) for t in range(ring)]
    n = min(qp + 1, ring)
    live = sorted(int(p) for p in ps[:n] if p <= qp and p + W > qp)
    assert live == list(range(max(0, qp - W + 1), qp + 1))


def test_slot_rule_on_the_device_side_matches():
    """The attention kernels' SlotRule (cachemode 1), transcribed in 32-bit
    unsigned arithmetic from e4b-webgpu_b200/csrc/attn.cuh: its live slots are
    the query's window, before and long after the ring first wraps."""
    def slot_valid(qp, t, ring, window):
        u = np.uint32
        ps = u(qp) - u((u(qp) + u(ring) - u(t)) % u(ring))
        return bool(ps <= u(qp) and u(ps + u(window)) > u(qp))
    for ring, W in ((24, 16), (1024, 512), (1536, 1024)):
        for qp in (0, 1, W - 1, W, ring - 1, ring, 3 * ring + 5, 40000):
            n = min(qp + 1, ring)
            live = sorted(rec_ps(t, qp, ring) for t in range(n) if slot_valid(qp, t, ring, W))
            assert live == list(range(max(0, qp - W + 1), qp + 1)), (ring, W, qp)

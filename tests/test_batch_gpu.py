"""Batched MoE decode (BatchEngine: B sequences in lockstep, grouped experts,
tensor-core GEMMs) against the oracle run on each sequence separately."""
import numpy as np
import pytest

from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
TIE = 5e-3


@pytest.mark.parametrize("B", [1, 3, 9])
def test_batched_moe_decode_matches_oracle(e4b, models, B):
    buf = models("tiny_moe")
    cfg = e4b.config.get("tiny_moe")
    P, N = 10, 8
    prompts = np.stack([e4b.synth.prompt_ids(P, cfg.vocab, seed=100 + b) for b in range(B)])
    eng = e4b.BatchEngine(buf, B, 0)
    try:
        ids = eng.generate(prompts, N)
        h = eng.read_hidden()
        assert eng.dev.status() == 0
    finally:
        eng.close()
    for b in range(B):
        ref = OracleModel(buf)
        rids, margins, recs = ref.generate([int(t) for t in prompts[b]], N, record=True)
        got = [int(t) for t in ids[b]]
        for i, (x, y) in enumerate(zip(got, rids)):
            if x != y:
                assert margins[i] < TIE, (b, i, x, y, margins[i])
                break
        if got == rids:
            href = recs[-1]["hidden"][-1]
            assert np.linalg.norm(h[b] - href) / np.linalg.norm(href) < 1e-2


def _pack_tiles_ref(w, V, N):
    """numpy restatement of the tile-packed layout: superblock sb of row 128 t + m at
    ((t * nsb + sb) * 128 + m) * 212 (210 bytes + 2 zero bytes), zero rows past V."""
    nsb, T = N // 256, (V + 127) // 128
    blocks = np.zeros((T * 128, nsb, 212), np.uint8)
    blocks[:V, :, :210] = np.frombuffer(bytes(w), np.uint8).reshape(V, nsb, 210)
    return blocks.reshape(T, 128, nsb, 212).transpose(0, 2, 1, 3).reshape(-1)


@pytest.mark.parametrize("V,N,n", [(3000, 512, 11), (1000, 768, 64), (1000, 768, 1), (40000, 1024, 64),
                                   (40000, 512, 33), (4096, 2816, 64), (40000, 2048, 1), (3000, 256, 1)])
@pytest.mark.parametrize("tc", [2, 1])
def test_lmhead_tiles(e4b, dev, V, N, n, tc):
    """e4b_q6k_pack_tiles lays the bytes out as the numpy restatement says, and
    e4b_q6k_lmhead_tiles on the packed copy matches the oracle q6_K matvec per row.
    n = 1 runs the one-token warp-MMA GEMV (k_q6gv); n > 1 the warp-MMA kernel
    over activation slabs (tc = 2) or the tcgen05 kernel (tc = 1), which then
    also equals the row-major e4b_q6k_lmhead_rows to the last bit (the same
    per-superblock accumulation order).  V = 40000 gives the warps several units."""
    from oracle import ops as O
    w = e4b.synth.quant_q6_K(e4b.synth.normal_f32(V * N, 43 + V, "lmtiles", 0.02))
    nbytes = int(dev.L.e4b_q6k_packed_bytes(N, V))
    assert nbytes == (V + 127) // 128 * (N // 256) * 128 * 212
    bw, wt = dev.upload(w), dev.alloc(nbytes)
    dev.call("e4b_q6k_pack_tiles", bw.ptr, wt.ptr, N, V)
    dev.sync()
    assert np.array_equal(dev.read(wt, np.uint8, nbytes), _pack_tiles_ref(w, V, N))
    x = np.random.default_rng(44).standard_normal((n, N)).astype(np.float32)
    bx, y, y2, scr = dev.upload(x), dev.alloc(n * V * 4), dev.alloc(n * V * 4), dev.alloc(2 * 64 * N * 2)
    dev.call("e4b_set_option", b"lmhead_tiles_tc", tc)
    try:
        dev.call("e4b_q6k_lmhead_tiles", wt.ptr, bx.ptr, scr.ptr, y.ptr, N, V, np.float32(30.0), n)
        dev.call("e4b_q6k_lmhead_rows", bw.ptr, bx.ptr, scr.ptr, y2.ptr, N, V, np.float32(30.0), n)
        dev.sync()
    finally:
        dev.call("e4b_set_option", b"lmhead_tiles_tc", 0)
    assert dev.status() == 0
    got = dev.read(y, np.float32, n * V).reshape(n, V)
    if n > 1 and tc == 1:
        assert np.array_equal(got, dev.read(y2, np.float32, n * V).reshape(n, V))
    for r in range(n):
        ref = O.softcap(O.q6k_matvec(w, x[r], V, N), 30.0)
        assert np.max(np.abs(got[r] - ref)) / np.max(np.abs(ref)) < 2e-5


@pytest.mark.parametrize("tc", [1, 65])
@pytest.mark.parametrize("V,N,n", [(3000, 512, 11), (1000, 768, 64), (520, 256, 70), (4, 256, 1), (1000, 768, 1),
                                   (520, 256, 30), (40000, 1024, 64), (40000, 512, 33)])
def test_batched_lmhead_rows(e4b, dev, V, N, n, tc):
    """e4b_q6k_lmhead_rows against the oracle q6_K matvec per row.  With
    lmhead_tc_min = 1, n <= 64 and V % 8 == 0 take the tcgen05 kernel (weights
    split exactly into f16 hi + lo, x as f16 hi + lo); with 65 (and for n > 64)
    the mma.sync kernels: V % 8 == 0 the staged one, other V the direct one.
    V = 40000 spans more 128-row tiles than a B200 has SMs (the persistent
    grid's second round); the synthetic scales reach +-127, so ~2 % of the
    weights have a non-zero lo part."""
    from oracle import ops as O
    w = e4b.synth.quant_q6_K(e4b.synth.normal_f32(V * N, 41 + V, "lmrows", 0.02))
    x = np.random.default_rng(42).standard_normal((n, N)).astype(np.float32)
    y = dev.alloc(n * V * 4)
    scr = dev.alloc(2 * max(64, (n + 7) // 8 * 8) * N * 2)
    dev.call("e4b_set_option", b"lmhead_tc_min", tc)
    try:
        dev.call("e4b_q6k_lmhead_rows", dev.upload(w).ptr, dev.upload(x).ptr, scr.ptr, y.ptr, N, V,
                 np.float32(30.0), n)
        dev.sync()
    finally:
        dev.call("e4b_set_option", b"lmhead_tc_min", 1)
    assert dev.status() == 0
    got = dev.read(y, np.float32, n * V).reshape(n, V)
    for r in range(n):
        ref = O.softcap(O.q6k_matvec(w, x[r], V, N), 30.0)
        assert np.max(np.abs(got[r] - ref)) / np.max(np.abs(ref)) < 2e-5

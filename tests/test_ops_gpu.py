"""Per-operator parity on the GPU: each C-ABI kernel against the CPU oracle on
the same seeded inputs.  Dequantisation is compared bit for bit; f32 outputs
within 2e-5 relative (fp32 summation order); f16 outputs within one f16 ulp
of the oracle's value (the f32 value before rounding may differ in its last
bits)."""
import math

import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu
F32 = np.float32
RTOL = 2e-5


def rel_err(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def f16_close(a16, ref32):
    a = np.asarray(a16, np.float16).astype(np.float64)
    r = np.asarray(ref32, np.float64)
    ulp = np.abs(np.asarray(ref32, np.float16).astype(np.float64)) * 2.0 ** -10 + 2.0 ** -24
    return bool(np.all(np.abs(a - r) <= 1.01 * ulp + 1e-7))


def rng(seed):
    return np.random.default_rng(seed)


def up(dev, a):
    return dev.upload(np.ascontiguousarray(a))


def get(dev, buf, dtype, n):
    dev.sync()
    return dev.read(buf, dtype, n)


def q40(e4b, rows, n_in, seed):
    return e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, seed, f"w{rows}x{n_in}", 0.02))


def q6k(e4b, rows, n_in, seed):
    return e4b.synth.quant_q6_K(e4b.synth.normal_f32(rows * n_in, seed, f"w6{rows}x{n_in}", 0.02))


# ------------------------------------------------------------------ dequant
def test_dequant_bit_exact(e4b, dev):
    raw = q40(e4b, 64, 704, 1)
    out = dev.alloc(raw.size // 18 * 32 * 4)
    e4b.ops.dequant_q40(dev, up(dev, raw), out, raw.size // 18)
    assert np.array_equal(get(dev, out, F32, raw.size // 18 * 32).view(np.uint32), O.deq_q40(raw).view(np.uint32))
    raw6 = q6k(e4b, 8, 512, 2)
    out6 = dev.alloc(raw6.size // 210 * 256 * 4)
    e4b.ops.dequant_q6k(dev, up(dev, raw6), out6, raw6.size // 210)
    assert np.array_equal(get(dev, out6, F32, raw6.size // 210 * 256).view(np.uint32),
                          O.deq_q6k(raw6).view(np.uint32))


# ------------------------------------------------------------------ q4_0 GEMVs
@pytest.mark.parametrize("n_in,rows,xf16", [(256, 2048, 1), (512, 768, 0), (704, 2816, 1), (2048, 3072, 1),
                                             (2112, 2816, 1), (16384, 256, 1), (16384, 2048, 1), (2048, 8960, 0),
                                             (4096, 2816, 1), (192, 96, 1), (64, 40, 0), (32, 5, 0)])
def test_q40mv(e4b, dev, n_in, rows, xf16):
    raw = q40(e4b, rows, n_in, 3)
    x = rng(n_in).standard_normal(n_in).astype(F32)
    if xf16:
        x = O.f16r(x)
    xd = up(dev, x.astype(np.float16) if xf16 else x)
    y = dev.alloc(rows * 4)
    e4b.ops.q40mv(dev, xd, up(dev, raw), None, y, IN=n_in, OUT=rows, XF16=xf16)
    assert rel_err(get(dev, y, F32, rows), O.q40mv(raw, x, rows, n_in)) < RTOL


def test_q40mv_reference_kat(e4b, dev):
    """The reference's synthetic q40mv known-answer test (resident-a4b.html:421-456,
    "mvtest") on the CUDA GEMV: f16 x[i] = ((13 i + 5) mod 17 - 8) / 8 through the
    A4B down projection shape (2112 -> 2816); every row within f32 accumulation
    error of the exact per-block sum."""
    from test_oracle import mvtest_exact, mvtest_x
    rows, n_in = 2816, 2112
    raw = q40(e4b, rows, n_in, 41)
    x = mvtest_x(n_in)
    y = dev.alloc(rows * 4)
    e4b.ops.q40mv(dev, up(dev, x.astype(np.float16)), up(dev, raw), None, y, IN=n_in, OUT=rows, XF16=1)
    exact, mag = mvtest_exact(raw, x, rows, n_in)
    assert np.all(np.abs(get(dev, y, F32, rows) - exact) <= 1e-5 * mag)


def test_q40mv_stream_matches_simple_kernel(e4b, dev):
    """The streaming tensor-core GEMV and the one-warp-per-row kernel agree to
    fp32 summation order on a split-K shape, with the f32-input path too."""
    import ctypes
    for n_in, rows, xf16 in [(16384, 512, 1), (2048, 1024, 0)]:
        raw = up(dev, q40(e4b, rows, n_in, 33))
        x = rng(34).standard_normal(n_in).astype(F32)
        xd = up(dev, x.astype(np.float16) if xf16 else x)
        y1, y2 = dev.alloc(rows * 4), dev.alloc(rows * 4)
        e4b.ops.q40mv(dev, xd, raw, None, y1, IN=n_in, OUT=rows, XF16=xf16)
        ws = dev.L.e4b_workspace_bytes()
        wsbuf = [b for b in dev.buffers if b.name == "workspace"][0]
        dev.call("e4b_set_workspace", None, ctypes.c_size_t(0))
        try:
            e4b.ops.q40mv(dev, xd, raw, None, y2, IN=n_in, OUT=rows, XF16=xf16)
        finally:
            dev.call("e4b_set_workspace", wsbuf.ptr, ctypes.c_size_t(ws))
        a, b = get(dev, y1, F32, rows), get(dev, y2, F32, rows)
        assert rel_err(a, b) < RTOL
        # run-to-run determinism of the split-K merge
        e4b.ops.q40mv(dev, xd, raw, None, y2, IN=n_in, OUT=rows, XF16=xf16)
        assert np.array_equal(get(dev, y2, F32, rows), a)


@pytest.mark.parametrize("H,FF", [(2048, 16384), (512, 1024), (2816, 2112)])
def test_q40gu_dense_stream(e4b, dev, H, FF):
    wd = q40(e4b, 2 * FF, H, 35)
    x = O.f16r(rng(36).standard_normal(H).astype(F32))
    yh = dev.alloc(FF * 2)
    e4b.ops.q40gu(dev, None, None, None, None, up(dev, x.astype(np.float16)), up(dev, wd), yh, IN=H, FF=0, FF2=FF, K=0)
    gu = O.q40mv(wd, x, 2 * FF, H)
    assert f16_close(get(dev, yh, np.float16, FF), O.gelu_tanh(gu[:FF]) * gu[FF:])


def test_q40mv_expert_slots(e4b, dev):
    E, K, n_in, rows = 6, 3, 192, 96
    raw = q40(e4b, E * rows, n_in, 4)
    per = rows * n_in // 32 * 18
    topk = np.array([5, 0, 3], np.uint32)
    x = O.f16r(rng(5).standard_normal((K, n_in)).astype(F32))
    y = dev.alloc(K * rows * 4)
    e4b.ops.q40mv(dev, up(dev, x.astype(np.float16)), up(dev, raw), up(dev, topk), y, IN=n_in, OUT=rows, EXPERT=1,
                  XSLOT=1, XF16=1, NZ=K)
    got = get(dev, y, F32, K * rows).reshape(K, rows)
    for k, e in enumerate(topk):
        assert rel_err(got[k], O.q40mv(raw[e * per:(e + 1) * per], x[k], rows, n_in)) < RTOL


def test_q40gu_dense_and_experts(e4b, dev):
    E, K, H, FF, EF = 8, 4, 512, 384, 192
    wd = q40(e4b, 2 * FF, H, 6)
    we = q40(e4b, E * 2 * EF, H, 7)
    topk = np.array([7, 2, 2, 0], np.uint32)           # repeated expert is legal
    x = O.f16r(rng(8).standard_normal(H).astype(F32))
    x2 = O.f16r(rng(9).standard_normal(H).astype(F32))
    yh, yh2 = dev.alloc(K * EF * 2), dev.alloc(FF * 2)
    e4b.ops.q40gu(dev, up(dev, x.astype(np.float16)), up(dev, we), up(dev, topk), yh, up(dev, x2.astype(np.float16)),
                  up(dev, wd), yh2, IN=H, FF=EF, FF2=FF, K=K)
    gd = O.gelu_tanh(O.q40mv(wd, x2, 2 * FF, H)[:FF]) * O.q40mv(wd, x2, 2 * FF, H)[FF:]
    assert f16_close(get(dev, yh2, np.float16, FF), gd)
    per = 2 * EF * H // 32 * 18
    got = get(dev, yh, np.float16, K * EF).reshape(K, EF)
    for k, e in enumerate(topk):
        gu = O.q40mv(we[e * per:(e + 1) * per], x, 2 * EF, H)
        assert f16_close(got[k], O.gelu_tanh(gu[:EF]) * gu[EF:])


def test_q40moedown(e4b, dev):
    E, K, n_in, H = 8, 4, 192, 512
    w = q40(e4b, E * H, n_in, 10)
    topk = np.array([1, 6, 3, 4], np.uint32)
    tw = np.array([0.4, 0.3, 0.2, 0.1], F32)
    x = O.f16r(rng(11).standard_normal((K, n_in)).astype(F32))
    y = dev.alloc(H * 4)
    e4b.ops.q40moedown(dev, up(dev, x.astype(np.float16)), up(dev, w), up(dev, topk), up(dev, tw), y, IN=n_in,
                       OUT=H, K=K)
    assert rel_err(get(dev, y, F32, H), O.moe_down(x, w, topk, tw, n_in, H)) < RTOL


def test_plegatemv(e4b, dev):
    H, PD, L = 512, 64, 3
    w = q40(e4b, PD, H, 12)
    x = O.f16r(rng(13).standard_normal(H).astype(F32))
    ple = rng(14).standard_normal(L * PD).astype(F32)
    y = dev.alloc(PD * 2)
    e4b.ops.plegatemv(dev, up(dev, x.astype(np.float16)), up(dev, w), up(dev, ple), y, IN=H, OUT=PD, OFF=PD)
    assert f16_close(get(dev, y, np.float16, PD), O.gelu_tanh(O.q40mv(w, x, PD, H)) * ple[PD:2 * PD])


# ------------------------------------------------------------------ q6_K
def test_q6k_embed_bit_exact(e4b, dev):
    V, N = 300, 512
    w = q6k(e4b, V, N, 15)
    params = np.array([0, 1, 217, 0, 0, 1, 0, 0], np.uint32)
    y = dev.alloc(N * 4)
    mult = float(F32(math.sqrt(N)))
    e4b.ops.q6k_embed(dev, up(dev, w), up(dev, params), None, y, N=N, ROWS=V, MULT=mult)
    assert np.array_equal(get(dev, y, F32, N), O.q6k_row(w, 217, N, mult))
    # out-of-range token: zeros + device status flag, no fault
    params[2] = V + 5
    e4b.ops.q6k_embed(dev, up(dev, w), up(dev, params), None, y, N=N, ROWS=V, MULT=mult)
    assert not get(dev, y, F32, N).any()
    assert dev.status() != 0 and dev.status() == 0


@pytest.mark.parametrize("V,N,cap", [(4096, 512, 30.0), (1000, 2048, 0.0), (3, 2048, 30.0), (20011, 4096, 30.0)])
def test_q6k_lmhead(e4b, dev, V, N, cap):
    w = q6k(e4b, V, N, 16)
    x = rng(17).standard_normal(N).astype(F32)
    y = dev.alloc(V * 4)
    e4b.ops.q6k_lmhead(dev, up(dev, w), up(dev, x), y, N=N, OUT=V, SOFTCAP=cap)
    assert rel_err(get(dev, y, F32, V), O.softcap(O.q6k_matvec(w, x, V, N), cap)) < RTOL


def test_pleprep(e4b, dev):
    L, PD, V, H = 4, 64, 50, 512
    table = q6k(e4b, V, L * PD, 18)
    proj = rng(19).standard_normal(L * PD).astype(F32)
    nw = rng(20).uniform(0.5, 1.5, PD).astype(F32)
    params = np.array([0, 1, 33, 0, 0, 1, 0, 0], np.uint32)
    out = dev.alloc(L * PD * 4)
    ps, mult = float(F32(1 / math.sqrt(H))), float(F32(math.sqrt(PD)))
    e4b.ops.pleprep(dev, up(dev, table), up(dev, params), None, up(dev, proj), up(dev, nw), out, PD=PD, LAYERS=L,
                    ROWS=V, MULT=mult, PROJ_SCALE=ps)
    ident = O.q6k_row(table, 33, L * PD, mult)
    ref = np.empty(L * PD, F32)
    for l in range(L):
        b = proj[l * PD:(l + 1) * PD] * F32(ps)
        ref[l * PD:(l + 1) * PD] = (b * O.rms_inv(b, 1e-6) * nw + ident[l * PD:(l + 1) * PD]) * F32(math.sqrt(0.5))
    assert rel_err(get(dev, out, F32, L * PD), ref) < RTOL


# ------------------------------------------------------------------ norms
def test_rmsnorm_variants(e4b, dev):
    D, R = 2816, 3
    x = rng(21).standard_normal((R, D)).astype(F32) * 3
    w = rng(22).uniform(0.5, 1.5, D).astype(F32)
    y, yh, sums = dev.alloc(R * D * 4), dev.alloc(R * D * 2), dev.alloc(R * 4)
    xd, wd = up(dev, x), up(dev, w)
    e4b.ops.rmsnorm(dev, xd, wd, y, sums, None, DIM=D, ROWS=R, SUMOUT=1)
    ref = O.rmsnorm(x, w, 1e-6)
    assert rel_err(get(dev, y, F32, R * D).reshape(R, D), ref) < RTOL
    assert rel_err(get(dev, sums, F32, R), ref.sum(axis=1)) < 1e-4
    e4b.ops.rmsnorm(dev, xd, wd, None, None, yh, DIM=D, ROWS=R, F16OUT=1)
    assert f16_close(get(dev, yh, np.float16, R * D), ref.reshape(-1))


def test_rmsacc_and_rmsaccn(e4b, dev):
    D = 2048
    t = rng(23).standard_normal(D).astype(F32)
    h = rng(24).standard_normal(D).astype(F32)
    w1 = rng(25).uniform(0.5, 1.5, D).astype(F32)
    w2 = rng(26).uniform(0.5, 1.5, D).astype(F32)
    hd = up(dev, h)
    e4b.ops.rmsacc(dev, up(dev, t), up(dev, w1), hd, DIM=D, MUL=0.75)
    assert rel_err(get(dev, hd, F32, D), O.rmsacc(t, w1, h, 1e-6, 0.75)) < RTOL
    for norm2 in (1, 0):
        hd = up(dev, h)
        yh = dev.alloc(D * 2)
        e4b.ops.rmsaccn(dev, up(dev, t), up(dev, w1), hd, up(dev, w2), yh, DIM=D, MUL=1.25, NORM2=norm2)
        hr = O.rmsacc(t, w1, h, 1e-6, 1.25)
        assert rel_err(get(dev, hd, F32, D), hr) < RTOL
        assert f16_close(get(dev, yh, np.float16, D), O.rmsnorm(hr, w2, 1e-6) if norm2 else hr)


def test_rmsacc3_and_a4btail_batched(e4b, dev):
    H, B = 2816, 3
    r = rng(27)
    t, hin, m = (r.standard_normal((B, H)).astype(F32) for _ in range(3))
    ws = [r.uniform(0.5, 1.5, H).astype(F32) for _ in range(5)]
    bufs = [dev.alloc(B * H * s) for s in (2, 4, 2, 4)]
    e4b.ops.rmsacc3(dev, up(dev, t), *[up(dev, w) for w in ws[:4]], up(dev, hin), *bufs, DIM=H, BATCH=B)
    for b in range(B):
        ho, y1, y2, y3 = O.rmsacc3(t[b], ws[0], ws[1], ws[2], ws[3], hin[b], 1e-6)
        assert rel_err(get(dev, bufs[3], F32, B * H).reshape(B, H)[b], ho) < RTOL
        assert rel_err(get(dev, bufs[1], F32, B * H).reshape(B, H)[b], y2) < RTOL
        assert f16_close(get(dev, bufs[0], np.float16, B * H).reshape(B, H)[b], (ho * O.rms_inv(ho, 1e-6)) * ws[1])
    yn, ho = dev.alloc(B * H * 2), dev.alloc(B * H * 4)
    e4b.ops.a4btail(dev, up(dev, t), up(dev, ws[0]), up(dev, m), up(dev, ws[1]), up(dev, ws[2]), up(dev, hin),
                    up(dev, ws[3]), yn, ho, H=H, MUL=0.5, NEXT=1, BATCH=B)
    for b in range(B):
        hr, _ = O.a4btail(t[b], ws[0], m[b], ws[1], ws[2], hin[b], ws[3], 1e-6, 0.5)
        assert rel_err(get(dev, ho, F32, B * H).reshape(B, H)[b], hr) < RTOL
        assert f16_close(get(dev, yn, np.float16, B * H).reshape(B, H)[b], O.rmsnorm(hr, ws[3], 1e-6))


def test_geglu_elementwise(e4b, dev):
    N, K = 1000, 3
    a = rng(28).standard_normal(N).astype(F32) * 4
    b = rng(29).standard_normal(N).astype(F32)
    y = dev.alloc(N * 4)
    e4b.ops.geglumul(dev, up(dev, a), up(dev, b), y, N=N)
    assert rel_err(get(dev, y, F32, N), O.gelu_tanh(a) * b) < RTOL
    gu = rng(30).standard_normal((K, 2 * N)).astype(F32)
    out, outh = dev.alloc(K * N * 4), dev.alloc(K * N * 2)
    e4b.ops.geglusl(dev, up(dev, gu), out, FF=N, K=K)
    ref = O.gelu_tanh(gu[:, :N]) * gu[:, N:]
    assert rel_err(get(dev, out, F32, K * N).reshape(K, N), ref) < RTOL
    e4b.ops.geglub(dev, up(dev, gu), outh, N=N, ROWS=K)
    assert f16_close(get(dev, outh, np.float16, K * N), ref.reshape(-1))
    ple = rng(31).standard_normal(2 * N).astype(F32)
    e4b.ops.plemul(dev, up(dev, a), up(dev, ple), y, N=N, OFF=N)
    assert rel_err(get(dev, y, F32, N), O.gelu_tanh(a) * ple[N:]) < RTOL


# ------------------------------------------------------------------ router / argmax
@pytest.mark.parametrize("H,E,K,B", [(2816, 128, 8, 4), (2816, 128, 8, 64), (512, 16, 4, 37), (200, 40, 3, 2)])
def test_routertop_batched(e4b, dev, H, E, K, B):
    """batch > 1 with the fixture's workspace: split-K score GEMM + per-token top-K."""
    x = rng(32).standard_normal((B, H)).astype(F32) * 0.05
    wr = (rng(33).standard_normal((E, H)) * 0.02).astype(F32)
    pes = rng(34).uniform(0.5, 1.5, E).astype(F32)
    idx, w = dev.alloc(B * K * 4), dev.alloc(B * K * 4)
    e4b.ops.routertop(dev, up(dev, x), up(dev, wr), up(dev, pes), idx, w, H=H, E=E, K=K, BATCH=B)
    gi = get(dev, idx, np.uint32, B * K).reshape(B, K)
    gw = get(dev, w, F32, B * K).reshape(B, K)
    for b in range(B):
        ri, rw = O.router_topk(x[b], wr, pes, K)
        assert list(gi[b]) == list(ri)
        assert rel_err(gw[b], rw) < 1e-5


def test_top8_ties(e4b, dev):
    s = np.zeros(128, F32)
    s[[3, 9, 40]] = 2.0
    idx, w = dev.alloc(32), dev.alloc(32)
    e4b.ops.top8(dev, up(dev, s), up(dev, np.ones(128, F32)), idx, w, E=128, K=8)
    gi = get(dev, idx, np.uint32, 8)
    ri, rw = O.router_topk(np.ones(1, F32), s.reshape(128, 1), np.ones(128, F32), 8)
    assert list(gi) == list(ri) == [3, 9, 40, 0, 1, 2, 4, 5]
    assert rel_err(get(dev, w, F32, 8), rw) < 1e-6


@pytest.mark.parametrize("N", [262144, 4096, 1000, 7])
def test_argmax_ties_lowest(e4b, dev, N):
    x = rng(N).standard_normal(N).astype(F32)
    x[N // 2] = 50.0
    x[N - 1] = 50.0
    part, out = dev.alloc(256 * 8), dev.alloc(8)
    e4b.ops.argmax(dev, up(dev, x), part, out, N=N, PARTS=256)
    o = get(dev, out, np.uint32, 2)
    assert int(o[0]) == (N // 2 if N > 1 else 0) and o[1].view(F32) == 50.0


def test_feedtok_advances_params(e4b, dev):
    amax = up(dev, np.array([1234, 0], np.uint32))
    params = up(dev, np.array([9, 10, 0, 0, 9, 10, 3, 0], np.uint32))
    ring = dev.alloc(16 * 4)
    e4b.ops.feedtok(dev, amax, params, ring, RING_CAP=16)
    assert list(get(dev, params, np.uint32, 8)) == [10, 11, 1234, 0, 10, 11, 4, 0]
    assert get(dev, ring, np.uint32, 16)[3] == 1234


# ------------------------------------------------------------------ attention
def _cache(r, slots, kvh, hd):
    return O.f16r(r.standard_normal((slots, kvh, hd)).astype(F32)).astype(np.float16)


@pytest.mark.parametrize("cm,qp,window,ring,slots", [(2, 0, 0, 1, 64), (2, 700, 0, 1, 1024), (1, 5, 16, 24, 24),
                                                      (1, 100, 16, 24, 24), (1, 1500, 512, 1024, 1024),
                                                      (0, 300, 128, 1, 512)])
def test_attention_split_vs_dense(e4b, dev, cm, qp, window, ring, slots):
    QH, KVH, HD, CS = 8, 2, 256, 64
    r = rng(qp + 7 * cm)
    kc, vc = _cache(r, slots, KVH, HD), _cache(r, slots, KVH, HD)
    q = r.standard_normal((QH, HD)).astype(F32) * 0.1
    if cm == 1:
        plant = qp % ring
    else:
        plant = min(qp, slots - 1) // 2
    kc[plant, 0] = (8 * q[0] / np.linalg.norm(q[0]) * np.linalg.norm(q[0])).astype(np.float16)
    length = qp + 1
    params = np.array([qp, length, 0, 0, qp, length, 0, 0], np.uint32)
    chunks = (slots + CS - 1) // CS
    po, pml = dev.alloc(QH * chunks * HD * 4), dev.alloc(QH * chunks * 8)
    oh, of, lse = dev.alloc(QH * HD * 2), dev.alloc(QH * HD * 4), dev.alloc(QH * 4)
    e4b.ops.attsplit(dev, up(dev, q), up(dev, kc), up(dev, vc), up(dev, params), po, pml, Q_HEADS=QH, KV_HEADS=KVH,
                     HEAD_DIM=HD, WINDOW=window, CACHEMODE=cm, RING=ring, CS=CS, CHUNKS=chunks)
    e4b.ops.attcomb(dev, po, pml, oh, of, lse, Q_HEADS=QH, HEAD_DIM=HD, CHUNKS=chunks)
    got = get(dev, of, F32, QH * HD).reshape(QH, HD)
    glse = get(dev, lse, F32, QH)
    if cm == 1:
        n = min(qp + 1, ring)
        ps = O.ring_positions(qp, ring)[:n]
        valid = np.nonzero((ps <= qp) & (ps + window > qp))[0]
    elif cm == 2:
        valid = np.arange(length)
    else:
        valid = np.arange(max(0, length - window), length)
    for h in range(QH):
        o, l_ = O.attend(q[h], kc[:, h // (QH // KVH)], vc[:, h // (QH // KVH)], valid)
        assert rel_err(got[h], o) < 1e-4
        assert abs(float(glse[h]) - float(l_)) < 1e-4 * max(1.0, abs(float(l_)))
    assert f16_close(get(dev, oh, np.float16, QH * HD), got.reshape(-1))


def test_headprep_all_roles(e4b, dev):
    QH, KVH, HD, ring = 4, 2, 128, 24
    for keqv, cm, angles, theta in [(0, 1, 64, 10000.0), (1, 2, 16, 1e6)]:
        r = rng(40 + keqv)
        rows = QH * HD + KVH * HD * (1 if keqv else 2)
        qkv = r.standard_normal(rows).astype(F32)
        qw = r.uniform(0.5, 1.5, HD).astype(F32)
        kw = r.uniform(0.5, 1.5, HD).astype(F32)
        pos = 37
        params = np.array([pos, pos + 1, 0, 0, 11, 12, 0, 0], np.uint32)
        kc, vc, qo = dev.alloc(ring * KVH * HD * 2), dev.alloc(ring * KVH * HD * 2), dev.alloc(QH * HD * 4)
        e4b.ops.headprep(dev, up(dev, qkv), up(dev, qw), up(dev, kw), up(dev, params), kc, vc, qo, QH=QH, KVH=KVH,
                         HEAD_DIM=HD, ROPE_ANGLES=angles, THETA=theta, KEQV=keqv, CACHEMODE=cm, RING=ring, SLOTS=ring)
        q, k, v = O.headprep(qkv, qw, kw, pos, QH, KVH, HD, angles, theta, 1e-6, keqv)
        slot = pos % ring if cm == 1 else 11
        assert rel_err(get(dev, qo, F32, QH * HD).reshape(QH, HD), q) < 1e-4
        gk = get(dev, kc, np.float16, ring * KVH * HD).reshape(ring, KVH, HD)[slot]
        gv = get(dev, vc, np.float16, ring * KVH * HD).reshape(ring, KVH, HD)[slot]
        assert np.max(np.abs(gk.astype(F32) - k)) <= 2e-3 * np.max(np.abs(k))
        assert np.max(np.abs(gv.astype(F32) - v)) <= 2e-3 * np.max(np.abs(v))

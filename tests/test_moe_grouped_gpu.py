"""Grouped MoE for batched decode (expgroup -> q40gugrp -> q40downgrp -> wacc)
against the per-token oracle: y_t = sum_k w_tk * W_down[e_tk] f16(gelu(gate) * up)
with [gate | up] = W_gu[e_tk] x_t (kernels/q40gugrp.wgsl, q40downgrp.wgsl,
wacc.wgsl semantics; src/engine-a4b.js:437-462 per token), plus the dense
multi-token GEMMs (q40mm / q40gumm) and the fragment-order activation layout
their producers write."""
import numpy as np
import pytest

from oracle import ops as O
from pack_layout import pack_q40

pytestmark = pytest.mark.gpu
F32 = np.float32


def q40(e4b, rows, n_in, seed):
    return e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, seed, f"g{rows}x{n_in}", 0.02))


def _topk(rng, n, K, E, hot):
    """Distinct experts per token; `hot` tokens all route expert 3 first (a >64-token group)."""
    idx = np.empty((n, K), np.uint32)
    for t in range(n):
        sel = rng.choice(E, K, replace=False)
        if t < hot and 3 not in sel:
            sel[0] = 3
        idx[t] = sel
    w = rng.uniform(0.05, 0.4, (n, K)).astype(F32)
    return idx, w


@pytest.mark.parametrize("n,hot", [(1, 0), (13, 0), (64, 0), (80, 75)])
def test_grouped_moe_matches_per_token_oracle(e4b, dev, n, hot):
    E, K, H, EF = 16, 4, 512, 192
    rng = np.random.default_rng(n)
    wgu = q40(e4b, E * 2 * EF, H, 31)
    wdn = q40(e4b, E * H, EF, 32)
    x = O.f16r(rng.standard_normal((n, H)).astype(F32))
    idx, w = _topk(rng, n, K, E, hot)
    # device
    d = dev
    xfo = e4b.batch.to_xfo
    bx, bgu, bdn = d.upload(xfo(x.astype(np.float16))), d.upload(wgu), d.upload(wdn)
    bidx, bw = d.upload(idx), d.upload(w)
    off, ent, inv = d.alloc((E + 1) * 4), d.alloc(n * K * 4), d.alloc(n * K * 4)
    g = d.alloc(n * K * EF * 2)
    yo = d.alloc(n * K * H * 4)
    out = d.alloc(n * H * 4)
    d.call("e4b_expgroup", bidx.ptr, n, K, E, off.ptr, ent.ptr, inv.ptr)
    d.call("e4b_q40gugrp", bx.ptr, bgu.ptr, off.ptr, ent.ptr, g.ptr, H, EF, E, K)
    d.call("e4b_q40downgrp", g.ptr, bdn.ptr, off.ptr, ent.ptr, yo.ptr, EF, H, E)
    d.call("e4b_wacc", yo.ptr, inv.ptr, bw.ptr, out.ptr, n, K, H)
    d.sync()
    offsets = d.read(off, np.uint32, E + 1)
    entries = d.read(ent, np.uint32, n * K)
    got = d.read(out, F32, n * H).reshape(n, H)
    assert d.status() == 0
    # the sort: stable by expert
    flat = idx.reshape(-1)
    want = np.argsort(flat, kind="stable")
    assert np.array_equal(entries, want.astype(np.uint32))
    assert np.array_equal(offsets, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]).astype(np.uint32))
    # per-token oracle
    per_gu = 2 * EF * H // 32 * 18
    worst = 0.0
    for t in range(n):
        slots = np.stack([O.geglu_rows(O.q40mv(wgu[int(e) * per_gu:(int(e) + 1) * per_gu], x[t], 2 * EF, H), EF)
                          for e in idx[t]])
        ref = O.moe_down(slots, wdn, idx[t], w[t], EF, H)
        worst = max(worst, float(np.max(np.abs(got[t] - ref)) / np.max(np.abs(ref))))
    assert worst < 2e-3, worst     # f16 GeGLU intermediates may round one ulp apart


@pytest.mark.parametrize("H,n,hot", [(512, 13, 0), (512, 80, 75), (256, 64, 0)])
def test_q40gugrp_tiles_bit_identical(e4b, dev, H, n, hot):
    """The tile-packed copy matches its numpy restatement byte for byte, and the
    grouped gate|up on it equals e4b_q40gugrp bit for bit (ragged groups and a
    >64-token expert)."""
    E, K, EF = 16, 4, 192
    rng = np.random.default_rng(100 + n)
    wgu = q40(e4b, E * 2 * EF, H, 41)
    x = O.f16r(rng.standard_normal((n, H)).astype(F32))
    idx, _ = _topk(rng, n, K, E, hot)
    d = dev
    bx, bgu, bidx = d.upload(e4b.batch.to_xfo(x.astype(np.float16))), d.upload(wgu), d.upload(idx)
    bt = d.alloc(wgu.nbytes)
    off, ent, inv = d.alloc((E + 1) * 4), d.alloc(n * K * 4), d.alloc(n * K * 4)
    g0, g1 = d.alloc(n * K * EF * 2), d.alloc(n * K * EF * 2)
    d.call("e4b_q40_pack_tiles", bgu.ptr, bt.ptr, E * 2 * EF, H)
    d.call("e4b_expgroup", bidx.ptr, n, K, E, off.ptr, ent.ptr, inv.ptr)
    d.call("e4b_q40gugrp", bx.ptr, bgu.ptr, off.ptr, ent.ptr, g0.ptr, H, EF, E, K)
    d.call("e4b_q40gugrp_tiles", bx.ptr, bt.ptr, off.ptr, ent.ptr, g1.ptr, H, EF, E, K)
    d.sync()
    assert d.status() == 0
    packed = d.read(bt, np.uint8, wgu.nbytes)
    assert np.array_equal(packed, pack_q40(wgu.view(np.uint8), E * 2 * EF, H))
    a, b = d.read(g0, np.uint16, n * K * EF), d.read(g1, np.uint16, n * K * EF)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("IN,OUT", [(512, 96), (256, 40), (192, 64), (704, 48)])
@pytest.mark.parametrize("n", [1, 7, 16, 37, 64])
def test_dense_q40mm(e4b, dev, IN, OUT, n):
    """y[t] = W x[t] per token (kernels/q40mv.wgsl per row); IN % 256 == 0 takes the
    TMA-box weight stream, other IN the whole-row bulk stream."""
    rng = np.random.default_rng(IN + n)
    w = q40(e4b, OUT, IN, 7 + IN)
    x = O.f16r(rng.standard_normal((n, IN)).astype(F32))
    y = dev.alloc(n * OUT * 4)
    dev.call("e4b_q40mm", dev.upload(e4b.batch.to_xfo(x.astype(np.float16))).ptr, dev.upload(w).ptr, y.ptr, IN,
             OUT, n)
    dev.sync()
    got = dev.read(y, F32, n * OUT).reshape(n, OUT)
    assert dev.status() == 0
    for t in range(n):
        ref = O.q40mv(w, x[t], OUT, IN)
        assert np.max(np.abs(got[t] - ref)) <= 1e-5 * np.max(np.abs(ref)), t


@pytest.mark.parametrize("n", [1, 9, 64])
def test_dense_q40gumm(e4b, dev, n):
    IN, FF = 512, 96
    rng = np.random.default_rng(n)
    w = q40(e4b, 2 * FF, IN, 11)
    x = O.f16r(rng.standard_normal((n, IN)).astype(F32))
    yh = dev.alloc(n * FF * 2)
    dev.call("e4b_q40gumm", dev.upload(e4b.batch.to_xfo(x.astype(np.float16))).ptr, dev.upload(w).ptr, yh.ptr, IN,
             FF, n)
    dev.sync()
    got = e4b.batch.from_xfo(dev.read(yh, np.float16, n * FF).reshape(n, FF)).astype(F32)
    for t in range(n):
        ref = O.geglu_rows(O.q40mv(w, x[t], 2 * FF, IN), FF)
        assert np.allclose(got[t], ref, rtol=2e-3, atol=1e-4), t


def test_fragment_order_producers(e4b, dev):
    """rmsnorm f16out=2 and rmsacc3 / a4btail / attcomb_seq with xfo=1 write the
    same f16 values as the plain layout, permuted by xfo_perm."""
    H, B = 256, 3
    rng = np.random.default_rng(5)
    x = rng.standard_normal((B, H)).astype(F32)
    w = rng.uniform(0.5, 1.5, H).astype(F32)
    bx, bw = dev.upload(x), dev.upload(w)
    plain, perm = dev.alloc(B * H * 2), dev.alloc(B * H * 2)
    for f16out, buf in ((1, plain), (2, perm)):
        dev.call("e4b_rmsnorm", bx.ptr, bw.ptr, None, None, buf.ptr, H, B, np.float32(1e-6), 1, 0, f16out)
    dev.sync()
    a = dev.read(plain, np.uint16, B * H).reshape(B, H)
    b = dev.read(perm, np.uint16, B * H).reshape(B, H)
    assert np.array_equal(e4b.batch.to_xfo(a), b)
    # rmsacc3: y1, y3 permuted, y2 / h_out untouched
    t = rng.standard_normal((B, H)).astype(F32)
    ws = [dev.upload(rng.uniform(0.5, 1.5, H).astype(F32)) for _ in range(4)]
    outs = {}
    for xfo in (0, 1):
        bufs = [dev.alloc(B * H * 2), dev.alloc(B * H * 4), dev.alloc(B * H * 2), dev.alloc(B * H * 4)]
        dev.call("e4b_rmsacc3", dev.upload(t).ptr, *[q.ptr for q in ws], bx.ptr, *[q.ptr for q in bufs], H,
                 np.float32(1e-6), B, xfo, 1)
        dev.sync()
        outs[xfo] = [dev.read(bufs[0], np.uint16, B * H).reshape(B, H), dev.read(bufs[1], F32, B * H),
                     dev.read(bufs[2], np.uint16, B * H).reshape(B, H), dev.read(bufs[3], F32, B * H)]
    assert np.array_equal(e4b.batch.to_xfo(outs[0][0]), outs[1][0])
    assert np.array_equal(e4b.batch.to_xfo(outs[0][2]), outs[1][2])
    assert np.array_equal(outs[0][1], outs[1][1]) and np.array_equal(outs[0][3], outs[1][3])
    # a4btail
    m = rng.standard_normal((B, H)).astype(F32)
    tails = {}
    for xfo in (0, 1):
        yn, ho = dev.alloc(B * H * 2), dev.alloc(B * H * 4)
        dev.call("e4b_a4btail", dev.upload(t).ptr, ws[0].ptr, dev.upload(m).ptr, ws[1].ptr, ws[2].ptr, bx.ptr,
                 ws[3].ptr, yn.ptr, ho.ptr, H, np.float32(1e-6), np.float32(0.5), 1, B, xfo)
        dev.sync()
        tails[xfo] = dev.read(yn, np.uint16, B * H).reshape(B, H)
    assert np.array_equal(e4b.batch.to_xfo(tails[0]), tails[1])
    # attcomb_seq: QH heads x HD per sequence row
    QH, HD, MC = 2, 128, 3
    po = rng.standard_normal((B, QH, MC, HD)).astype(F32)
    ml = np.stack([rng.standard_normal((B, QH, MC)), rng.uniform(0.5, 2.0, (B, QH, MC))], -1).astype(F32)
    combs = {}
    for xfo in (0, 1):
        oh = dev.alloc(B * QH * HD * 2)
        dev.call("e4b_attcomb_seq", dev.upload(po).ptr, dev.upload(ml).ptr, oh.ptr, None, None, QH, HD, MC, B, xfo)
        dev.sync()
        combs[xfo] = dev.read(oh, np.uint16, B * QH * HD).reshape(B, QH * HD)
    assert np.array_equal(e4b.batch.to_xfo(combs[0]), combs[1])


@pytest.mark.parametrize("n,K,E", [(64, 8, 128), (1, 8, 128), (700, 2, 16), (37, 4, 300), (2000, 3, 256)])
def test_expgroup_stable_sort(e4b, dev, n, K, E):
    """Entries sorted by expert, stable in the entry index (both sort kernels)."""
    rng = np.random.default_rng(n + E)
    idx = np.stack([rng.choice(E, K, replace=False) for _ in range(n)]).astype(np.uint32)
    off, ent, inv = dev.alloc((E + 1) * 4), dev.alloc(n * K * 4), dev.alloc(n * K * 4)
    dev.call("e4b_expgroup", dev.upload(idx).ptr, n, K, E, off.ptr, ent.ptr, inv.ptr)
    dev.sync()
    flat = idx.reshape(-1)
    want = np.argsort(flat, kind="stable").astype(np.uint32)
    entries = dev.read(ent, np.uint32, n * K)
    assert np.array_equal(entries, want)
    assert np.array_equal(dev.read(inv, np.uint32, n * K)[want], np.arange(n * K, dtype=np.uint32))
    assert np.array_equal(dev.read(off, np.uint32, E + 1),
                          np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]).astype(np.uint32))
    assert dev.status() == 0


def test_a4btail_wacc_equals_wacc_then_a4btail(e4b, dev):
    """The fused expert combine + tail is bit-identical to e4b_wacc followed by e4b_a4btail."""
    H, B, K = 512, 5, 4
    rng = np.random.default_rng(9)
    y = rng.standard_normal((B * K, H)).astype(F32)
    inv = rng.permutation(B * K).astype(np.uint32)
    tw = rng.uniform(0.1, 0.5, (B, K)).astype(F32)
    t1 = rng.standard_normal((B, H)).astype(F32)
    hin = rng.standard_normal((B, H)).astype(F32)
    ws = [dev.upload(rng.uniform(0.5, 1.5, H).astype(F32)) for _ in range(4)]
    by, binv, btw, bt, bh = (dev.upload(a) for a in (y, inv, tw, t1, hin))
    m = dev.alloc(B * H * 4)
    outs = []
    for fused in (0, 1):
        yn, ho = dev.alloc(B * H * 2), dev.alloc(B * H * 4)
        if fused:
            dev.call("e4b_a4btail_wacc", bt.ptr, ws[0].ptr, by.ptr, binv.ptr, btw.ptr, K, ws[1].ptr, ws[2].ptr, bh.ptr,
                     ws[3].ptr, yn.ptr, ho.ptr, H, np.float32(1e-6), np.float32(0.7), 1, B, 1)
        else:
            dev.call("e4b_wacc", by.ptr, binv.ptr, btw.ptr, m.ptr, B, K, H)
            dev.call("e4b_a4btail", bt.ptr, ws[0].ptr, m.ptr, ws[1].ptr, ws[2].ptr, bh.ptr, ws[3].ptr, yn.ptr, ho.ptr,
                     H, np.float32(1e-6), np.float32(0.7), 1, B, 1)
        dev.sync()
        outs.append((dev.read(yn, np.uint16, B * H), dev.read(ho, F32, B * H)))
    assert np.array_equal(outs[0][0], outs[1][0]) and np.array_equal(outs[0][1], outs[1][1])


@pytest.mark.parametrize("IN,OUT,n,kparts", [(2816, 6144, 64, 8), (4096, 2816, 64, 16), (512, 96, 37, 2),
                                             (256, 40, 5, 1), (768, 200, 64, 3)])
def test_q40mm_kparts(e4b, dev, IN, OUT, n, kparts):
    """K split over CTA groups, all tokens per weight decode: the parts sum (in
    order) to W x per token, within the oracle's f32 tolerance."""
    rng = np.random.default_rng(IN + OUT)
    w = q40(e4b, OUT, IN, 3 + IN)
    x = O.f16r(rng.standard_normal((n, IN)).astype(F32))
    y = dev.alloc(kparts * n * OUT * 4)
    dev.call("e4b_q40mm_kparts", dev.upload(e4b.batch.to_xfo(x.astype(np.float16))).ptr, dev.upload(w).ptr, y.ptr,
             IN, OUT, n, kparts)
    dev.sync()
    assert dev.status() == 0
    parts = dev.read(y, F32, kparts * n * OUT).reshape(kparts, n, OUT)
    got = parts[0].copy()
    for k in range(1, kparts):
        got += parts[k]
    for t in range(0, n, 7):
        ref = O.q40mv(w, x[t], OUT, IN)
        assert np.max(np.abs(got[t] - ref)) <= 1e-5 * np.max(np.abs(ref)), t


def test_kpart_consumers(e4b, dev):
    """headprep_seq and rmsacc3 with nparts > 1 equal the single-part call on
    the summed input (sums in part order)."""
    rng = np.random.default_rng(8)
    H, B, P = 256, 3, 4
    parts = rng.standard_normal((P, B, H)).astype(F32)
    total = parts[0].copy()
    for k in range(1, P):
        total += parts[k]
    ws = [dev.upload(rng.uniform(0.5, 1.5, H).astype(F32)) for _ in range(4)]
    hin = dev.upload(rng.standard_normal((B, H)).astype(F32))
    res = []
    for src, npart in ((parts, P), (total, 1)):
        bufs = [dev.alloc(B * H * 2), dev.alloc(B * H * 4), dev.alloc(B * H * 2), dev.alloc(B * H * 4)]
        dev.call("e4b_rmsacc3", dev.upload(src).ptr, *[q.ptr for q in ws], hin.ptr, *[q.ptr for q in bufs], H,
                 np.float32(1e-6), B, 1, npart)
        dev.sync()
        res.append([dev.read(bufs[i], np.uint8, B * H * (2 if i % 2 == 0 else 4)) for i in range(4)])
    for a, b in zip(*res):
        assert np.array_equal(a, b)

"""Operator-level host API: one function per reference WGSL operator.

Mirrors the reference's `Kernels.pipeline(file, params)` + `run(kern, buffers,
grid)` pair (src/gpu.js:67-84, src/engine-a4b.js:417-420): each function takes
the device, the buffers in the reference's binding order and the former ${}
parameters as keyword arguments with the reference's names, and enqueues the
CUDA kernel on the device's stream.  Missing required buffers raise, like the
reference's "missing param" error (src/gpu.js:72).
"""
from __future__ import annotations

import math

from .device import Device


def _p(x):
    return None if x is None else int(x)


def q40mv(dev: Device, x, w, topk, y, *, IN, OUT, EXPERT=0, XSLOT=0, XF16=0, NZ=1, BATCH=1):
    """kernels/q40mv.wgsl"""
    dev.call("e4b_q40mv", _p(x), _p(w), _p(topk), _p(y), IN, OUT, EXPERT, XSLOT, XF16, NZ, BATCH)


def q40gu(dev: Device, x, w, topk, yh, x2, w2, yh2, *, IN, FF, FF2, K, BATCH=1):
    """kernels/q40gu.wgsl (EXPERT=2 merged: dense on x2/w2 -> yh2, K expert slots on x/w -> yh)."""
    dev.call("e4b_q40gu", _p(x), _p(w), _p(topk), _p(yh), _p(x2), _p(w2), _p(yh2), IN, FF, FF2, K, BATCH)


def q40moedown(dev: Device, x, w, topk, tkw, y, *, IN, OUT, K, BATCH=1):
    """kernels/q40moedown.wgsl"""
    dev.call("e4b_q40moedown", _p(x), _p(w), _p(topk), _p(tkw), _p(y), IN, OUT, K, BATCH)


def moecomb(dev: Device, slots, topk_w, y, *, H, K):
    """kernels/moecomb.wgsl"""
    dev.call("e4b_moecomb", _p(slots), _p(topk_w), _p(y), H, K)


def q6k_embed(dev: Device, w, params, tok, y, *, N, ROWS, MULT=None, TOKSRC=0, BATCH=0):
    """kernels/q6k.wgsl MODE 0"""
    mult = math.sqrt(N) if MULT is None else MULT
    dev.call("e4b_q6k_embed", _p(w), _p(params), _p(tok), _p(y), N, ROWS, float(mult), TOKSRC, BATCH)


def q6k_lmhead(dev: Device, w, x, y, *, N, OUT, SOFTCAP=0.0, BATCH=1):
    """kernels/q6k.wgsl MODE 1"""
    dev.call("e4b_q6k_lmhead", _p(w), _p(x), _p(y), N, OUT, float(SOFTCAP), BATCH)


def rmsnorm(dev: Device, x, w, y, sums, yh, *, DIM, ROWS=1, EPS=1e-6, WITH_SCALE=1, SUMOUT=0, F16OUT=0):
    """kernels/rmsnorm.wgsl"""
    dev.call("e4b_rmsnorm", _p(x), _p(w), _p(y), _p(sums), _p(yh), DIM, ROWS, float(EPS), WITH_SCALE, SUMOUT, F16OUT)


def rmsacc(dev: Device, x, w, hidden, *, DIM, EPS=1e-6, MUL=1.0):
    """kernels/rmsacc.wgsl"""
    dev.call("e4b_rmsacc", _p(x), _p(w), _p(hidden), DIM, float(EPS), float(MUL))


def rmsaccn(dev: Device, t, w1, hidden, w2, yh, *, DIM, EPS=1e-6, MUL=1.0, NORM2=1):
    """kernels/rmsaccsrq.wgsl without the int8 activation quantisation (f16 output)."""
    dev.call("e4b_rmsaccn", _p(t), _p(w1), _p(hidden), _p(w2), _p(yh), DIM, float(EPS), float(MUL), NORM2)


def rmsacc3(dev: Device, t, w_acc, w1, w2, w3, h_in, y1, y2, y3, h_out, *, DIM, EPS=1e-6, BATCH=1, XFO=0, NPARTS=1):
    """kernels/rmsacc3.wgsl"""
    dev.call("e4b_rmsacc3", _p(t), _p(w_acc), _p(w1), _p(w2), _p(w3), _p(h_in), _p(y1), _p(y2), _p(y3), _p(h_out),
             DIM, float(EPS), BATCH, XFO, NPARTS)


def a4btail(dev: Device, t1, w1, m, w2, wp, h_in, w_next, y_next, h_out, *, H, EPS=1e-6, MUL=1.0, NEXT=1, BATCH=1,
            XFO=0):
    """kernels/a4btail.wgsl"""
    dev.call("e4b_a4btail", _p(t1), _p(w1), _p(m), _p(w2), _p(wp), _p(h_in), _p(w_next), _p(y_next), _p(h_out), H,
             float(EPS), float(MUL), NEXT, BATCH, XFO)


def routertop(dev: Device, x, wr, pes, topk_idx, topk_w, *, H, E, K, BATCH=1):
    """kernels/routertop.wgsl"""
    dev.call("e4b_routertop", _p(x), _p(wr), _p(pes), _p(topk_idx), _p(topk_w), H, E, K, BATCH)


def router(dev: Device, h, scale, wr, pes, topk_idx, topk_w, *, H, E, K, EPS=1e-6):
    """kernels/router.wgsl"""
    dev.call("e4b_router", _p(h), _p(scale), _p(wr), _p(pes), _p(topk_idx), _p(topk_w), H, E, K, float(EPS))


def top8(dev: Device, scores, pes, topk_idx, topk_w, *, E, K):
    """kernels/top8.wgsl"""
    dev.call("e4b_top8", _p(scores), _p(pes), _p(topk_idx), _p(topk_w), E, K)


def headprep(dev: Device, qkv, qw, kw, params, kcache, vcache, q_out, *, QH, KVH, HEAD_DIM, ROPE_ANGLES, THETA,
             EPS=1e-6, KEQV=0, CACHEMODE=1, RING=1, SLOTS, BATCH=1):
    """kernels/headprep.wgsl"""
    dev.call("e4b_headprep", _p(qkv), _p(qw), _p(kw), _p(params), _p(kcache), _p(vcache), _p(q_out), QH, KVH,
             HEAD_DIM, ROPE_ANGLES, float(THETA), float(EPS), KEQV, CACHEMODE, RING, SLOTS, BATCH)


def rope(dev: Device, x, params, *, HEADS, HEAD_DIM, ROPE_ANGLES, THETA):
    """kernels/rope.wgsl"""
    dev.call("e4b_rope", _p(x), _p(params), HEADS, HEAD_DIM, ROPE_ANGLES, float(THETA))


def kvwrite(dev: Device, src, params, dst, *, N):
    """kernels/kvwrite.wgsl"""
    dev.call("e4b_kvwrite", _p(src), _p(params), _p(dst), N)


def attsplit(dev: Device, q, kcache, vcache, params, part_o, part_ml, *, Q_HEADS, KV_HEADS, HEAD_DIM, WINDOW=0,
             CACHEMODE=0, RING=1, CS=64, CHUNKS, SCALE=1.0):
    """kernels/attsplit.wgsl"""
    dev.call("e4b_attsplit", _p(q), _p(kcache), _p(vcache), _p(params), _p(part_o), _p(part_ml), Q_HEADS, KV_HEADS,
             HEAD_DIM, WINDOW, CACHEMODE, RING, CS, CHUNKS, float(SCALE))


def attcomb(dev: Device, part_o, part_ml, out_h, out_f, lse, *, Q_HEADS, HEAD_DIM, CHUNKS):
    """kernels/attcomb.wgsl"""
    dev.call("e4b_attcomb", _p(part_o), _p(part_ml), _p(out_h), _p(out_f), _p(lse), Q_HEADS, HEAD_DIM, CHUNKS)


def geglumul(dev: Device, a, b, y, *, N):
    dev.call("e4b_geglumul", _p(a), _p(b), _p(y), N)


def geglusl(dev: Device, gu, out, *, FF, K):
    dev.call("e4b_geglusl", _p(gu), _p(out), FF, K)


def geglub(dev: Device, gu, yh, *, N, ROWS):
    dev.call("e4b_geglub", _p(gu), _p(yh), N, ROWS)


def pleprep(dev: Device, table, params, tok, proj, norm_w, ple_in, *, PD, LAYERS, ROWS, MULT=None, PROJ_SCALE=1.0,
            EPS=1e-6, TOKSRC=0):
    """kernels/pleprep.wgsl (q6_K table)"""
    mult = math.sqrt(PD) if MULT is None else MULT
    dev.call("e4b_pleprep", _p(table), _p(params), _p(tok), _p(proj), _p(norm_w), _p(ple_in), PD, LAYERS, ROWS,
             float(mult), float(PROJ_SCALE), float(EPS), TOKSRC)


def plegatemv(dev: Device, x, w, ple, y, *, IN, OUT, OFF):
    """kernels/plegatemv.wgsl (q4_0 weights, f16 activations)"""
    dev.call("e4b_plegatemv", _p(x), _p(w), _p(ple), _p(y), IN, OUT, OFF)


def plemul(dev: Device, a, ple, y, *, N, OFF):
    dev.call("e4b_plemul", _p(a), _p(ple), _p(y), N, OFF)


def argmax(dev: Device, x, part, out, *, N, PARTS=256):
    """kernels/argmax2.wgsl (stage 0 and stage 1)"""
    dev.call("e4b_argmax", _p(x), _p(part), _p(out), N, PARTS)


def feedtok(dev: Device, amax, params, ring=None, *, RING_CAP=1024):
    """kernels/feedtok.wgsl + token-ring copy + parameter advance"""
    dev.call("e4b_feedtok", _p(amax), _p(params), _p(ring), RING_CAP)


def dequant_q40(dev: Device, w, out, nblocks: int):
    dev.call("e4b_dequant_q40", _p(w), _p(out), nblocks)


def dequant_q6k(dev: Device, w, out, nblocks: int):
    dev.call("e4b_dequant_q6k", _p(w), _p(out), nblocks)

"""CPU ORACLE -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of each operator on the reference's per-token decode path.
Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg use it,
and only as the checker / the timed CPU baseline; the product path never does.

Parity status: the reference's own golden vectors (goldens/*.json) were made on
real checkpoints that are not in the reference tree, so they cannot pin these
synthetic-weight computations: parity is anchored here on (a) the python `gguf`
package's independent Q4_0 / Q6_K decoders and Q4_0 encoder (bit-exact checks in
tests/test_oracle.py) and (b) this restatement of the reference kernels, each
function below citing the WGSL it follows.  Arithmetic is f32, with values
rounded to f16 exactly where the reference stores f16.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

F32 = np.float32


def qlib():
    """The oracle's C helper (oracle/qdot.c), built by oracle/build.py."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle_q.so")
        if not os.path.exists(path):
            from . import build as _b
            _b.build()
        lib = ctypes.CDLL(path)
        u8p, f32p, i64 = ctypes.POINTER(ctypes.c_uint8), ctypes.POINTER(ctypes.c_float), ctypes.c_int64
        lib.oracle_q40_matvec.argtypes = [u8p, f32p, f32p, i64, i64]
        lib.oracle_q6k_matvec.argtypes = [u8p, f32p, f32p, i64, i64]
        lib.oracle_q6k_rows.argtypes = [u8p, f32p, i64, i64, i64, ctypes.c_float]
        lib.oracle_threads.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def _u8(a):
    a = np.ascontiguousarray(a, dtype=np.uint8)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


# Where the reference stores an f16 buffer (activations feeding a GEMV, the
# KV caches) the oracle rounds to f16.  STORE_F16 = False keeps those values
# in f32: the same graph with f32 storage, which is what an f32 implementation
# of the architecture computes (the reference's golden generator,
# goldens/gen.py, runs transformers in f32 on the CPU).
STORE_F16 = True


def f16r(x):
    """Round to f16 and back (where the reference stores an f16 buffer)."""
    if not STORE_F16:
        return np.array(x, dtype=F32)
    return np.asarray(x, dtype=F32).astype(np.float16).astype(F32)


# ------------------------------------------------------------ dequantisation

def deq_q40(raw: np.ndarray) -> np.ndarray:
    """q4_0 blocks -> f32: w = d * (n - 8); byte j = element j (lo) | element j+16 (hi).
    (scripts/ternarize_a4b.py:80-87; kernels/q40mv.wgsl:21-54)"""
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).astype(F32)            # [nb, 1]
    qs = b[:, 2:]
    lo = (qs & 0x0F).astype(np.int8) - 8
    hi = (qs >> 4).astype(np.int8) - 8
    q = np.concatenate([lo, hi], axis=1).astype(F32)             # [nb, 32]
    return (d * q).reshape(-1)


def deq_q6k(raw: np.ndarray) -> np.ndarray:
    """q6_K blocks -> f32: w = (d * sc[e/16]) * (q_e - 32) with the ggml element order
    (kernels/q6k.wgsl:44-68: q1..q4 from ql[l], ql[l+32] lo/hi nibbles and qh[l] bit pairs)."""
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 210)
    nb = b.shape[0]
    ql = b[:, :128].reshape(nb, 2, 64)
    qh = b[:, 128:192].reshape(nb, 2, 32)
    sc = b[:, 192:208].copy().view(np.int8).astype(F32)          # [nb, 16]
    d = b[:, 208:210].copy().view(np.float16).astype(F32)        # [nb, 1]
    q = np.empty((nb, 2, 4, 32), dtype=np.int32)                 # [half][j][l]
    for j in range(4):
        src = ql[:, :, (j & 1) * 32:(j & 1) * 32 + 32]
        lo = (src >> ((j >> 1) * 4)) & 0xF
        hb = (qh >> (2 * j)) & 3
        q[:, :, j, :] = lo.astype(np.int32) | (hb.astype(np.int32) << 4)
    q = (q - 32).reshape(nb, 256).astype(F32)
    scale = (d * np.repeat(sc, 16, axis=1))                      # exact: d*sc
    return (scale * q).reshape(-1)


# ------------------------------------------------------------ primitives

def gelu_tanh(g):
    """gelu_pytorch_tanh with the reference's inner clamp (kernels/q40gu.wgsl:114)."""
    g = np.asarray(g, dtype=F32)
    t = F32(0.7978845608028654) * (g + F32(0.044715) * (g * g * g))
    t = np.clip(t, F32(-20.0), F32(20.0))
    return (F32(0.5) * g) * (F32(1.0) + np.tanh(t))


def rms_inv(x, eps):
    x = np.asarray(x, dtype=F32)
    ms = np.sum(x * x, dtype=F32, axis=-1, keepdims=True) / F32(x.shape[-1])
    return (ms + F32(eps)) ** F32(-0.5)


def rmsnorm(x, w, eps, with_scale=True):
    """y = x * (mean(x^2)+eps)^-0.5 [* w]  (kernels/rmsnorm.wgsl:13-51)."""
    x = np.asarray(x, dtype=F32)
    y = x * rms_inv(x, eps)
    return y * w if with_scale else y


def q40mv(w_raw, x, rows, n_in):
    """y[o] = sum_b d_b sum_i (n_i-8) x_i  (kernels/q40mv.wgsl:56-89)."""
    w_raw, wp = _u8(w_raw)
    x, xp = _f32(x)
    assert x.size == n_in and w_raw.size == rows * n_in // 32 * 18
    y = np.empty(rows, dtype=F32)
    qlib().oracle_q40_matvec(wp, xp, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rows, n_in)
    return y


def q6k_matvec(w_raw, x, rows, n_in):
    """logits[o] = sum d*sc*(q-32)*x  (kernels/q6k.wgsl:75-127)."""
    w_raw, wp = _u8(w_raw)
    x, xp = _f32(x)
    y = np.empty(rows, dtype=F32)
    qlib().oracle_q6k_matvec(wp, xp, y.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), rows, n_in)
    return y


def q6k_row(w_raw, row, n_in, mult):
    """One embedding row: ((d*sc)*(q-32))*mult  (kernels/q6k.wgsl:37-73, MODE 0)."""
    w_raw, wp = _u8(w_raw)
    out = np.empty(n_in, dtype=F32)
    qlib().oracle_q6k_rows(wp, out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), int(row), 1, n_in, F32(mult))
    return out


def softcap(z, cap):
    """cap * tanh(z / cap)  (kernels/q6k.wgsl:129)."""
    if cap == 0:
        return np.asarray(z, dtype=F32)
    return F32(cap) * np.tanh(np.asarray(z, dtype=F32) / F32(cap))


def argmax_first(x):
    """Largest value, ties -> lowest index (kernels/argmax2.wgsl:21, 37)."""
    return int(np.argmax(np.asarray(x, dtype=F32)))


# ------------------------------------------------------------ fused norms

def rmsacc(x, w, hidden, eps, mul=1.0):
    """hidden = (hidden + rms(x)*w) * mul  (kernels/rmsacc.wgsl:10-26)."""
    return (np.asarray(hidden, F32) + rmsnorm(x, w, eps)) * F32(mul)


def rmsacc3(t, w_acc, w1, w2, w3, h_in, eps):
    """hOut = hIn + rms(t)*wAcc; v = rms(hOut); y1 = f16(v*w1), y2 = v*w2, y3 = f16(v*w3)
    (kernels/rmsacc3.wgsl:27-53)."""
    h = np.asarray(h_in, F32) + rmsnorm(t, w_acc, eps)
    v = h * rms_inv(h, eps)
    return h, f16r(v * w1), (v * w2).astype(F32), f16r(v * w3)


def a4btail(t1, w1, m, w2, wp, h_in, w_next, eps, mul, nxt=True):
    """c = rms(t1)*w1 + rms(m)*w2; h = (hIn + rms(c)*wp)*mul; yNext = f16(rms(h)*wNext)
    (kernels/a4btail.wgsl:26-71)."""
    c = rmsnorm(t1, w1, eps) + rmsnorm(m, w2, eps)
    h = (np.asarray(h_in, F32) + rmsnorm(c, wp, eps)) * F32(mul)
    y = f16r(rmsnorm(h, w_next, eps)) if nxt else None
    return h, y


# ------------------------------------------------------------ attention

def rope_pairs(x, pos, angles, theta, hd):
    """Rotate pairs (p, p+hd/2) for p < angles by pos*theta^(-2p/hd)  (kernels/rope.wgsl:8-27)."""
    x = np.asarray(x, F32).copy()
    half = hd // 2
    p = np.arange(angles, dtype=F32)
    inv = np.power(F32(theta), (F32(-2.0) * p) / F32(hd)).astype(F32)
    th = (F32(pos) * inv).astype(F32)
    c, s = np.cos(th).astype(F32), np.sin(th).astype(F32)
    x0 = x[..., :angles].copy()
    x1 = x[..., half:half + angles].copy()
    x[..., :angles] = x0 * c - x1 * s
    x[..., half:half + angles] = x0 * s + x1 * c
    return x


def headprep(qkv, qw, kw, pos, qh, kvh, hd, angles, theta, eps, keqv):
    """Per-head RMSNorm (q_norm / k_norm; scale-less for v) + RoPE on q and k
    (kernels/headprep.wgsl:19-87).  Returns q [qh,hd] f32, k, v [kvh,hd] as stored
    in the f16 cache."""
    qkv = np.asarray(qkv, F32)
    q = qkv[:qh * hd].reshape(qh, hd)
    k = qkv[qh * hd:(qh + kvh) * hd].reshape(kvh, hd)
    v = k if keqv else qkv[(qh + kvh) * hd:(qh + 2 * kvh) * hd].reshape(kvh, hd)
    qn = rope_pairs(q * rms_inv(q, eps) * qw, pos, angles, theta, hd)
    kn = rope_pairs(k * rms_inv(k, eps) * kw, pos, angles, theta, hd)
    vn = v * rms_inv(v, eps)
    return qn.astype(F32), f16r(kn), f16r(vn)


def ring_positions(qp, ring):
    """True position of every ring slot when the newest written position is qp
    (kernels/attnf32.wgsl:36-53: ps = maxW - ((maxW + RING - t) % RING))."""
    t = np.arange(ring, dtype=np.int64)
    return qp - ((qp + ring - t) % ring)


def attend(q, kc, vc, valid, scale=1.0):
    """Dense fp32 softmax attention of one q head over slots `valid` of one kv head.
    Returns (o [hd], lse).  (kernels/attnos.wgsl / attsplit.wgsl semantics.)"""
    k = kc[valid].astype(F32)
    v = vc[valid].astype(F32)
    s = (k @ np.asarray(q, F32)) * F32(scale)
    m = s.max()
    e = np.exp(s - m)
    den = e.sum(dtype=F32)
    o = (e @ v) / den
    return o.astype(F32), F32(m + np.log(den))


def attention_mass(q, kcache, length, kvh, scale=1.0):
    """Per-slot normalised attention probability of every q head over the first
    `length` slots of a counted cache, [qh][length] f32: the SCORE=1 pass of
    kernels/attnos.wgsl:82-97 (exp(s - gm) / denom)."""
    qh, hd = q.shape
    grp = qh // kvh
    out = np.empty((qh, length), F32)
    for h in range(qh):
        k = kcache[:length, h // grp].astype(F32)
        s = (k @ np.asarray(q[h], F32)) * F32(scale)
        e = np.exp(s - s.max())
        out[h] = e / e.sum(dtype=F32)
    return out


def budget_keep(scores, n, budget, protect):
    """The slots a budget compaction keeps (src/engine-a4b.js:589-603): mass[t] =
    sum over heads of the accumulated scores (f64), the `protect` most recent
    slots always, plus the top (budget - protect) others by mass (ties: lower
    slot first, the stable sort), ascending."""
    mass = np.asarray(scores, np.float64)[:, :n].sum(axis=0)
    prot = min(protect, n)
    cand = np.argsort(-mass[:n - prot], kind="stable")
    keep = np.concatenate([cand[:max(budget - prot, 0)], np.arange(n - prot, n)])
    return np.sort(keep).astype(np.uint32)


def decode_attention(q, kcache, vcache, qp, kvh, window, ring, cachemode, length):
    """Decode attention for all q heads (GQA kvh = h / (QH/KVH)); output f16-rounded
    like the reference's attnOut buffer.  cachemode 1 = sliding ring, 2 = linear."""
    qh, hd = q.shape
    grp = qh // kvh
    out = np.empty((qh, hd), F32)
    if cachemode == 1:
        n = min(qp + 1, ring)
        ps = ring_positions(qp, ring)[:n]
        valid = np.nonzero((ps <= qp) & (ps + window > qp))[0]
    else:
        valid = np.arange(length)
    for h in range(qh):
        o, _ = attend(q[h], kcache[:, h // grp], vcache[:, h // grp], valid)
        out[h] = o
    return f16r(out)


# ------------------------------------------------------------ ternary experts

def t2_unpack(w, cols):
    """2-bit shift-group planes -> t in {-1, 0, 1} [rows][cols]: element 4g + j of a
    word at bits 2g + 8j, stored t + 1 (scripts/ternarize_a4b.py pack_t2,
    kernels/t2gu.wgsl t2dot16)."""
    w = np.asarray(w, np.uint32).reshape(-1, cols // 16)
    out = np.empty((w.shape[0], cols // 16, 16), np.int8)
    for g in range(4):
        for j in range(4):
            out[:, :, 4 * g + j] = ((w >> np.uint32(2 * g + 8 * j)) & np.uint32(3)).astype(np.int8) - 1
    return out.reshape(w.shape[0], cols)


def t2gu(x, w, scale, topk, n_in, ff):
    """Expert slots of the fused gate|up + GeGLU on ternary rows [e][gate ff | up ff]
    (kernels/t2gu.wgsl expert branch): f16(gelu(a_g t_g.x) * a_u t_u.x) per slot."""
    xs = np.asarray(x, F32)
    out = np.empty((len(topk), ff), F32)
    for k, e in enumerate(topk):
        rows = t2_unpack(w[int(e) * 2 * ff * (n_in // 16):(int(e) + 1) * 2 * ff * (n_in // 16)], n_in).astype(F32)
        sc = np.asarray(scale[int(e) * 2 * ff:(int(e) + 1) * 2 * ff]).astype(F32)
        acc = (rows @ xs).astype(F32) * sc
        out[k] = gelu_tanh(acc[:ff]) * acc[ff:]
    return f16r(out)


def t2moedown(x_slots, w, scale, topk, topk_w, n_in, n_out):
    """y = sum_k w_k * a[e_k] * t[e_k] . x_k  (kernels/t2moedown.wgsl)."""
    y = np.zeros(n_out, F32)
    for k, e in enumerate(topk):
        rows = t2_unpack(w[int(e) * n_out * (n_in // 16):(int(e) + 1) * n_out * (n_in // 16)], n_in).astype(F32)
        sc = np.asarray(scale[int(e) * n_out:(int(e) + 1) * n_out]).astype(F32)
        y = y + F32(topk_w[k]) * ((rows @ np.asarray(x_slots[k], F32)).astype(F32) * sc)
    return y.astype(F32)


# ------------------------------------------------------------ MoE

def router_topk(router_in, wr, pes, k):
    """scores = Wr . routerIn; softmax; k x (strict >, lowest index wins) ; renorm ; x pes
    (kernels/routertop.wgsl:51-69; the H^-0.5 / input-scale fold is in routerIn,
    src/engine-a4b.js:174-179)."""
    s = (np.asarray(wr, F32) @ np.asarray(router_in, F32)).astype(F32)
    mx = s.max()
    p = np.exp(s - mx).astype(F32)
    tot = F32(0.0)
    for v in p:                      # sequential f32 sum, as the single-thread epilogue does
        tot = F32(tot + v)
    idx, w = [], []
    wsum = F32(0.0)
    pp = p.copy()
    for _ in range(k):
        bi = int(np.argmax(pp))      # first maximum == strict '>' scan from index 0
        bv = pp[bi]
        idx.append(bi)
        w.append(F32(bv / tot))
        wsum = F32(wsum + F32(bv / tot))
        pp[bi] = F32(-2.0)
    w = np.array([F32(x / wsum) * F32(pes[i]) for x, i in zip(w, idx)], dtype=F32)
    return np.array(idx, dtype=np.uint32), w


def moe_down(x_slots, w_exps_raw, topk_idx, topk_w, n_in, n_out):
    """y = sum_k w_k * (W_e(k) x_k)  (kernels/q40moedown.wgsl:42-75)."""
    per = n_out * n_in // 32 * 18
    y = np.zeros(n_out, F32)
    for k, e in enumerate(topk_idx):
        yk = q40mv(w_exps_raw[int(e) * per:(int(e) + 1) * per], x_slots[k], n_out, n_in)
        y += F32(topk_w[k]) * yk
    return y


def geglu_rows(gu, ff):
    """[gate | up] -> f16(gelu_tanh(gate) * up)  (kernels/q40gu.wgsl:111-117)."""
    gu = np.asarray(gu, F32)
    return f16r(gelu_tanh(gu[..., :ff]) * gu[..., ff:2 * ff])

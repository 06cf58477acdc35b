"""Grouped MoE for batched decode (expgroup -> q40gugrp -> q40downgrp -> wacc)
against the per-token oracle: y_t = sum_k w_tk * W_down[e_tk] f16(gelu(gate) * up)
with [gate | up] = W_gu[e_tk] x_t (kernels/q40gugrp.wgsl, q40downgrp.wgsl,
wacc.wgsl semantics; src/engine-a4b.js:437-462 per token)."""
import numpy as np
import pytest

from oracle import ops as O

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
    bx, bgu, bdn = d.upload(x.astype(np.float16)), d.upload(wgu), d.upload(wdn)
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

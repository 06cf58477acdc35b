"""Ternary MoE experts: the reference's Campaign-6 expert format
(scripts/ternarize_a4b.py, kernels/t2gu.wgsl, kernels/t2moedown.wgsl).

Every expert row of the q4_0 gate|up and down tensors becomes t in {-1, 0, 1}
times one f16 row scale alpha (round-to-nearest ternarisation: alpha =
mean |w| of the row, t = clip(round(w / alpha), -1, 1); with per-column
activation statistics h, a few rounds of the h-weighted least-squares alpha,
as the reference's "aa" mode).  Storage: 2-bit planes, 16 values per u32 in
the shift-group layout (element 4g + j of a word at bits 2g + 8j, value t + 1),
2.25 bits per weight with the scales versus 4.5 for q4_0.
"""
from __future__ import annotations

import numpy as np

from . import gguf


def pack_t2(t: np.ndarray) -> np.ndarray:
    """t [rows][cols] in {-1, 0, 1}, cols % 16 == 0 -> u32 [rows][cols / 16]."""
    r, c = t.shape
    if c % 16:
        raise ValueError(f"ternary rows need a multiple of 16 columns, got {c}")
    u = (np.asarray(t, np.int64) + 1).astype(np.uint32).reshape(r, c // 16, 4, 4)   # [.., group g, lane j]
    out = np.zeros((r, c // 16), np.uint32)
    for g in range(4):
        for j in range(4):
            out |= u[:, :, g, j] << np.uint32(2 * g + 8 * j)
    return out


def ternarize_rows(w: np.ndarray, h: np.ndarray | None = None, iters: int = 5):
    """w [rows][cols] f32 -> (alpha [rows] f32, t [rows][cols] int8)."""
    w = np.asarray(w, np.float32)
    alpha = np.clip(np.abs(w).mean(axis=1, keepdims=True), 1e-8, None)
    t = np.clip(np.round(w / alpha), -1, 1)
    if h is not None:
        hw = np.clip(np.asarray(h, np.float32), 1e-12, None)[None, :]
        for _ in range(iters):
            num = (hw * w * t).sum(1, keepdims=True)
            den = np.clip((hw * t * t).sum(1, keepdims=True), 1e-12, None)
            alpha = np.clip(num / den, 1e-8, None)
            t = np.clip(np.round(w / alpha), -1, 1)
    return alpha[:, 0].astype(np.float32), t.astype(np.int8)


def _deq_q40(raw: np.ndarray) -> np.ndarray:
    b = np.asarray(raw, np.uint8).reshape(-1, 18)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    q = b[:, 2:]
    vals = np.concatenate([(q & 15).astype(np.int8) - 8, (q >> 4).astype(np.int8) - 8], axis=1).astype(np.float32)
    return (d * vals).reshape(-1)


def ternarize_model(src, layers=None, h_stats=None, rows_per_pass: int = 4096):
    """Ternary copies of every MoE layer's expert tensors of a GGUF image:
    {layer: {"gu": (planes, scales), "down": (planes, scales)}} with planes u32
    [E * rows][cols / 16] and scales f16 [E * rows] (rows in the q4_0 tensor's
    order: gate|up = [e][gate FF | up FF] x H, down = [e][H] x FF).  h_stats:
    optional {(layer, "gu" | "down"): per-column weights} for the weighted mode."""
    g = gguf.open_gguf(src)
    kv = g.kv
    L = int(kv["gemma4.block_count"])
    H = int(kv["gemma4.embedding_length"])
    EF = int(kv.get("gemma4.expert_feed_forward_length", 0))
    if not EF:
        raise ValueError("the model has no experts")
    out = {}
    for l in (range(L) if layers is None else layers):
        res = {}
        for key, name, cols in (("gu", f"blk.{l}.ffn_gate_up_exps.weight", H), ("down", f"blk.{l}.ffn_down_exps.weight", EF)):
            raw = np.asarray(g.fetch(name), np.uint8)
            nrows = raw.size // (cols // 32 * 18)
            planes = np.empty((nrows, cols // 16), np.uint32)
            scales = np.empty(nrows, np.float16)
            h = None if h_stats is None else h_stats.get((l, key))
            for r0 in range(0, nrows, rows_per_pass):
                r1 = min(nrows, r0 + rows_per_pass)
                w = _deq_q40(raw[r0 * (cols // 32) * 18:r1 * (cols // 32) * 18]).reshape(r1 - r0, cols)
                a, t = ternarize_rows(w, h)
                planes[r0:r1] = pack_t2(t)
                scales[r0:r1] = a.astype(np.float16)
            res[key] = (planes, scales)
        out[l] = res
    return out

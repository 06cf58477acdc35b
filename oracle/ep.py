"""CPU ORACLE -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the expert-parallel MoE exchange that the batched
decode runs over NCCL (e4b-webgpu_b200/csrc/ep.cu, e4b-webgpu_b200/batch.py
BatchEngine._moe_ep): experts in contiguous blocks of E/N per rank; entry
i = t*K + k of a rank's topk goes to rank e // (E/N) at the next free position
of that peer's fixed-capacity slab (entry order); the owner groups what it
received by local expert, computes the expert rows, and sends each result back
into the slab position it came from; the source combines sum_k w[t][k] *
y[slot[t*K+k]] in slot order (kernels/wacc.wgsl).  The reference itself is
single-GPU (src/engine-a4b.js:437-462 per token): this protocol must reproduce
its per-token MoE output exactly.  Only tests use this module, as a checker.
"""
from __future__ import annotations

import numpy as np

from . import ops as O

NONE = 0xFFFFFFFF
F32 = np.float32


def owner(e: int, E: int, N: int) -> int:
    return int(e) // (E // N)


def dispatch(topk: np.ndarray, E: int, N: int, cap: int):
    """topk [T][K] -> (ids [N][cap] local expert ids or NONE, src [N][cap] entry
    index or -1, slot [T*K] = dest*cap + pos)."""
    flat = np.asarray(topk).reshape(-1)
    ids = np.full((N, cap), NONE, np.uint32)
    src = np.full((N, cap), -1, np.int64)
    slot = np.zeros(flat.size, np.int64)
    fill = [0] * N
    per = E // N
    for i, e in enumerate(flat):
        d = owner(e, E, N)
        pos = fill[d]
        if pos >= cap:
            raise OverflowError(f"peer {d} slab of {cap} entries is full")
        fill[d] += 1
        ids[d, pos] = int(e) - d * per
        src[d, pos] = i
        slot[i] = d * cap + pos
    return ids, src, slot


def expert_rows(recv_ids: np.ndarray, recv_x: np.ndarray, rank: int, E: int, N: int, w_gu: np.ndarray,
                w_dn: np.ndarray, H: int, EF: int) -> np.ndarray:
    """Result row for every received row (zeros where the id is NONE): the
    owner's expert e_local applied to the row (GeGLU in f16, as q40gugrp)."""
    per = E // N
    per_gu = 2 * EF * H // 32 * 18
    per_dn = H * EF // 32 * 18
    ids = np.asarray(recv_ids).reshape(-1)
    xs = np.asarray(recv_x, F32).reshape(ids.size, H)
    out = np.zeros((ids.size, H), F32)
    for i, el in enumerate(ids):
        if el == NONE:
            continue
        e = rank * per + int(el)
        g = O.geglu_rows(O.q40mv(w_gu[e * per_gu:(e + 1) * per_gu], xs[i], 2 * EF, H), EF)
        out[i] = O.q40mv(w_dn[e * per_dn:(e + 1) * per_dn], g, H, EF)
    return out


def combine(recv_y: np.ndarray, slot: np.ndarray, topk_w: np.ndarray) -> np.ndarray:
    """m[t] = sum_k w[t][k] * y[slot[t*K+k]], slots in order (kernels/wacc.wgsl)."""
    T, K = np.asarray(topk_w).shape
    ys = np.asarray(recv_y, F32).reshape(-1, np.asarray(recv_y).shape[-1])
    m = np.zeros((T, ys.shape[1]), F32)
    for t in range(T):
        acc = np.zeros(ys.shape[1], F32)
        for k in range(K):
            acc = (acc + F32(topk_w[t, k]) * ys[slot[t * K + k]]).astype(F32)
        m[t] = acc
    return m


def exchange(send: list) -> list:
    """The NCCL all-to-all of fixed slabs: recv[d][p*cap + j] = send[p][d*cap + j]
    (send[p] of N*cap rows on rank p)."""
    N = len(send)
    cap = send[0].shape[0] // N
    return [np.concatenate([send[p][d * cap:(d + 1) * cap] for p in range(N)]) for d in range(N)]


def push(rows_by_entry: list, slots: list, cap: int, template) -> list:
    """The peer-memory transport (ep_push / ep_push_back): rank p stores the row
    of each entry with slot d*cap + pos straight into rank d's receive slab at
    row p*cap + pos; rows not stored keep `template` (unused slots)."""
    N = len(slots)
    recv = [np.array(template, copy=True) for _ in range(N)]
    for p in range(N):
        for i, sl in enumerate(np.asarray(slots[p]).reshape(-1)):
            if sl < 0:
                continue
            d, pos = divmod(int(sl), cap)
            recv[d][p * cap + pos] = rows_by_entry[p][i]
    return recv

"""The expert-parallel exchange protocol on CPU: two gloo ranks run the
dispatch / all-to-all / expert / return / combine steps of oracle/ep.py and
must reproduce the single-process per-token MoE (src/engine-a4b.js:437-462)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import ep as EP
from oracle import ops as O

F32 = np.float32
E, K, H, EF, T = 8, 3, 64, 32, 5        # T tokens per rank


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _problem(N):
    from importlib import import_module
    e4b = import_module("e4b-webgpu_b200")
    rng = np.random.default_rng(11)
    w_gu = e4b.synth.quant_q4_0(e4b.synth.normal_f32(E * 2 * EF * H, 5, "epgu", 0.05))
    w_dn = e4b.synth.quant_q4_0(e4b.synth.normal_f32(E * H * EF, 6, "epdn", 0.05))
    x = O.f16r(rng.standard_normal((N, T, H)).astype(F32))
    topk = np.stack([[rng.choice(E, K, replace=False) for _ in range(T)] for _ in range(N)]).astype(np.uint32)
    if N > 1:
        topk[1, :, 0] = 0           # rank 1 sends its first slot of every token to rank 0
    w = rng.uniform(0.1, 0.5, (N, T, K)).astype(F32)
    return w_gu, w_dn, x, topk, w


def _rank(rank, N, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=N)
    try:
        w_gu, w_dn, x, topk, w = _problem(N)
        cap = T * K
        ids, src, slot = EP.dispatch(topk[rank], E, N, cap)
        sx = np.zeros((N, cap, H), F32)
        for d in range(N):
            for p in range(cap):
                if src[d, p] >= 0:
                    sx[d, p] = x[rank, src[d, p] // K]
        rx = torch.empty(N * cap * H)
        dist.all_to_all_single(rx, torch.from_numpy(sx.reshape(-1)))
        rid = torch.empty(N * cap, dtype=torch.int64)
        dist.all_to_all_single(rid, torch.from_numpy(ids.reshape(-1).astype(np.int64)))
        y = EP.expert_rows(rid.numpy().astype(np.uint32), rx.numpy(), rank, E, N, w_gu, w_dn, H, EF)
        ry = torch.empty(N * cap * H)
        dist.all_to_all_single(ry, torch.from_numpy(y.reshape(-1)))
        m = EP.combine(ry.numpy().reshape(N * cap, H), slot, w[rank])
        q.put((rank, m))
    finally:
        dist.destroy_process_group()


def _reference(N):
    w_gu, w_dn, x, topk, w = _problem(N)
    per_gu = 2 * EF * H // 32 * 18
    out = np.zeros((N, T, H), F32)
    for r in range(N):
        for t in range(T):
            slots = np.stack([O.geglu_rows(O.q40mv(w_gu[int(e) * per_gu:(int(e) + 1) * per_gu], x[r, t], 2 * EF, H),
                                           EF) for e in topk[r, t]])
            out[r, t] = O.moe_down(slots, w_dn, topk[r, t], w[r, t], EF, H)
    return out


def test_dispatch_slots_and_owners():
    topk = np.array([[7, 0, 3], [4, 1, 6]], np.uint32)
    ids, src, slot = EP.dispatch(topk, 8, 2, 6)
    # rank 0 owns experts 0-3, rank 1 owns 4-7; positions in entry order
    assert list(ids[0, :3]) == [0, 3, 1] and list(src[0, :3]) == [1, 2, 4]
    assert list(ids[1, :3]) == [3, 0, 2] and list(src[1, :3]) == [0, 3, 5]
    assert list(slot) == [6, 0, 1, 7, 2, 8]
    assert (ids[:, 3:] == EP.NONE).all()
    with pytest.raises(OverflowError):
        EP.dispatch(topk, 8, 2, 2)


@pytest.mark.parametrize("N", [2])
def test_ep_exchange_matches_single_process_moe(N):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, N, port, q)) for r in range(N)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(N))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    ref = _reference(N)
    for r in range(N):
        # same products and slot order; numpy's f32 dot inside q40mv may sum in another order
        assert np.allclose(got[r], ref[r], rtol=1e-5, atol=1e-6), r


@pytest.mark.parametrize("N", [2, 4])
def test_peer_stores_land_where_the_nccl_exchange_puts_rows(N):
    """Rows stored by the peer-memory transport (entry with slot d*cap + pos of
    rank p -> rank d's slab row p*cap + pos) fill the same receive slab as the
    NCCL exchange of the dispatched send slabs, ids included; the results go back
    the same way (owner row p*cap + pos -> source p's row owner*cap + pos)."""
    rng = np.random.default_rng(N)
    T, K, E, H = 5, 3, 4 * N, 8
    cap = T * K
    topks = [np.stack([rng.choice(E, K, replace=False) for _ in range(T)]) for _ in range(N)]
    xs = [rng.standard_normal((T, H)).astype(np.float32) for _ in range(N)]
    disp = [EP.dispatch(tk, E, N, cap) for tk in topks]
    send_x, send_id = [], []
    for p in range(N):
        ids, src, slot = disp[p]
        sx = np.zeros((N * cap, H), np.float32)
        for d in range(N):
            for j in range(cap):
                if src[d, j] >= 0:
                    sx[d * cap + j] = xs[p][src[d, j] // K]
        send_x.append(sx)
        send_id.append(ids.reshape(-1, 1).astype(np.int64))
    via_nccl = EP.exchange(send_x)
    ids_nccl = EP.exchange(send_id)
    rows = [np.repeat(xs[p], K, axis=0) for p in range(N)]
    via_push = EP.push(rows, [disp[p][2] for p in range(N)], cap, np.zeros((N * cap, H), np.float32))
    # id rows: every slot of a peer's cap region is written (NONE where unused)
    ids_push = [np.concatenate([disp[p][0][d].reshape(-1, 1) for p in range(N)]).astype(np.int64) for d in range(N)]
    for d in range(N):
        assert np.array_equal(ids_push[d], ids_nccl[d])
        used = ids_nccl[d][:, 0] != EP.NONE
        assert np.array_equal(via_push[d][used], via_nccl[d][used])
    # results: owner d's row p*cap + pos back to source p's row d*cap + pos
    ys = [rng.standard_normal((N * cap, H)).astype(np.float32) for _ in range(N)]
    back_nccl = EP.exchange(ys)
    back_push = [np.zeros((N * cap, H), np.float32) for _ in range(N)]
    for d in range(N):
        for i in range(N * cap):
            p, pos = divmod(i, cap)
            back_push[p][d * cap + pos] = ys[d][i]
    for p in range(N):
        assert np.array_equal(back_push[p], back_nccl[p])

"""Expert-parallel batched MoE decode (benchmark config 5) on the GPU: the
dispatch kernel against the oracle's slab layout, a one-rank NCCL group (the
full dispatch / exchange / return path on one GPU) and, where the box has two
GPUs, two ranks over each transport (NCCL send/recv; rows and results stored
into the peers' memory through CUDA IPC) -- each must reproduce the single-GPU
BatchEngine exactly.  The peer-memory transport needs a process per GPU, so it
has no one-GPU case."""
import os
import socket

import numpy as np
import pytest

from oracle import ep as EP

pytestmark = pytest.mark.gpu


def test_ep_dispatch_matches_oracle(e4b, dev):
    rng = np.random.default_rng(4)
    T, K, E, N, H = 9, 4, 16, 4, 64
    topk = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.uint32)
    x = rng.standard_normal((T, H)).astype(np.float16)
    cap = T * K
    sx, sid, slot = dev.alloc(N * cap * H * 2), dev.alloc(N * cap * 4), dev.alloc(T * K * 4)
    dev.call("e4b_ep_dispatch", dev.upload(topk).ptr, T, K, E, N, cap, dev.upload(x).ptr, H, sx.ptr, sid.ptr, slot.ptr)
    dev.sync()
    assert dev.status() == 0
    ids, src, rslot = EP.dispatch(topk, E, N, cap)
    assert np.array_equal(dev.read(sid, np.uint32, N * cap).reshape(N, cap), ids)
    assert np.array_equal(dev.read(slot, np.uint32, T * K), rslot.astype(np.uint32))
    gx = dev.read(sx, np.float16, N * cap * H).reshape(N, cap, H)
    for d in range(N):
        for p in range(cap):
            if src[d, p] >= 0:
                assert np.array_equal(gx[d, p], x[src[d, p] // K])


def _run_batch(e4b, buf, prompts, n_new, device, ep=None, zipf=None, tok0=0, transport="nccl"):
    """Token-by-token prefill on every path, so that one GPU and the expert-
    parallel ranks (which prefill token by token) run the same arithmetic."""
    eng = e4b.BatchEngine(buf, prompts.shape[0], device, ep=ep, zipf=zipf, tok0=tok0, ep_transport=transport)
    try:
        ids = eng.generate(prompts, n_new, chunk=0)
        h = eng.read_hidden()
        assert eng.dev.status() == 0
    finally:
        eng.close()
    return ids, h


def test_ep_one_rank_matches_single_gpu(e4b, models):
    buf = models("tiny_moe")
    cfg = e4b.config.get("tiny_moe")
    B, P, N = 4, 6, 5
    prompts = np.stack([e4b.synth.prompt_ids(P, cfg.vocab, seed=300 + b) for b in range(B)])
    ids0, h0 = _run_batch(e4b, buf, prompts, N, 0)
    dev = e4b.Device(0)
    try:
        nid = e4b.batch.nccl_unique_id(dev)
    finally:
        dev.close()
    ids1, h1 = _run_batch(e4b, buf, prompts, N, 0, ep=(1, 0, nid))
    assert np.array_equal(ids0, ids1)
    assert np.array_equal(h0, h1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _ep_rank(rank, N, port, B, P, n_new, q, transport):
    import importlib
    import sys
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    e4b = importlib.import_module("e4b-webgpu_b200")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=N, timeout=datetime.timedelta(seconds=120))
    try:
        cfg = e4b.config.get("tiny_moe")
        buf = e4b.synth.build_model(cfg)
        prompts = np.stack([e4b.synth.prompt_ids(P, cfg.vocab, seed=300 + b) for b in range(B)])
        mine = prompts[rank * (B // N):(rank + 1) * (B // N)]
        obj = [None]
        if rank == 0:
            dev = e4b.Device(0)
            obj[0] = e4b.batch.nccl_unique_id(dev)
            dev.close()
        dist.broadcast_object_list(obj, src=0)
        ids, h = _run_batch(e4b, buf, mine, n_new, rank, ep=(N, rank, obj[0]), zipf=1.1, tok0=rank * (B // N),
                            transport=transport)
        q.put((rank, ids, h))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_ep_two_ranks_match_single_gpu(e4b, models, transport):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    buf = models("tiny_moe")
    cfg = e4b.config.get("tiny_moe")
    B, P, n_new, N = 6, 6, 5, 2
    prompts = np.stack([e4b.synth.prompt_ids(P, cfg.vocab, seed=300 + b) for b in range(B)])
    ids0, h0 = _run_batch(e4b, buf, prompts, n_new, 0, zipf=1.1)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, N, port, B, P, n_new, q, transport)) for r in range(N)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(N):
        r, ids, h = q.get(timeout=300)
        got[r] = (ids, h)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ids = np.concatenate([got[r][0] for r in range(N)])
    h = np.concatenate([got[r][1] for r in range(N)])
    assert np.array_equal(ids, ids0)
    assert np.array_equal(h, h0)


def test_route_zipf(e4b, dev):
    """Benchmark routing: K distinct experts per token, a pure function of
    (seed, layer, position, global token), skewed towards few experts."""
    n, K, E = 512, 8, 128
    params = np.zeros(8, np.uint32)
    params[0] = 77
    bp = dev.upload(params)
    out = []
    for tok0, cnt in ((0, n), (100, n - 100)):
        idx, w = dev.alloc(cnt * K * 4), dev.alloc(cnt * K * 4)
        dev.call("e4b_route_zipf", bp.ptr, idx.ptr, w.ptr, cnt, K, E, np.float32(1.1), np.uint32(5), 3, tok0)
        dev.sync()
        out.append((dev.read(idx, np.uint32, cnt * K).reshape(cnt, K), dev.read(w, np.float32, cnt * K)))
    a, wa = out[0]
    assert all(len(set(r)) == K for r in a) and a.max() < E
    assert np.allclose(wa, 1.0 / K)
    assert np.array_equal(a[100:], out[1][0])            # same draw for the same global token
    counts = np.bincount(a.reshape(-1), minlength=E)
    assert counts.max() > 4 * counts.mean()               # skewed load


def test_route_zipf_layers_matches_per_layer(e4b, dev):
    """The one-launch-per-step form (a table built once by e4b_zipf_table, every
    layer's rows in one grid) draws exactly what e4b_route_zipf draws layer by
    layer."""
    n, K, E, layers, s, seed, tok0 = 64, 8, 128, 5, 1.1, 1234, 3
    params = np.zeros(8, np.uint32)
    params[0] = 517
    bp = dev.upload(params)
    table = dev.alloc(2 * E * 4)
    dev.call("e4b_zipf_table", table.ptr, E, np.float32(s), np.uint32(seed))
    idx_all, w_all = dev.alloc(layers * n * K * 4), dev.alloc(layers * n * K * 4)
    dev.call("e4b_route_zipf_layers", bp.ptr, table.ptr, idx_all.ptr, w_all.ptr, n, layers, K, E, np.uint32(seed), 0,
             tok0)
    dev.sync()
    got = dev.read(idx_all, np.uint32, layers * n * K).reshape(layers, n, K)
    gw = dev.read(w_all, np.float32, layers * n * K)
    assert np.allclose(gw, 1.0 / K)
    for layer in range(layers):
        idx, w = dev.alloc(n * K * 4), dev.alloc(n * K * 4)
        dev.call("e4b_route_zipf", bp.ptr, idx.ptr, w.ptr, n, K, E, np.float32(s), np.uint32(seed), layer, tok0)
        dev.sync()
        assert np.array_equal(got[layer], dev.read(idx, np.uint32, n * K).reshape(n, K)), layer
    assert dev.status() == 0

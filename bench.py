#!/usr/bin/env python
"""Decode benchmark: bs1 greedy decode tok/s of the E4B-shaped q4_0 model
(benchmark config 2: 35 layers, H=2048, 8q/2kv x 256, FF 16384, V 262144, PLE
256/layer, 4 sliding (W=512) : 1 global), as a fraction of the HBM roofline.

A step is one decoded token (one pass of the per-token plan).  Flow:
synthetic GGUF (seeded, in memory) -> Engine (weights resident in HBM) ->
512-token prefill -> W warm-up tokens -> K timed tokens (CUDA events on the
engine's stream; weights >> L2, so no flush is needed between steps) -> the
same K-token decode again through the host API with a host->device parameter
write and a device->host token read every step (`e2e`) -> the dominant
kernel's launches timed alone for the roofline -> the CPU oracle timed on a
bounded sample (`cpu_baseline`).

Multi-GPU: the dense decode does not shard, so N GPUs run N independent
replicas ("replicas only"); value = all tokens / max-over-ranks time.
`--impl reference` times the reference path's CPU restatement (the oracle) on
the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import csv
import importlib
import io
import json
import math
import os
import re
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s bs1 E4B-shaped q4_0 (% of HBM roofline)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def under_torchrun() -> bool:
    """Launched by torch.distributed.run (any --nproc-per-node, 1 included)."""
    return "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ


class Dist:
    """Barrier and max-over-ranks for N > 1 (torch.distributed is plumbing only)."""

    def __init__(self, world, local_rank, backend, timeout_s: float = 120.0):
        """timeout_s bounds every collective: a rank that died or never joined
        ends the others' next barrier / max with an error instead of a hang."""
        self.world = world
        self.pg = None
        if world > 1:
            import datetime
            import torch
            import torch.distributed as td
            if backend == "nccl":
                torch.cuda.set_device(local_rank)
            td.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s))
            self.td, self.torch = td, torch
            self.dev = f"cuda:{local_rank}" if backend == "nccl" else "cpu"

    def barrier(self):
        if self.world > 1:
            self.td.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        self.td.all_reduce(t, op=self.td.ReduceOp.MAX)
        return float(t.item())

    def bcast_bytes(self, b: bytes | None) -> bytes:
        if self.world == 1:
            return b
        obj = [b]
        self.td.broadcast_object_list(obj, src=0)
        return obj[0]

    def close(self):
        if self.world > 1:
            self.td.destroy_process_group()


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled while the timed region runs."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.p = gpu, None

    def start(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-i", str(self.gpu), "-lms", "100"], stdout=subprocess.PIPE,
                                      stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.p = None

    def stop(self):
        if not self.p:
            return None
        self.p.terminate()
        out, _ = self.p.communicate(timeout=10)
        rows = [r for r in csv.reader(io.StringIO(out)) if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if "Active" in v and "Not" not in v:
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].strip().replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def traffic_from_profile(name: str):
    """dram bytes per launch of the dominant kernel from the committed ncu summary."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        txt = open(path).read()
    except OSError:
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)", txt)
    return float(m.group(1)) if m else None


def token_bytes(cfg, ctx_len: int) -> dict:
    """Algorithmic HBM bytes of one decode token (all weights touched once, the
    q6_K LM head, the embedding and PLE-table rows, and the KV cache read over
    the attended positions plus the new K/V write)."""
    H, L = cfg.hidden, cfg.layers
    q4 = lambda rows, n_in: rows * n_in // 32 * 18
    w = 0
    for l in range(L):
        w += q4(cfg.qkv_rows(l), H) + q4(H, cfg.q_dim) + q4(2 * cfg.ff, H) + q4(H, cfg.ff)
        if cfg.ple_dim:
            w += q4(cfg.ple_dim, H) + q4(H, cfg.ple_dim)
    if cfg.ple_dim:
        w += q4(L * cfg.ple_dim, H) + L * cfg.ple_dim // 256 * 210
    head = cfg.vocab * H // 256 * 210
    emb_row = H // 256 * 210
    kv = 0
    per_pos = cfg.kv_heads * cfg.head_dim * 2 * 2
    for l in range(L):
        att = min(ctx_len, cfg.window) if cfg.is_sliding(l) else ctx_len
        kv += att * per_pos + per_pos
    return {"weights": w, "lm_head": head, "embed": emb_row, "kv": kv, "total": w + head + emb_row + kv}


def bench_config(e4b, args):
    """The benchmark config by name; --layers keeps its layer shapes with fewer
    layers (small cases for ncu captures)."""
    import dataclasses
    cfg = e4b.config.get(args.config)
    if args.layers:
        n = args.layers
        cfg = dataclasses.replace(cfg, name=f"{cfg.name}-{n}l", layers=n,
                                  sliding=list(cfg.sliding[:n]) if cfg.sliding else cfg.sliding)
    return cfg


def moe_metric(B: int, world: int) -> str:
    return f"MoE decode tok/s bs{B} A4B-shaped (batched, grouped experts" + (", expert parallel)" if world > 1 else ")")


def expected_unique_experts(E: int, K: int, B: int, zipf: float | None, trials: int = 200) -> float:
    """Expected distinct experts one step's B x K routing touches: uniform
    top-K without replacement, or the Zipf(s) benchmark routing (simulated)."""
    if not zipf:
        return E * (1.0 - (1.0 - K / E) ** B)
    rng = np.random.default_rng(0)
    p = np.arange(1, E + 1, dtype=np.float64) ** (-zipf)
    p /= p.sum()
    tot = 0
    for _ in range(trials):
        seen = set()
        for _ in range(B):
            seen.update(rng.choice(E, K, replace=False, p=p).tolist())
        tot += len(seen)
    return tot / trials


def moe_step_bytes(cfg, B: int, ctx_len: int, zipf: float | None = None) -> dict:
    """Algorithmic HBM bytes of one batched MoE decode step (B tokens): every dense
    / attention / router weight once, the experts the step touches (expected
    distinct experts of B tokens x top-K: E (1 - (1 - K/E)^B) for uniform
    routing, simulated for the Zipf benchmark routing),
    the q6_K LM head, the B embedding rows and every sequence's KV over its
    attended positions plus the new K/V."""
    H, L, E, K = cfg.hidden, cfg.layers, cfg.experts, cfg.topk
    q4 = lambda rows, n_in: rows * n_in // 32 * 18
    uniq = expected_unique_experts(E, K, B, zipf)
    expert = q4(2 * cfg.expert_ff, H) + q4(H, cfg.expert_ff)
    w = 0
    ew = 0
    for l in range(L):
        w += q4(cfg.qkv_rows(l), H) + q4(H, cfg.q_dim) + q4(2 * cfg.ff, H) + q4(H, cfg.ff) + E * H * 4
        ew += int(uniq * expert)
    w += ew
    head = cfg.vocab * H // 256 * 210
    kv = 0
    for l in range(L):
        sliding = cfg.is_sliding(l)
        att = min(ctx_len, cfg.window) if sliding else ctx_len
        shared = cfg.keqv_global and not sliding          # K and V are one cache on those layers
        kv += B * (att + 1) * cfg.kv_heads * cfg.head_dim * 2 * (1 if shared else 2)
    emb = B * (H // 256 * 210)
    return {"weights": w, "expert_weights": ew, "lm_head": head, "embed": emb, "kv": kv,
            "unique_experts_per_layer": round(uniq, 1), "total": w + head + emb + kv}


def run_moe_batch(args, rank, world, local_rank):
    """benchmark configs 4/5: B sequences decoded in lockstep through the grouped
    MoE path; on N > 1 GPUs expert parallelism (B/N sequences and E/N experts
    per rank, NCCL exchange per MoE layer).  value = tokens of all sequences /
    the slowest rank's device time."""
    import ctypes
    e4b = importlib.import_module("e4b-webgpu_b200")
    import __graft_entry__
    __graft_entry__.build()
    dist = Dist(world, local_rank, "gloo" if world > 1 else None)
    cfg = bench_config(e4b, args)
    B = args.batch
    if B % world:
        raise SystemExit(f"--batch {B} does not split over {world} GPUs")
    nloc = B // world
    zipf = args.zipf if args.zipf > 0 else None
    need = args.prefill + args.warmup + 2 * args.steps      # prefill, warm-up, timed and end-to-end tokens
    if need > cfg.max_ctx:
        raise SystemExit(f"{need} positions exceed the {cfg.max_ctx}-slot global-layer KV cache of {cfg.name}; "
                         f"use fewer --steps / --warmup / --prefill")
    t0 = time.time()
    if world > 1:
        # one rank synthesises the image into a shared file, the others map it
        import shutil
        import tempfile
        d = "/dev/shm" if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > (48 << 30) \
            else tempfile.gettempdir()
        path = os.path.join(d, f"e4b_bench_{cfg.name}_seed0_{os.getenv('MASTER_PORT', '0')}.gguf")
        if rank == 0:
            img0 = e4b.synth.build_model(cfg, seed=0)
            img0.tofile(path + ".part")
            del img0
            os.replace(path + ".part", path)       # appears whole or not at all
        else:
            # bounded wait for rank 0's file (the process group's own timeout stays short)
            t_wait = time.time()
            while not os.path.exists(path):
                if time.time() - t_wait > 1800:
                    raise SystemExit(f"rank {rank}: model image {path} not written within 30 min")
                time.sleep(1.0)
        dist.barrier()
        img = path
    else:
        img = e4b.synth.build_model(cfg, seed=0)
    t_build = time.time() - t0
    ep = None
    if world > 1:
        nid = None
        if rank == 0:
            probe = e4b.Device(local_rank)
            nid = e4b.batch.nccl_unique_id(probe)
            probe.close()
        ep = (world, rank, dist.bcast_bytes(nid))
    transport = args.ep_transport if world > 1 else "nccl"
    eng = e4b.BatchEngine(img, nloc, local_rank, ep=ep, zipf=zipf, tok0=rank * nloc, ep_overlap=bool(args.ep_overlap),
                          overlap_route=bool(args.overlap_route),
                          ep_transport=transport)
    dev = eng.dev
    prompts = np.stack([e4b.synth.prompt_ids(args.prefill, cfg.vocab, seed=1000 + b)
                        for b in range(rank * nloc, (rank + 1) * nloc)])
    t1 = time.time()
    dev.sync()
    dev.call("e4b_event_record", 6)
    eng.prefill(prompts)
    dev.call("e4b_event_record", 7)
    dev.sync()
    t_prefill = time.time() - t1
    pms = ctypes.c_float()
    dev.call("e4b_event_elapsed", 6, 7, ctypes.byref(pms))
    t_prefill_dev = dist.max(pms.value / 1000.0)
    pos = args.prefill
    eng.decode_chunk(args.warmup)
    dev.sync()
    pos += args.warmup
    ctx_mid = pos + args.steps // 2
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    dev.sync()
    dev.call("e4b_event_record", 0)
    eng.decode_chunk(args.steps)
    dev.call("e4b_event_record", 1)
    dev.sync()
    dist.barrier()
    ms = ctypes.c_float()
    dev.call("e4b_event_elapsed", 0, 1, ctypes.byref(ms))
    t_dev = dist.max(ms.value / 1000.0)
    pos += args.steps
    clk = clocks.stop()
    # end to end: per step this rank's tokens go host -> device and its results come back
    toks = eng.dev.read(eng.A.tok, np.uint32, nloc)
    host = np.empty(nloc, np.uint32)
    dist.barrier()
    dev.sync()
    dev.call("e4b_event_record", 2)
    for i in range(args.steps):
        eng.step(toks, pos)
        dev.call("e4b_download", host.ctypes.data_as(ctypes.c_void_p), eng.A.tok.ptr, ctypes.c_size_t(4 * nloc))
        toks = host.copy()
        pos += 1
    dev.call("e4b_event_record", 3)
    dev.sync()
    dist.barrier()
    dev.call("e4b_event_elapsed", 2, 3, ctypes.byref(ms))
    t_e2e = dist.max(ms.value / 1000.0)
    a2a = eng.exchange_time(pos) if world > 1 else 0.0
    a2a = dist.max(a2a)
    status = dev.status()
    kpt = eng.kernels_per_token
    eng.close()
    if world > 1:
        dist.barrier()
        if rank == 0:
            os.unlink(img)
    if status:
        raise RuntimeError(f"device status word {status:#x} after the run")
    peak, peak_kind = peaks()
    sb = moe_step_bytes(cfg, B, ctx_mid, zipf)
    # per-GPU algorithmic bytes: replicated dense / attention weights and LM head,
    # this rank's share of the expert bytes and of the KV
    rank_bytes = sb["weights"] - sb["expert_weights"] + sb["expert_weights"] / world + sb["lm_head"] + \
        (sb["embed"] + sb["kv"]) / world
    value = B * args.steps / t_dev
    ach = rank_bytes * args.steps / t_dev / 1e9
    out = {
        "metric": moe_metric(B, world),
        "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1000 * t_dev / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "q4_0/q6_K weights, f32 accumulate, f16 activations",
        "data": "synthetic: seeded N(0,0.02) weights quantised to q4_0/q6_K, uniform prompt ids"
                + (f", seeded Zipf({zipf}) expert routing" if zipf else ""),
        "config": {"workload": f"{cfg.name}: {B} sequences in lockstep after a {args.prefill}-token prefill"
                               + (f", {nloc} per GPU, {cfg.experts // world} experts per GPU" if world > 1 else ""),
                   "model": cfg.name, "global_batch": B, "seq_len": ctx_mid,
                   "parallelism": f"ep{world}" if world > 1 else "single",
                   "exchange": ("peer memory (CUDA IPC)" if transport == "p2p" else "NCCL send/recv") if world > 1
                   else None,
                   "routing": f"zipf{zipf}" if zipf else "router top-8",
                   "l2": "weights (%.1f GB/step) >> 126 MB L2: no flush needed" % (sb["total"] / 1e9)},
        "e2e": {"value": round(B * args.steps / t_e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4 * B + 32 * world,
                "d2h_bytes_per_step": 4 * B},
        "roofline": {"bound": "hbm", "kernel": "whole step (all kernels), per GPU", "achieved": round(ach, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4), "peak_source": peak_kind,
                     "bytes_per_step": sb, "bytes_per_gpu_step": int(rank_bytes), "traffic": None},
        "exposed_all_to_all_us_per_step": round(a2a, 1) if world > 1 else None,
        "clocks": clk, "gpu_launches": int(kpt * args.steps), "kernels_per_step": kpt,
        "prefill_s": round(t_prefill, 1), "model_build_s": round(t_build, 1),
        "prefill": {"positions": args.prefill, "sequences": B,
                    "mode": "chunked batched (tcgen05 GEMMs)" if world == 1 else "token by token (expert parallel)",
                    "device_s": round(t_prefill_dev, 3), "tok_s": round(B * args.prefill / t_prefill_dev, 1)},
    }
    dist.close()
    return out, img, cfg


def wants_moe_point(args, world: int, config_given: bool, prefill_given: bool) -> bool:
    """The default one-GPU run (no --config / --prefill / --layers) also
    measures benchmark config 5's workload on this GPU and reports it inside
    its line, so the BENCH record carries the MoE bs64 single-GPU number too."""
    return (world == 1 and args.impl == "ours" and not config_given and not prefill_given and not args.layers
            and not args.no_moe_point and not under_torchrun())


def moe_point(args, budget_s: float) -> dict:
    """Benchmark config 5's workload (A4B, 64 sequences, 1024-token prefill,
    Zipf(1.1) routing) on this one GPU, run as a child process under a
    wall-clock budget: a failure or an overrun is recorded beside the headline
    instead of taking it down."""
    cap = importlib.import_module("e4b-webgpu_b200").config.get("a4b").max_ctx
    steps = max(1, min(args.steps, (cap - 1024 - args.warmup) // 2))
    cmd = [sys.executable, os.path.abspath(__file__), "--config", "a4b", "--batch", "64", "--prefill", "1024",
           "--zipf", "1.1", "--steps", str(steps), "--warmup", str(args.warmup), "--no-cpu"]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "TORCHELASTIC_RUN_ID",
                                                             "LOCAL_WORLD_SIZE")}
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=budget_s, env=env)
    except subprocess.TimeoutExpired:
        return {"error": f"not finished within its {budget_s:.0f} s budget"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        tail = (r.stderr or r.stdout).strip().splitlines()[-3:]
        return {"error": f"rc {r.returncode}: " + " | ".join(tail)}
    out = json.loads(lines[-1])
    keep = ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "config", "e2e", "clocks",
            "gpu_launches", "prefill_s", "model_build_s", "prefill")
    pt = {k: out[k] for k in keep if k in out}
    pt["roofline"] = {k: out["roofline"][k] for k in ("bound", "achieved", "peak", "unit", "frac")}
    pt["note"] = ("config 5 on one GPU (bench.py --config a4b --batch 64); the scaling series runs the same "
                  "workload under torchrun at every N, N = 1 included")
    return pt


def run_ours(args, rank, world, local_rank):
    e4b = importlib.import_module("e4b-webgpu_b200")
    import __graft_entry__
    __graft_entry__.build()
    dist = Dist(world, local_rank, "nccl" if world > 1 else None)
    cfg = bench_config(e4b, args)
    t0 = time.time()
    img = e4b.synth.build_model(cfg, seed=0)
    t_build = time.time() - t0
    eng = e4b.Engine(img, local_rank, fused=None if args.fused else False)
    dev = eng.dev
    prompt = e4b.synth.prompt_ids(args.prefill, cfg.vocab, seed=0)
    eng.prefill(prompt)
    dev.sync()
    pos = len(prompt)
    # warm-up (plan already recorded by the prefill)
    eng.decode_chunk(args.warmup)
    dev.sync()
    pos += args.warmup
    ctx_mid = pos + args.steps // 2
    # ---- device-resident timed region
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    dist.barrier()
    dev.sync()
    dev.call("e4b_event_record", 0)
    eng.decode_chunk(args.steps)
    dev.call("e4b_event_record", 1)
    dev.sync()
    import ctypes
    ms = ctypes.c_float()
    dev.call("e4b_event_elapsed", 0, 1, ctypes.byref(ms))
    t_dev = dist.max(ms.value / 1000.0)
    pos += args.steps
    clk = clocks.stop()
    # ---- end to end through the host API: per step one H2D parameter write from
    # pinned memory, the token plan, one D2H token read, host sync.
    tok = int(eng.read_ring(pos - 1, 1)[0])
    dist.barrier()
    dev.sync()
    dev.call("e4b_event_record", 2)
    for i in range(args.steps):
        eng.set_params(tok, pos)
        eng.run_token(1)
        dev.call("e4b_download_async", ctypes.c_void_p(eng._host_tok_ptr), eng.A.amax.ptr, ctypes.c_size_t(4))
        dev.sync()
        tok = int(eng.host_tok[0])
        pos += 1
    dev.call("e4b_event_record", 3)
    dev.sync()
    dev.call("e4b_event_elapsed", 2, 3, ctypes.byref(ms))
    t_e2e = dist.max(ms.value / 1000.0)
    peak, peak_kind = peaks()
    tb = token_bytes(cfg, ctx_mid)
    A = eng.A
    H, FF = cfg.hidden, cfg.ff
    if eng.fused:
        # ---- dominant kernel timed alone: the fused token kernel (every layer's
        # weights, 2.2 GB >> L2, streamed once per launch), repeated on the same
        # token; CUDA events on the engine's stream
        nrep = 10
        dev.call("e4b_event_record", 4)
        for _ in range(nrep):
            dev.call("e4b_dense_plan_run", eng.dense_plan)
        dev.call("e4b_event_record", 5)
        dev.sync()
        dev.call("e4b_event_elapsed", 4, 5, ctypes.byref(ms))
        dom_launch_s = ms.value / 1000.0 / nrep
        dom_bytes = tb["weights"] + tb["kv"] + tb["embed"]
        dom_name = "k_decode_dense (fused token: all layers' q4_0 weights + KV, one persistent kernel)"
        dom_profile = "decode_dense_e4b.md"
    else:
        # ---- dominant kernel timed alone: the dense gate|up GEMV (+GeGLU) of every
        # layer, each launch over different weights (cold L2), CUDA events on the stream
        nrep = 3
        dev.call("e4b_event_record", 4)
        for _ in range(nrep):
            for L in eng.layers:
                e4b.ops.q40gu(dev, None, None, None, None, A.normed, L.gu, A.geglu, IN=H, FF=0, FF2=FF, K=0)
        dev.call("e4b_event_record", 5)
        dev.sync()
        dev.call("e4b_event_elapsed", 4, 5, ctypes.byref(ms))
        dom_launch_s = ms.value / 1000.0 / (nrep * cfg.layers)
        dom_bytes = 2 * FF * H // 32 * 18 + H * 2 + FF * 2
        dom_name = "q40gu (dense gate|up + GeGLU, 2048 -> 2x16384)"
        dom_profile = "q40gu_e4b.md"
    kernels_per_token = eng.kernels_per_token
    eng_fused, plan_mode = eng.fused, eng.plan_mode
    status = dev.status()
    eng.close()
    if status:
        raise RuntimeError(f"device status word {status:#x} after the run")
    value = world * args.steps / t_dev
    e2e = world * args.steps / t_e2e
    out = None
    if rank == 0:
        ach = dom_bytes / dom_launch_s / 1e9
        traffic = traffic_from_profile(dom_profile)
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(1000 * t_dev / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q4_0/q6_K weights, f32 accumulate, f16 activations",
            "data": "synthetic: seeded N(0,0.02) weights quantised to q4_0/q6_K, uniform prompt ids (seed 0)",
            "config": {"workload": f"{cfg.name}: bs1 greedy decode after a {args.prefill}-token prefill",
                       "model": cfg.name, "layers": cfg.layers, "hidden": cfg.hidden, "ff": cfg.ff,
                       "vocab": cfg.vocab, "global_batch": world, "seq_len": ctx_mid,
                       "parallelism": f"replicas x{world}" if world > 1 else "single",
                       "l2": "weights (%.2f GB/token) >> 126 MB L2: no flush needed" % (tb["total"] / 1e9)},
            "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 32, "d2h_bytes_per_step": 4},
            "roofline": {"bound": "hbm", "kernel": dom_name,
                         "achieved": round(ach, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(ach / peak, 4), "peak_source": peak_kind,
                         "bytes_per_launch": dom_bytes, "launch_us": round(dom_launch_s * 1e6, 2),
                         "traffic": traffic},
            "token_roofline": {"bytes_per_token": tb["total"], "breakdown": tb,
                               "achieved_gbs": round(tb["total"] * value / world / 1e9, 1),
                               "frac": round(tb["total"] * value / world / 1e9 / peak, 4),
                               "roofline_tok_s": round(peak * 1e9 / tb["total"], 1)},
            "clocks": clk,
            "gpu_launches": int(kernels_per_token * args.steps),
            "kernels_per_token": kernels_per_token,
            "fused": eng_fused, "plan_mode": plan_mode,
            "model_build_s": round(t_build, 1),
        }
    dist.close()
    return out, img, cfg


def oracle_at_context(img, ctx0: int, seed: int = 7):
    """The oracle model with its KV caches holding `ctx0` positions of seeded
    N(0, 1) f16 keys / values (the attention work of a decode step at context
    ctx0, as after a ctx0-token prefill, without spending minutes on a CPU
    prefill)."""
    from oracle.model import OracleModel
    m = OracleModel(img)
    rng = np.random.default_rng(seed)
    for l in range(m.L):
        n = min(ctx0, m.kc[l].shape[0])
        m.kc[l][:n] = rng.standard_normal(m.kc[l][:n].shape, dtype=np.float32).astype(m.kc[l].dtype)
        m.vc[l][:n] = rng.standard_normal(m.vc[l][:n].shape, dtype=np.float32).astype(m.vc[l].dtype)
    m.kv_count = ctx0
    return m


def cpu_decode(img, ctx0: int, warmup: int, steps: int, budget_s: float):
    """Greedy decode steps of the oracle (the CPU restatement of the reference
    path) from context ctx0: `warmup` untimed, then up to `steps` timed ones,
    stopping early once budget_s of timed work is spent.  Returns (steps done,
    seconds, cores, last position)."""
    from oracle import ops as O
    m = oracle_at_context(img, ctx0)
    cores = int(O.qlib().oracle_threads())
    tok, pos = 1, ctx0
    for _ in range(warmup):
        tok, _ = m.step(tok, pos)
        pos += 1
    n, t0 = 0, time.time()
    while n < steps and (n == 0 or time.time() - t0 < budget_s):
        tok, _ = m.step(tok, pos)
        pos += 1
        n += 1
    return n, time.time() - t0, cores, pos


def cpu_baseline(img, cfg, ctx0: int, budget_s: float, max_steps: int):
    """The oracle on this host's cores, at the GPU arm's context (bounded sample)."""
    n, dt, cores, pos = cpu_decode(img, ctx0, 1, max_steps, budget_s)
    return {"value": round(n / dt, 4), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} greedy decode steps of {cfg.name} (one sequence) at context {ctx0}..{pos} "
                      f"(KV caches pre-filled with seeded values), after 1 untimed step; oracle C q4_0/q6_K "
                      f"matvecs on {cores} OpenMP threads + numpy"}


def run_reference(args, rank, world):
    """The reference arm: the reference path's CPU restatement (the oracle; the
    reference itself is JavaScript + WGSL on WebGPU and cannot run here), on
    rank 0 only, with every host thread.  One step = one greedy decode token of
    one sequence at the GPU arm's context; W untimed steps, then K timed ones
    (capped by a time budget so the arm ends within minutes).  Loads only the
    host libraries (synthetic weights, oracle), not the CUDA library."""
    if rank != 0:
        return None
    e4b = importlib.import_module("e4b-webgpu_b200")
    importlib.import_module("e4b-webgpu_b200.build").build_host()
    from oracle import build as ob
    ob.build()
    cfg = bench_config(e4b, args)
    img = e4b.synth.build_model(cfg, seed=0)
    n, dt, cores, pos = cpu_decode(img, args.prefill, args.warmup, args.steps, budget_s=args.cpu_budget * 6)
    v = round(n / dt, 4)
    sample = (f"{n} timed greedy decode steps of {cfg.name} (one sequence) at context "
              f"{args.prefill + args.warmup}..{pos} after {args.warmup} untimed ones; KV caches pre-filled with "
              f"seeded values for the {args.prefill}-token prompt; oracle C q4_0/q6_K matvecs on {cores} "
              f"OpenMP threads + numpy")
    if args.batch > 1 or cfg.moe:
        # the reference path decodes one token of one sequence at a time; a
        # batch of independent sequences runs at its per-token rate
        metric = moe_metric(args.batch, world)
        workload = f"{cfg.name}: {args.batch} sequences, CPU reference decoding them one token at a time"
    else:
        metric, workload = METRIC, f"{cfg.name}: bs1 greedy decode after a {args.prefill}-token prefill"
    base = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample}
    return {"metric": metric, "value": v, "unit": "tok/s", "n_gpus": world, "steps": n, "warmup": args.warmup,
            "ms_per_step": round(1000.0 * dt / n, 2) if n else None, "higher_is_better": True,
            "scaling": "strong" if args.batch > 1 else "weak",
            "vs_baseline": None, "dtype": "q4_0/q6_K weights, f32 accumulate, f16 activations",
            "data": "synthetic (same seeded model as the ours arm)", "impl": "reference",
            "config": {"workload": workload, "model": cfg.name, "seq_len": args.prefill + args.warmup + n // 2},
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


KERNELS = {
    # name: (description, rows, IN, kind)   -- weights > 126 MB L2 so every launch streams from HBM
    "q40gu": ("dense gate|up + GeGLU, E4B layer shape (2048 -> 2x16384), 4 layers of weights", 2 * 16384, 2048, "gu"),
    "q40down": ("down projection, E4B shape (16384 -> 2048), 8 layers of weights", 2048, 16384, "mv"),
    "q40qkv": ("qkv projection, E4B shape (2048 -> 3072), 48 layers of weights", 3072, 2048, "mv"),
    "q40big": ("gate|up + GeGLU, 2048 -> 2x65536 (4x the E4B layer), 2 copies", 2 * 65536, 2048, "gu"),
}


def graph_time(dev, enqueue, reps: int = 5) -> float:
    """Record enqueue() as a CUDA graph, replay it `reps` times (after one warm-up
    replay) and return the device time of one replay in microseconds, so host
    launch overhead is not part of the measurement."""
    import ctypes
    dev.call("e4b_plan_begin")
    try:
        enqueue()
    finally:
        pl = ctypes.c_int()
        dev.call("e4b_plan_end", ctypes.byref(pl))
    dev.call("e4b_plan_launch", pl.value, 1)
    dev.sync()
    ms = ctypes.c_float()
    dev.call("e4b_event_record", 0)
    dev.call("e4b_plan_launch", pl.value, reps)
    dev.call("e4b_event_record", 1)
    dev.sync()
    dev.call("e4b_event_elapsed", 0, 1, ctypes.byref(ms))
    dev.call("e4b_plan_destroy", pl.value)
    return ms.value * 1000.0 / reps


def run_rmschain(e4b, dev, args):
    """Launch-to-launch latency floor: a chain of dependent single-CTA RMSNorms."""
    import ctypes
    dev.call("e4b_set_pdl", int(args.pdl))
    H = 2048
    x = dev.upload(np.random.default_rng(0).standard_normal(H).astype(np.float32))
    w = dev.upload(np.ones(H, np.float32))
    y = dev.alloc(H * 4)
    def chain():
        for i in range(args.launches):
            e4b.ops.rmsnorm(dev, x if i % 2 == 0 else y, w, y if i % 2 == 0 else x, None, None, DIM=H)
    us = graph_time(dev, chain) / args.launches
    print(json.dumps({"kernel": "rmschain", "pdl": args.pdl, "launches": args.launches,
                      "us_per_launch": round(us, 3)}))
    dev.close()


PHASE_NAMES = ["ple_proj", "qkv", "attention", "o", "gate_up", "down", "ple_gate", "ple_layer_proj", "final"]


def run_trace(args):
    """Per-phase timing of the fused token kernel (e4b_dense_plan_trace): mean
    microseconds per phase kind of CTA 0's residual step, input build, GEMV
    (and the part of it spent waiting for weight copies), epilogue, the latest
    CTA's finish and the grid barrier, after a prefill of --prefill tokens."""
    import ctypes
    e4b = importlib.import_module("e4b-webgpu_b200")
    import __graft_entry__
    __graft_entry__.build()
    cfg = bench_config(e4b, args)
    eng = e4b.Engine(e4b.synth.build_model(cfg, seed=0), 0)
    if not eng.fused:
        raise SystemExit("--trace needs the fused token kernel")
    d = eng.dev
    eng.prefill(e4b.synth.prompt_ids(args.prefill, cfg.vocab, seed=0))
    d.sync()
    kinds = (ctypes.c_int * 8192)()
    nph = d.L.e4b_dense_plan_phases(d.ctx, eng.dense_plan, kinds, 8192)
    kinds = np.array(kinds[:nph])
    tb = d.alloc(nph * 64, "trace")
    d.call("e4b_dense_plan_trace", eng.dense_plan, tb.ptr)
    for _ in range(max(2, args.steps)):
        d.memset(tb, 0)
        d.call("e4b_dense_plan_run", eng.dense_plan)
        d.sync()
    t = d.read(tb, np.uint64, nph * 8).reshape(nph, 8).astype(np.int64)
    d.call("e4b_dense_plan_trace", eng.dense_plan, None)
    out = {"workload": cfg.name, "context": args.prefill, "phases": int(nph),
           "kernel_us": round((t[-1, 0] - t[0, 0]) / 1e3, 1), "kinds": {}}
    for k, name in enumerate(PHASE_NAMES[:-1]):
        sel = np.nonzero(kinds[:-1] == k)[0]
        if len(sel) == 0:
            continue
        m = lambda a, b: round(float(((t[sel, b] - t[sel, a]) / 1e3).mean()), 2)
        row = {"n": int(len(sel)), "residual": m(0, 1), "slowest_done": m(0, 5), "barrier": m(5, 6),
               "phase": m(0, 6)}
        if name != "attention":
            row.update({"input": m(1, 2), "gemv": m(2, 3), "weight_wait": round(float((t[sel, 7] / 1e3).mean()), 2),
                        "epilogue": m(3, 4)})
        else:   # CTA 0's first item: q/k/v prep, scores + softmax, p.V + partials
            row.update({"prep": m(1, 2), "scores_softmax": m(2, 3), "pv": m(3, 4)})
        out["kinds"][name] = row
    eng.close()
    print(json.dumps(out))


def run_attn(e4b, dev, args):
    """benchmark config 3 on the batched tensor-core attention (e4b_attdec_seq):
    GQA 8q / 2kv x 256, f16 K/V N(0,1), KV 4096 / 8192 / 32768, batch 1 and 16,
    global and sliding-window (512) masks.  Bytes = the K/V rows of the live
    chunks; K/V > L2 for the large cases, smaller ones rotate over copies."""
    import ctypes
    QH, KVH, HD = 8, 2, 256
    peak, kind_p = peaks()
    rows = []
    rng = np.random.default_rng(0)
    for kv in (4096, 8192, 32768):
        for nseq in (1, 16):
            cache = nseq * kv * KVH * HD * 2
            copies = max(1, int(math.ceil(256e6 / cache)))
            q = dev.upload(rng.standard_normal((nseq, QH, HD)).astype(np.float32))
            kvs = [(dev.upload(rng.standard_normal(cache // 2, dtype=np.float32).astype(np.float16)),
                    dev.upload(rng.standard_normal(cache // 2, dtype=np.float32).astype(np.float16)))
                   for _ in range(copies)]
            maxch = kv // 64
            po, pm = dev.alloc(nseq * QH * maxch * HD * 4), dev.alloc(nseq * QH * maxch * 8)
            out = dev.alloc(nseq * QH * HD * 2)
            for window in (0, 512):
                params = np.zeros(8, np.uint32)
                params[0], params[1], params[5] = kv - 1, kv, kv
                bp = dev.upload(params)
                mode = 0 if window else 2

                def loop(kvs=kvs, bp=bp, mode=mode, window=window):
                    for i in range(args.launches):
                        kb, vb = kvs[i % len(kvs)]
                        dev.call("e4b_attdec_seq", q, kb, vb, bp, po, pm, out, QH, KVH, HD, window, mode, 0, maxch,
                                 ctypes.c_float(1.0 / 16), kv, nseq, 0)
                us = graph_time(dev, loop) / args.launches
                live = min(kv, (kv - (kv - window) // 64 * 64) if window else kv)
                nbytes = nseq * live * KVH * HD * 2 * 2
                rows.append({"kv": kv, "batch": nseq, "mask": f"sliding{window}" if window else "global",
                             "us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1),
                             "frac": round(nbytes / us / 1e3 / peak, 4)})
    st = dev.status()
    dev.close()
    print(json.dumps({"kernel": "attn", "desc": "e4b_attdec_seq (split-KV + combine), config 3 shapes",
                      "peak": peak, "peak_source": kind_p, "launches": args.launches, "cases": rows, "status": st}))
    if st:
        raise SystemExit(f"device status {st:#x}")


def tensor_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def run_tcgemm(e4b, dev, args):
    """The prefill GEMM (e4b_q40gemm, tcgen05) on one A4B prefill chunk of
    `--tokens` rows (default 64 sequences x 64 positions): the dense q|k|v, o,
    gate|up + GeGLU and down projections, and the grouped expert gate|up +
    GeGLU and down over the chunk's tokens x top-8 entries sorted by expert
    (uniform routing).  FLOPs = 2 M N K of the useful product; the tensor pipe
    runs twice that (f16 hi + lo weight halves)."""
    import ctypes
    cfg = e4b.config.get("a4b")
    H, QD, FF, E, K, EF = cfg.hidden, cfg.q_dim, cfg.ff, cfg.experts, cfg.topk, cfg.expert_ff
    R = args.tokens
    rng = np.random.default_rng(0)
    ent = R * K
    counts = np.bincount(np.stack([rng.choice(E, K, replace=False) for _ in range(R)]).ravel(), minlength=E)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.uint32)
    boffs = dev.upload(offs)
    def q40(rows, n_in, name):
        return dev.upload(e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, 0, name, 0.02)), name)
    cases = [  # name, IN, OUT, M, groups, epi, weights (rows)
        ("qkv", H, cfg.qkv_rows(0), R, 1, 0), ("o", QD, H, R, 1, 0), ("dense_gu", H, FF, R, 1, 1),
        ("dense_down", FF, H, R, 1, 0), ("expert_gu", H, EF, ent, E, 1), ("expert_down", EF, H, ent, E, 0)]
    peak, kind_p = tensor_peak()
    rows_out = []
    for name, IN, OUT, M, groups, epi in cases:
        wrows = 2 * OUT if epi == 1 else OUT
        w = q40(groups * wrows, IN, name)
        x = dev.upload(rng.standard_normal((M, IN), dtype=np.float32).astype(np.float16))
        y = dev.alloc(M * OUT * (2 if epi else 4))
        def loop(w=w, x=x, y=y, IN=IN, OUT=OUT, M=M, groups=groups, epi=epi):
            for _ in range(args.launches):
                dev.call("e4b_q40gemm", x, w, None if epi else y, y if epi else None,
                         boffs if groups > 1 else None, IN, OUT, M, groups, epi)
        us = graph_time(dev, loop) / args.launches
        flops = 2.0 * M * wrows * IN
        tf = flops / us / 1e6
        rows_out.append({"gemm": name, "M": M, "N": wrows, "K": IN, "groups": groups, "us": round(us, 1),
                         "tflops": round(tf, 1), "frac": round(tf / peak, 4), "tensor_pipe_frac": round(2 * tf / peak, 4)})
        dev.free(w), dev.free(x), dev.free(y)
    tot_us = sum(r["us"] for r in rows_out)
    tot_f = sum(2.0 * r["M"] * r["N"] * r["K"] for r in rows_out)
    st = dev.status()
    dev.close()
    print(json.dumps({"kernel": "tcgemm", "desc": "e4b_q40gemm on one A4B prefill chunk", "tokens": R,
                      "peak_tflops": peak, "peak_source": kind_p, "cases": rows_out,
                      "layer_us": round(tot_us, 1), "layer_tflops": round(tot_f / tot_us / 1e6, 1), "status": st}))
    if st:
        raise SystemExit(f"device status {st:#x}")


def run_lmhead(e4b, dev, args):
    """The batched LM head at the A4B shape: 262144 x 2816 q6_K (605 MB, above L2,
    so every launch streams the weights from HBM) for n token rows, each n on
    the tile-packed copy (e4b_q6k_lmhead_tiles), and through
    e4b_q6k_lmhead_rows on the tcgen05 kernel and on the mma.sync one
    ("lmhead_tc_min" 1 / 65).  Weights are random q6_K bytes with a fixed
    superblock scale (timing only).  Algorithmic bytes = weights + x (f32) +
    logits (f32)."""
    cfg = e4b.config.get("a4b")
    V, H = cfg.vocab, cfg.hidden
    nsb = H // 256
    rng = np.random.default_rng(0)
    raw = rng.integers(0, 256, size=(V * nsb, 210), dtype=np.uint8)
    raw[:, 208:210] = np.frombuffer(np.float16(1e-3).tobytes(), np.uint8)
    w = dev.upload(raw.reshape(-1), "lm_w")
    del raw
    wt = dev.alloc(int(dev.L.e4b_q6k_packed_bytes(H, V)), "lm_wt")
    dev.call("e4b_q6k_pack_tiles", w, wt, H, V)
    dev.sync()           # the packing is not part of any timed launch
    hbm, kind_h = peaks()
    out = []
    for n in args.rows:
        x = dev.upload(rng.standard_normal((n, H), dtype=np.float32), "x")
        y = dev.alloc(n * V * 4, "y")
        scr = dev.alloc(2 * max(64, (n + 7) // 8 * 8) * H * 2, "scr")
        row = {"n": n}
        for label, tc in (("tiles", 0), ("tiles_mma", -2), ("tiles_tc", -1), ("tc", 1), ("mma_sync", 65)):
            if tc > 0:
                dev.call("e4b_set_option", b"lmhead_tc_min", tc)
            dev.call("e4b_set_option", b"lmhead_tiles_tc", -tc if tc < 0 else 0)
            def loop(x=x, y=y, scr=scr, n=n, tc=tc):
                for _ in range(args.launches):
                    if tc <= 0:
                        dev.call("e4b_q6k_lmhead_tiles", wt, x, scr, y, H, V, np.float32(cfg.softcap), n)
                    else:
                        dev.call("e4b_q6k_lmhead_rows", w, x, scr, y, H, V, np.float32(cfg.softcap), n)
            us = graph_time(dev, loop) / args.launches
            byts = V * nsb * 210 + n * H * 4 + n * V * 4
            row[label] = {"us": round(us, 1), "gbs": round(byts / us / 1e3, 1), "frac": round(byts / us / 1e3 / hbm, 4),
                          "useful_tflops": round(2.0 * n * V * H / us / 1e6, 1)}
        dev.call("e4b_set_option", b"lmhead_tc_min", 1)
        dev.call("e4b_set_option", b"lmhead_tiles_tc", 0)
        out.append(row)
        dev.free(x), dev.free(y), dev.free(scr)
    st = dev.status()
    dev.close()
    print(json.dumps({"kernel": "lmhead", "desc": "e4b_q6k_lmhead_rows, A4B LM head 262144 x 2816 q6_K",
                      "peak_gbs": hbm, "peak_source": kind_h, "rows": out, "status": st}))
    if st:
        raise SystemExit(f"device status {st:#x}")


def run_kernel(args):
    """Time one streaming kernel alone: `launches` launches cycling over enough
    distinct weight copies that the working set exceeds L2."""
    import ctypes
    e4b = importlib.import_module("e4b-webgpu_b200")
    import __graft_entry__
    __graft_entry__.build()
    dev = e4b.Device(0)
    if args.kernel == "rmschain":
        return run_rmschain(e4b, dev, args)
    if args.kernel == "attn":
        return run_attn(e4b, dev, args)
    if args.kernel == "tcgemm":
        return run_tcgemm(e4b, dev, args)
    if args.kernel == "lmhead":
        return run_lmhead(e4b, dev, args)
    desc, rows, n_in, kind = KERNELS[args.kernel]
    ws = int(dev.L.e4b_workspace_bytes())
    wsb = dev.alloc(ws, "workspace")
    dev.call("e4b_set_workspace", wsb.ptr, ctypes.c_size_t(ws))
    dev.call("e4b_set_pdl", int(args.pdl))
    dev.call("e4b_set_option", b"stream_ctas_per_sm", args.ctas_per_sm)
    dev.call("e4b_set_option", b"stream_stages", args.stages)
    dev.call("e4b_set_option", b"stream_variant", args.variant)
    per = rows * n_in // 32 * 18
    copies = max(2, int(math.ceil(160e6 / per)))
    w = e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, 0, "kernel", 0.02))
    bufs = [dev.upload(w, f"w{i}") for i in range(copies)]
    x = dev.upload(np.random.default_rng(0).standard_normal(n_in).astype(np.float16))
    y = dev.alloc(rows * 4)

    def one(i):
        b = bufs[i % copies]
        if kind == "gu":
            e4b.ops.q40gu(dev, None, None, None, None, x, b, y, IN=n_in, FF=0, FF2=rows // 2, K=0)
        else:
            e4b.ops.q40mv(dev, x, b, None, y, IN=n_in, OUT=rows, XF16=1)
    def loop():
        for i in range(args.launches):
            one(i)
    us = graph_time(dev, loop) / args.launches
    nbytes = per + n_in * 2 + (rows // 2 * 2 if kind == "gu" else rows * 4)
    peak, kind_p = peaks()
    st = dev.status()
    dev.close()
    print(json.dumps({"kernel": args.kernel, "desc": desc, "pdl": args.pdl, "ctas_per_sm": args.ctas_per_sm,
                      "stages": args.stages, "variant": args.variant, "launches": args.launches, "us_per_launch": round(us, 2),
                      "bytes_per_launch": nbytes, "gbs": round(nbytes / us / 1e3, 1),
                      "frac": round(nbytes / us / 1e3 / peak, 4), "peak": peak, "peak_source": kind_p,
                      "weight_copies": copies, "status": st}))
    if st:
        raise SystemExit(f"device status {st:#x}")


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default=None,
                    help="model config (default: e4b on 1 GPU -- benchmark config 2; a4b on N > 1 -- config 5)")
    ap.add_argument("--prefill", type=int, default=None, help="prompt tokens (default 512 for e4b, 1024 for a4b)")
    ap.add_argument("--layers", type=int, default=0, help="use only the first N layers (profiling cases)")
    ap.add_argument("--batch", type=int, default=None,
                    help="sequences decoded in lockstep (default 1 on 1 GPU, 64 -- expert parallel -- on N > 1)")
    ap.add_argument("--overlap-route", type=int, default=1,
                    help="one GPU: each layer's routing chain on a side stream beside the dense FFN (1) or in line (0)")
    ap.add_argument("--ep-overlap", type=int, default=1,
                    help="expert parallel: exchange the rows on a side stream beside the dense FFN (1) or in line (0)")
    ap.add_argument("--ep-transport", choices=["nccl", "p2p"], default="p2p",
                    help="expert parallel: slabs stored into the peers' memory (CUDA IPC; the default: exposed "
                         "exchange 0.50 / 0.75 ms per step at 2 / 4 GPUs against NCCL's 1.65), or NCCL send/recv")
    ap.add_argument("--zipf", type=float, default=1.1,
                    help="batched MoE: Zipf(s) expert routing of benchmark config 5 (0 = the router's top-8)")
    ap.add_argument("--fused", type=int, default=1, help="1: fused token kernel where the model allows it; "
                                                          "0: one kernel per operator")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU baseline sampling")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-moe-point", action="store_true",
                    help="default one-GPU run: skip the nested config-5 (A4B bs64) measurement")
    ap.add_argument("--moe-budget", type=float, default=600.0,
                    help="wall-clock budget (s) of the nested config-5 measurement")
    ap.add_argument("--kernel", choices=sorted(KERNELS) + ["rmschain", "attn", "tcgemm", "lmhead"],
                    help="time one kernel alone instead of the decode")
    ap.add_argument("--tokens", type=int, default=4096, help="--kernel tcgemm: token rows of the prefill chunk")
    ap.add_argument("--trace", action="store_true", help="per-phase timing of the fused token kernel")
    ap.add_argument("--launches", type=int, default=200)
    ap.add_argument("--rows", type=int, nargs="+", default=[1, 8, 16, 32, 64],
                    help="--kernel lmhead: token rows per launch")
    ap.add_argument("--pdl", type=int, default=1, help="programmatic dependent launch between kernels (1/0)")
    ap.add_argument("--ctas-per-sm", type=int, default=1)
    ap.add_argument("--stages", type=int, default=4)
    ap.add_argument("--variant", type=int, default=0, help="GEMV variant (warps x piece blocks): 0=8x32 1=16x16 2=16x8")
    args = ap.parse_args()
    rank, world, local_rank = dist_env()
    config_given, prefill_given = args.config is not None, args.prefill is not None
    # Plain `bench.py --gpus 1`: benchmark config 2 (E4B bs1).  Under torchrun,
    # at every N including 1: benchmark config 5 (A4B bs64, expert parallel), so
    # a scaling series compares one workload across N.
    scale_series = world > 1 or under_torchrun()
    if args.config is None:
        args.config = "a4b" if scale_series else "e4b"
    if args.batch is None:
        args.batch = 64 if (scale_series and args.config == "a4b") else 1
    if args.prefill is None:
        args.prefill = 1024 if args.config == "a4b" else 512
    if world > 1 and os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
        # NCCL's version banner goes to stdout; rank 0's stdout is the one JSON line
        os.environ["NCCL_DEBUG"] = "WARN"
    if world > 1:
        # torchrun starts every worker with OMP_NUM_THREADS=1; the host-side weight
        # synthesis (OpenMP, loaded lazily) gets its share of the cores back
        share = rank == 0 and args.batch > 1
        os.environ["OMP_NUM_THREADS"] = str(max(1, (os.cpu_count() or 1) // (1 if share else world)))
    if args.kernel:
        run_kernel(args)
        return
    if args.trace:
        run_trace(args)
        return
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        out = run_reference(args, rank, world)
    elif args.batch > 1 or importlib.import_module("e4b-webgpu_b200").config.get(args.config).moe:
        # MoE configs (any batch, including 1) run the batched engine
        out, img, cfg = run_moe_batch(args, rank, world, local_rank)
        if rank == 0:   # the CPU baseline is an N = 1 measurement
            out["cpu_baseline"] = None if (args.no_cpu or world > 1) else \
                cpu_baseline(img, cfg, args.prefill, args.cpu_budget, 8)
    else:
        out, img, cfg = run_ours(args, rank, world, local_rank)
        if rank == 0:
            out["cpu_baseline"] = None if (args.no_cpu or world > 1) else \
                cpu_baseline(img, cfg, args.prefill, args.cpu_budget, 64)
        if wants_moe_point(args, world, config_given, prefill_given):
            del img
            out["moe_bs64_1gpu"] = moe_point(args, args.moe_budget)
    if rank == 0 and out is not None:
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()

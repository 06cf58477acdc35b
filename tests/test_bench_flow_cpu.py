"""bench.py's flows end to end on the CPU, with the engines replaced by
stand-ins that answer the calls the timed regions make (events, copies, status):
the one-GPU line with its batch-64 expert-parallel point, the MoE line, and the
two-rank expert-parallel line (gloo plumbing, rank 0 prints) come out as JSON
with the contract's keys.  This exercises the host code of the GPU
paths; the numbers are the stand-ins' and mean nothing."""
import importlib
import json
import os
import sys
import types

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


class _Dev:
    def __init__(self):
        self.calls = []

    def call(self, name, *args):
        self.calls.append(name)
        if name == "e4b_event_elapsed":
            args[2]._obj.value = 4.0            # ms between the two events
        return 0

    def sync(self):
        pass

    def status(self):
        return 0

    def read(self, buf, dtype, n, offset=0):
        return np.zeros(n, dtype)


def _ptr():
    return types.SimpleNamespace(ptr=0)


class _Engine:
    """Engine: prefill / decode_chunk / set_params / run_token / read_ring."""
    def __init__(self, img, device=0, fused=None, **kw):
        self.dev = _Dev()
        self.fused, self.plan_mode, self.dense_plan = True, "graph", 0
        self.kernels_per_token = 5
        self.A = types.SimpleNamespace(amax=_ptr(), tok=_ptr())
        self._host_tok_ptr = 0
        self.host_tok = np.zeros(1, np.uint32)

    def prefill(self, prompt):
        pass

    def decode_chunk(self, n):
        pass

    def set_params(self, tok, pos):
        pass

    def run_token(self, n=1):
        pass

    def read_ring(self, start, n):
        return np.zeros(n, np.uint32)

    def close(self):
        pass


class _Batch(_Engine):
    made = []

    def __init__(self, img, nseq, device=0, **kw):
        super().__init__(img, device)
        self.kw = kw
        self.kernels_per_token = 400
        _Batch.made.append(kw)

    def step(self, toks, pos):
        pass

    def exchange_time(self, pos):
        return 0.0


@pytest.fixture
def bench(monkeypatch):
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    b = importlib.import_module("bench")
    e4b = importlib.import_module("e4b-webgpu_b200")
    monkeypatch.setattr(e4b, "Engine", _Engine)
    monkeypatch.setattr(e4b, "BatchEngine", _Batch)
    monkeypatch.setattr(e4b.synth, "build_model", lambda cfg, seed=0, **kw: np.zeros(16, np.uint8))
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK", "TORCHELASTIC_RUN_ID", "LOCAL_WORLD_SIZE"):
        monkeypatch.delenv(k, raising=False)
    _Batch.made.clear()
    return b


def _run(bench, monkeypatch, capsys, argv):
    monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
    bench.main()
    return json.loads(capsys.readouterr().out.strip().splitlines()[-1])


def _child_in_process(bench, monkeypatch, fail=None):
    """The nested config-5 point runs bench.py as a child process; here the
    child is bench.main() in this process (same stand-ins), or a failure."""
    import contextlib
    import io
    import subprocess

    def run(cmd, capture_output, text, timeout, env):
        if fail == "timeout":
            raise subprocess.TimeoutExpired(cmd, timeout)
        if fail == "rc":
            return subprocess.CompletedProcess(cmd, 1, "", "RuntimeError: device status word 0x2 after the run")
        argv = sys.argv
        out = io.StringIO()
        try:
            sys.argv = ["bench.py"] + cmd[2:]
            with contextlib.redirect_stdout(out):
                bench.main()
        finally:
            sys.argv = argv
        return subprocess.CompletedProcess(cmd, 0, out.getvalue(), "")
    monkeypatch.setattr(bench.subprocess, "run", run)


def test_default_line_with_the_expert_parallel_point(bench, monkeypatch, capsys):
    _child_in_process(bench, monkeypatch)
    line = _run(bench, monkeypatch, capsys, ["--steps", "4", "--warmup", "3", "--no-cpu"])
    for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
              "vs_baseline", "dtype", "data", "config", "e2e", "roofline", "clocks", "gpu_launches"):
        assert k in line, k
    assert line["metric"].startswith("decode tok/s bs1 E4B") and line["n_gpus"] == 1
    assert line["value"] == pytest.approx(4 / 0.004)
    assert {"bound", "achieved", "peak", "unit", "frac", "traffic"} <= set(line["roofline"])
    assert line["e2e"]["h2d_bytes_per_step"] == 32 and line["gpu_launches"] == 5 * 4
    pt = line["moe_bs64_1gpu"]
    assert "error" not in pt, pt
    assert pt["config"]["global_batch"] == 64 and pt["config"]["routing"] == "zipf1.1"
    assert pt["value"] == pytest.approx(64 * 4 / 0.004)
    assert _Batch.made[-1]["ep"] is None and _Batch.made[-1]["ep_transport"] == "nccl"


@pytest.mark.parametrize("fail", ["timeout", "rc"])
def test_failed_point_keeps_the_headline(bench, monkeypatch, capsys, fail):
    _child_in_process(bench, monkeypatch, fail)
    line = _run(bench, monkeypatch, capsys, ["--steps", "4", "--warmup", "3", "--no-cpu"])
    assert line["metric"].startswith("decode tok/s bs1 E4B") and line["value"] == pytest.approx(4 / 0.004)
    assert "error" in line["moe_bs64_1gpu"]


def test_torchrun_one_rank_runs_the_scaling_workload(bench, monkeypatch, capsys):
    """Under torchrun the N = 1 point of the scaling series is config 5 (A4B
    bs64, Zipf routing), the same workload as N > 1."""
    monkeypatch.setenv("TORCHELASTIC_RUN_ID", "x")
    line = _run(bench, monkeypatch, capsys, ["--gpus", "1", "--steps", "4", "--warmup", "3", "--no-cpu"])
    assert line["metric"].startswith("MoE decode tok/s bs64") and line["n_gpus"] == 1
    assert line["config"]["global_batch"] == 64 and line["config"]["routing"] == "zipf1.1"
    assert line["scaling"] == "strong" and "moe_bs64_1gpu" not in line


def test_profiling_cases_skip_the_point(bench, monkeypatch, capsys):
    line = _run(bench, monkeypatch, capsys, ["--prefill", "16", "--steps", "4", "--warmup", "3", "--no-cpu"])
    assert "moe_bs64_1gpu" not in line and not _Batch.made


def test_moe_line(bench, monkeypatch, capsys):
    line = _run(bench, monkeypatch, capsys, ["--config", "a4b", "--batch", "16", "--zipf", "0", "--steps", "4",
                                             "--warmup", "3", "--no-cpu"])
    assert line["metric"].startswith("MoE decode tok/s bs16") and line["config"]["routing"] == "router top-8"
    assert line["roofline"]["bytes_per_step"]["unique_experts_per_layer"] > 8
    assert line["e2e"]["h2d_bytes_per_step"] == 4 * 16 + 32 and line["gpu_launches"] == 400 * 4


def test_moe_line_refuses_more_positions_than_the_cache(bench, monkeypatch, capsys):
    monkeypatch.setattr(sys, "argv", ["bench.py", "--config", "a4b", "--batch", "16", "--steps", "2000",
                                      "--warmup", "3", "--no-cpu"])
    with pytest.raises(SystemExit):
        bench.main()


def _rank_main(rank, world, port, q):
    """One rank of `bench.py --gpus 2` (gloo plumbing, stand-in engines)."""
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import contextlib
    import io
    b = importlib.import_module("bench")
    e4b = importlib.import_module("e4b-webgpu_b200")
    e4b.Engine, e4b.BatchEngine = _Engine, _Batch
    e4b.synth.build_model = lambda cfg, seed=0, **kw: np.zeros(16, np.uint8)
    e4b.Device = lambda i: types.SimpleNamespace(close=lambda: None)
    e4b.batch.nccl_unique_id = lambda dev: bytes(128)
    sys.argv = ["bench.py", "--gpus", str(world), "--steps", "4", "--warmup", "3", "--prefill", "8",
                "--ep-transport", "p2p"]
    out = io.StringIO()
    with contextlib.redirect_stdout(out):
        b.main()
    q.put((rank, out.getvalue(), [m["ep"][:2] + (m["ep_transport"],) for m in _Batch.made]))


def test_two_rank_moe_line():
    import socket
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (o, m)) for r, o, m in (q.get(timeout=300) for _ in range(2)))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    line = json.loads(got[0][0].strip().splitlines()[-1])
    assert got[1][0].strip() == ""                      # only rank 0 prints
    assert line["n_gpus"] == 2 and line["config"]["parallelism"] == "ep2"
    assert line["config"]["exchange"] == "peer memory (CUDA IPC)"
    assert line["metric"].startswith("MoE decode tok/s bs64") and "exposed_all_to_all_us_per_step" in line
    assert got[0][1] == [(2, 0, "p2p")] and got[1][1] == [(2, 1, "p2p")]

"""The algorithmic byte counts behind bench.py's roofline fields (no GPU)."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    return importlib.import_module("bench")


def test_expected_unique_experts(bench):
    # uniform top-K without replacement: E (1 - (1 - K/E)^B)
    assert bench.expected_unique_experts(128, 8, 1, None) == pytest.approx(8.0)
    assert bench.expected_unique_experts(128, 8, 64, None) == pytest.approx(125.9, abs=0.1)
    # the Zipf(1.1) benchmark routing concentrates the load on fewer experts
    z = bench.expected_unique_experts(128, 8, 64, 1.1, trials=20)
    assert 60 < z < 125


def test_moe_step_bytes_a4b(bench):
    e4b = importlib.import_module("e4b-webgpu_b200")
    cfg = e4b.config.get("a4b")
    b = bench.moe_step_bytes(cfg, 64, 1043)
    # per layer: q|k|v, o, dense gate|up and down, router in f32; experts by unique count
    assert b["lm_head"] == 262144 * 2816 // 256 * 210
    assert b["embed"] == 64 * 2816 // 256 * 210
    assert 12.4e9 < b["expert_weights"] < 12.8e9
    assert 7.0e9 < b["kv"] < 8.0e9         # K and V per sliding layer, one shared cache per global layer
    assert b["total"] == b["weights"] + b["lm_head"] + b["embed"] + b["kv"]
    assert 21.0e9 < b["total"] < 22.5e9
    # batch 1 touches 8 experts per layer
    b1 = bench.moe_step_bytes(cfg, 1, 1043)
    assert b1["unique_experts_per_layer"] == pytest.approx(8.0)
    assert b1["total"] < 3.0e9


def test_moe_metric_names(bench):
    assert bench.moe_metric(64, 1).startswith("MoE decode tok/s bs64")
    assert "expert parallel" in bench.moe_metric(64, 8)


def test_moe_point_only_on_the_default_one_gpu_run(bench):
    import argparse
    a = argparse.Namespace(impl="ours", layers=0, no_moe_point=False)
    assert bench.wants_moe_point(a, 1, False, False)
    assert not bench.wants_moe_point(a, 2, False, False)          # N > 1 lines are the series itself
    assert not bench.wants_moe_point(a, 1, True, False)           # an explicit --config
    assert not bench.wants_moe_point(a, 1, False, True)           # profiling cases pass --prefill
    assert not bench.wants_moe_point(argparse.Namespace(impl="ours", layers=4, no_moe_point=False), 1, False, False)
    assert not bench.wants_moe_point(argparse.Namespace(impl="reference", layers=0, no_moe_point=False), 1, False, False)
    assert not bench.wants_moe_point(argparse.Namespace(impl="ours", layers=0, no_moe_point=True), 1, False, False)


def test_reference_arm_prints_its_line():
    """`bench.py --impl reference` (the CPU restatement timed on the host) on the
    small config: one JSON line with the contract's keys, no GPU needed."""
    import json
    import subprocess
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--config", "tiny",
                        "--steps", "2", "--warmup", "3"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["steps"] == 2 and line["warmup"] == 3            # the driver's --steps / --warmup


def test_reference_arm_does_not_load_the_cuda_library():
    """The reference arm runs the CPU restatement only: the process maps the
    host libraries (synthetic weights, oracle) but not libe4b_b200.so."""
    import subprocess
    code = ("import sys, runpy; sys.argv = ['bench.py', '--impl', 'reference', '--config', 'tiny', '--steps', '1', "
            "'--warmup', '3', '--prefill', '8']; runpy.run_path('bench.py', run_name='__main__'); "
            "maps = open('/proc/self/maps').read(); "
            "print('CUDA_LIB_MAPPED' if 'libe4b_b200.so' in maps else 'HOST_ONLY'); "
            "assert 'liboracle_q.so' in maps")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip().splitlines()[-1] == "HOST_ONLY"

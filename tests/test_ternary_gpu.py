"""Ternary experts on the GPU (e4b_t2gu, e4b_t2moedown; kernels/t2gu.wgsl,
kernels/t2moedown.wgsl) against the oracle's restatement on seeded planes, and
the per-operator MoE engine with ternary experts against the oracle model
with the same ternary tensors (greedy ids; final hidden state within 1e-2)."""
import importlib
import os
import sys

import numpy as np
import pytest

from oracle import ops as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

import pin_cases  # noqa: E402

pytestmark = pytest.mark.gpu


def planes(rng, rows, cols):
    t2 = importlib.import_module("e4b-webgpu_b200.ternary")
    t = rng.integers(-1, 2, size=(rows, cols)).astype(np.int8)
    sc = (np.abs(rng.standard_normal(rows)) * 0.02 + 1e-3).astype(np.float16)
    return t2.pack_t2(t), sc


@pytest.mark.parametrize("H,EF,E,K", [(2816, 704, 16, 8), (512, 192, 8, 4)])
def test_t2_kernels(e4b, dev, H, EF, E, K):
    rng = np.random.default_rng(H + EF)
    wgu, sgu = planes(rng, E * 2 * EF, H)
    wdn, sdn = planes(rng, E * H, EF)
    x = rng.standard_normal(H).astype(np.float16)
    topk = rng.choice(E, K, replace=False).astype(np.uint32)
    tw = rng.random(K).astype(np.float32)
    yh = dev.alloc(K * EF * 2)
    dev.call("e4b_t2gu", dev.upload(x).ptr, dev.upload(wgu).ptr, dev.upload(sgu).ptr, dev.upload(topk).ptr, yh.ptr,
             H, EF, K, E)
    dev.sync()
    got = dev.read(yh, np.float16, K * EF).reshape(K, EF).astype(np.float64)
    ref = O.t2gu(x.astype(np.float32), wgu.reshape(-1), sgu, topk, H, EF).astype(np.float64)
    assert np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -9 + 1e-6)
    xs = got.astype(np.float16)
    y = dev.alloc(H * 4)
    dev.call("e4b_t2moedown", dev.upload(xs).ptr, dev.upload(wdn).ptr, dev.upload(sdn).ptr, dev.upload(topk).ptr,
             dev.upload(tw).ptr, y.ptr, EF, H, K, E)
    dev.sync()
    gy = dev.read(y, np.float32, H).astype(np.float64)
    ry = O.t2moedown(xs.astype(np.float32), wdn.reshape(-1), sdn, topk, tw, EF, H).astype(np.float64)
    assert np.max(np.abs(gy - ry)) <= 2e-5 * np.max(np.abs(ry))
    assert dev.status() == 0


def test_ternary_engine_matches_oracle(e4b):
    from oracle.model import OracleModel
    t2 = importlib.import_module("e4b-webgpu_b200.ternary")
    cfg, img, prompt, n_new = pin_cases.build("a4b_heads")
    tern = t2.ternarize_model(img)
    eng = e4b.Engine(img, 0, ternary=tern)
    try:
        ids = eng.generate([int(t) for t in prompt], n_new)
        h = eng.read_hidden()
        assert eng.dev.status() == 0
    finally:
        eng.close()
    rids, margins, recs = OracleModel(img, ternary=tern).generate([int(t) for t in prompt], n_new, record=True)
    for i, (a, b) in enumerate(zip(ids, rids)):
        if a != b:
            assert margins[i] < 5e-3, (i, ids, rids, margins[i])
            break
    href = recs[-1]["hidden"][-1]
    assert np.linalg.norm(h - href) / np.linalg.norm(href) < 1e-2

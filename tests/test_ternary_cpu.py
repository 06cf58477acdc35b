"""Ternary expert format (scripts/ternarize_a4b.py semantics) on the CPU: the
2-bit shift-group packing round-trips through the oracle's unpacker, the
round-to-nearest ternarisation picks alpha = mean |w| per row and t =
clip(round(w / alpha), -1, 1), and ternarize_model converts a synthetic MoE
model's expert tensors row for row."""
import importlib

import numpy as np

from oracle import ops as O


def test_pack_roundtrip_and_layout():
    t2 = importlib.import_module("e4b-webgpu_b200.ternary")
    rng = np.random.default_rng(0)
    t = rng.integers(-1, 2, size=(5, 64)).astype(np.int8)
    w = t2.pack_t2(t)
    assert w.shape == (5, 4) and w.dtype == np.uint32
    assert np.array_equal(O.t2_unpack(w, 64), t)
    # element 4g + j of a word at bits 2g + 8j, value t + 1
    one = np.zeros((1, 16), np.int8)
    one[0, 4 * 2 + 3] = 1                          # g = 2, j = 3 -> value 2 at bits 4 + 24
    assert int(t2.pack_t2(one)[0, 0]) == (0x55555555 & ~(3 << 28)) | (2 << 28)


def test_ternarize_rows_rtn():
    t2 = importlib.import_module("e4b-webgpu_b200.ternary")
    w = np.array([[0.9, -1.1, 0.1, 0.0], [2.0, 2.0, -2.0, 0.5]], np.float32)
    a, t = t2.ternarize_rows(w)
    assert np.allclose(a, np.abs(w).mean(axis=1))
    assert t.tolist() == [[1, -1, 0, 0], [1, 1, -1, 0]]


def test_ternarize_model_rows():
    e4b = importlib.import_module("e4b-webgpu_b200")
    t2 = importlib.import_module("e4b-webgpu_b200.ternary")
    cfg = e4b.config.tiny_moe()
    img = e4b.synth.build_model(cfg, seed=0)
    tern = t2.ternarize_model(img, layers=[0])
    g = e4b.gguf.open_gguf(img)
    raw = np.asarray(g.fetch("blk.0.ffn_down_exps.weight"))
    w = O.deq_q40(raw).reshape(-1, cfg.expert_ff)
    planes, scales = tern[0]["down"]
    a, t = t2.ternarize_rows(w)
    assert np.array_equal(O.t2_unpack(planes, cfg.expert_ff), t)
    assert np.array_equal(scales, a.astype(np.float16))
    assert tern[0]["gu"][0].shape == (cfg.experts * 2 * cfg.expert_ff, cfg.hidden // 16)

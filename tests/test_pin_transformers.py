"""The oracle pinned to the reference's golden generator.

The reference makes its golden vectors with transformers in f32 on the CPU
(goldens/gen.py).  tests/golden/make_pin.py ran transformers' Gemma4ForCausalLM
on the synthetic models of tests/golden/pin_cases.py (weights decoded by the
python `gguf` package) and stored greedy ids, per-layer hidden states and the
top logits in tests/golden/pin_<case>.npz.

* With f32 storage (oracle.ops.STORE_F16 = False) the oracle computes the same
  graph transformers does: ids identical, every layer's hidden state and the
  top logits within 1e-4 relative.
* With the reference's f16 buffers (the default, and what the CUDA path is
  tested against) the ids are identical (a flip only at a top-2 margin below
  5e-3) and the first position's hidden states within 2e-3.
"""
import importlib
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

import pin_cases  # noqa: E402

TIE = 5e-3
CASES = sorted(pin_cases.CASES)


def fixture(name):
    return np.load(os.path.join(GOLDEN, f"pin_{name}.npz"))


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / np.linalg.norm(b))


def oracle_run(e4b, name, f16: bool):
    import oracle.ops as ops
    from oracle.model import OracleModel
    cfg, img, prompt, n_new = pin_cases.build(name)
    old = ops.STORE_F16
    ops.STORE_F16 = f16
    try:
        ids, margins, recs = OracleModel(img).generate([int(t) for t in prompt], n_new, record=True)
    finally:
        ops.STORE_F16 = old
    return cfg, img, prompt, ids, recs


def same_ids(got, ref, margins):
    """Identical greedy ids, or a first difference at a near-tie of the reference's logits."""
    for i, (x, y) in enumerate(zip(got, ref)):
        if x != y:
            assert margins[i] < TIE, (i, x, y, float(margins[i]))
            return False
    return True


@pytest.mark.parametrize("name", CASES)
def test_fixture_inputs_are_reproducible(e4b, name):
    import hashlib
    z = fixture(name)
    cfg, img, prompt, n_new = pin_cases.build(name)
    assert hashlib.sha256(np.asarray(img).tobytes()).digest() == z["sha256"].tobytes()
    assert np.array_equal(np.asarray(prompt, np.int64), z["prompt"]) and len(z["ids"]) == n_new


@pytest.mark.parametrize("name", CASES)
def test_oracle_f32_storage_equals_transformers(e4b, name):
    z = fixture(name)
    cfg, img, prompt, ids, recs = oracle_run(e4b, name, f16=False)
    assert list(ids) == z["ids"].tolist()
    for k, p in enumerate(z["pos"]):
        for l in range(cfg.layers):
            assert rel(recs[p]["hidden"][l], z["hidden"][k][l]) < 1e-4, (p, l)
    for p, r in enumerate(recs):
        top = z["top_logits"][p]
        assert np.max(np.abs(r["logits"][z["top_ids"][p]] - top)) < 1e-4 * np.max(np.abs(top)), p


@pytest.mark.parametrize("name", CASES)
def test_oracle_f16_storage_tracks_transformers(e4b, name):
    z = fixture(name)
    cfg, img, prompt, ids, recs = oracle_run(e4b, name, f16=True)
    same_ids(ids, z["ids"].tolist(), z["margins"])
    assert z["pos"][0] == 0
    for l in range(cfg.layers):
        assert rel(recs[0]["hidden"][l], z["hidden"][0][l]) < 2e-3, l


def test_a_planted_oracle_mistake_is_caught(e4b, monkeypatch):
    """The pin tells a wrong graph apart: dropping the per-expert router scale
    (a 15 % perturbation of the routing weights) moves the hidden states far
    beyond the f32 tolerance."""
    import oracle.ops as ops
    orig = ops.router_topk
    monkeypatch.setattr(ops, "router_topk", lambda x, wr, pes, k: orig(x, wr, np.ones_like(pes), k))
    z = fixture("tiny_moe")
    cfg, img, prompt, ids, recs = oracle_run(e4b, "tiny_moe", f16=False)
    worst = max(rel(recs[p]["hidden"][l], z["hidden"][k][l]) for k, p in enumerate(z["pos"])
                for l in range(cfg.layers))
    assert worst > 1e-2


def test_fixture_regenerates_with_transformers(e4b):
    """Rerun the generator for one case in this process (skipped where
    transformers is not importable) and compare with the committed fixture."""
    pytest.importorskip("transformers")
    pytest.importorskip("torch")
    make_pin = importlib.import_module("make_pin")
    out = make_pin.run_case("tiny_moe")
    z = fixture("tiny_moe")
    assert out["ids"].tolist() == z["ids"].tolist()
    assert np.max(np.abs(out["hidden"] - z["hidden"])) <= 1e-5 * np.max(np.abs(z["hidden"]))

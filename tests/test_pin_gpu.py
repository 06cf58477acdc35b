"""The CUDA decode path against the reference's golden generator: greedy ids of
the Engine (per-operator plan and fused token kernel) and of the BatchEngine on
the transformers parity models (tests/golden/pin_cases.py) equal the ids
transformers' Gemma4ForCausalLM produced for them (tests/golden/pin_<case>.npz),
a first difference allowed only at a top-2 logit margin below 5e-3 of the
transformers logits."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

import pin_cases  # noqa: E402

pytestmark = pytest.mark.gpu
TIE = 5e-3
CASES = sorted(pin_cases.CASES)


def fixture(name):
    return np.load(os.path.join(GOLDEN, f"pin_{name}.npz"))


def same_ids(got, ref, margins):
    for i, (x, y) in enumerate(zip(got, ref)):
        if x != y:
            assert margins[i] < TIE, (i, x, y, float(margins[i]))
            return
    assert len(got) == len(ref)


def engine_paths():
    out = []
    for name in CASES:
        cfg = pin_cases.config(name)
        out.append((name, False))
        if not cfg.moe:
            out.append((name, True))
    return out


@pytest.mark.parametrize("name,fused", engine_paths())
def test_engine_ids_equal_transformers(e4b, name, fused):
    z = fixture(name)
    cfg, img, prompt, n_new = pin_cases.build(name)
    eng = e4b.Engine(img, 0, fused=fused)
    try:
        ids = eng.generate([int(t) for t in prompt], n_new)
        assert eng.dev.status() == 0
    finally:
        eng.close()
    same_ids(ids, z["ids"].tolist(), z["margins"])


@pytest.mark.parametrize("name", [n for n in CASES if pin_cases.config(n).moe])
def test_batch_engine_ids_equal_transformers(e4b, name):
    """Three sequences of the same prompt in lockstep: every row decodes the
    transformers ids (and the rows agree with one another bit for bit)."""
    z = fixture(name)
    cfg, img, prompt, n_new = pin_cases.build(name)
    eng = e4b.BatchEngine(img, 3, 0)
    try:
        ids = eng.generate(np.stack([np.asarray(prompt)] * 3), n_new)
        assert eng.dev.status() == 0
    finally:
        eng.close()
    assert np.array_equal(ids[0], ids[1]) and np.array_equal(ids[0], ids[2])
    same_ids(ids[0].tolist(), z["ids"].tolist(), z["margins"])

"""End-to-end decode parity on the GPU: the Engine (GGUF load -> C-ABI kernels ->
recorded token plan) against the CPU oracle on the same synthetic GGUF.

Checks, per token: every layer's hidden state (relative error <= 1e-2, the
north-star bound; observed ~1e-6), the final logits, and the greedy ids over
the whole decode window.  A greedy id may only differ where the oracle's top-2
logit margin is below 1e-3 (a genuine near tie); none is expected.
"""
import numpy as np
import pytest

from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
HIDDEN_TOL = 1e-2


def _rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", ["tiny", "tiny_ple", "tiny_moe"])
def test_teacher_forced_layers(e4b, models, name):
    """Step both models through the same tokens; compare every layer, every step."""
    buf = models(name)
    eng = e4b.Engine(buf, 0, record=True)
    ref = OracleModel(buf)
    toks = e4b.synth.prompt_ids(40, eng.cfg.vocab, seed=3)     # > ring of the sliding layers (24)
    worst = 0.0
    try:
        for pos, t in enumerate(toks):
            eng.step(int(t), pos)
            eng.dev.sync()
            rid, rec = ref.step(int(t), pos, record=True)
            dump = eng.read_dump()
            for l in range(eng.cfg.layers):
                worst = max(worst, _rel(dump[l], rec["hidden"][l]))
            lg = eng.read_logits()
            assert _rel(lg, rec["logits"]) < HIDDEN_TOL
            top2 = np.sort(rec["logits"])[-2:]
            if eng.argmax_fast() != rid:
                assert top2[1] - top2[0] < 1e-3, (pos, eng.argmax_fast(), rid)
        assert eng.dev.status() == 0
    finally:
        eng.close()
    assert worst < HIDDEN_TOL, worst
    print(f"{name}: worst per-layer hidden rel err {worst:.2e}")


@pytest.mark.parametrize("name,P,N", [("tiny", 32, 32), ("tiny_ple", 20, 24), ("tiny_moe", 16, 24)])
def test_greedy_ids_match(e4b, models, name, P, N):
    """BASELINE config 1 shape for tiny: 32-token prompt (seed 0), 32 greedy tokens."""
    buf = models(name)
    prompt = e4b.synth.prompt_ids(P, e4b.config.get(name).vocab, seed=0)
    eng = e4b.Engine(buf, 0)
    try:
        ids = eng.generate(prompt, N)
        again = eng.generate(prompt, N)          # rerun on the same engine: caches need no reset
    finally:
        eng.close()
    rids, margins, _ = OracleModel(buf).generate(prompt, N, record=True)
    assert ids == again
    for i, (a, b) in enumerate(zip(ids, rids)):
        if a != b:
            assert margins[i] < 1e-3, (i, a, b, margins[i])
            break
    assert ids == rids or min(margins) < 1e-3

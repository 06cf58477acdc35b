"""Golden fixtures (tests/golden/golden.npz, made by tests/golden/make_golden.py).

CPU: the oracle decodes the q4_0 / q6_K golden blocks exactly as the python
`gguf` package did, the synthetic generator still produces the same model
images, and the oracle reproduces its recorded decodes (a regression pin).
GPU: the dequant kernels reproduce the package's values bit for bit, and both
decode paths reproduce the recorded greedy ids (a flip only at a top-2 margin
below TIE) and the final hidden state within the parity bound.
"""
import hashlib
import os

import numpy as np
import pytest

from oracle import ops as O
from oracle.model import OracleModel

G = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden.npz"))
TIE = 5e-3
MODELS = [("tiny", 32), ("tiny_ple", 24)]


def test_golden_blocks_oracle_matches_gguf_package():
    assert np.array_equal(O.deq_q40(G["q40_raw"]).view(np.uint32), G["q40_deq"].astype(np.float32).view(np.uint32))
    assert np.array_equal(O.deq_q6k(G["q6k_raw"]).view(np.uint32), G["q6k_deq"].astype(np.float32).view(np.uint32))


@pytest.mark.parametrize("name,N", MODELS)
def test_golden_models_and_oracle_decode(e4b, name, N):
    img = np.asarray(e4b.synth.build_model(e4b.config.get(name)))
    assert hashlib.sha256(img.tobytes()).digest() == G[f"{name}_sha256"].tobytes()
    ids, margins, recs = OracleModel(img).generate([int(t) for t in G[f"{name}_prompt"]], N, record=True)
    assert ids == [int(t) for t in G[f"{name}_ids"]]
    assert np.allclose(margins, G[f"{name}_margins"], rtol=0, atol=1e-6)
    P = len(G[f"{name}_prompt"])
    norms = np.array([np.linalg.norm(r["hidden"], axis=1) for r in recs[:P]])
    assert np.allclose(norms, G[f"{name}_hidden_norms"], rtol=1e-6, atol=0)


@pytest.mark.gpu
def test_golden_blocks_gpu_dequant(e4b, dev):
    for raw, ref, fn, per in ((G["q40_raw"], G["q40_deq"], "e4b_dequant_q40", 18),
                              (G["q6k_raw"], G["q6k_deq"], "e4b_dequant_q6k", 210)):
        nb = raw.size // per
        out = dev.alloc(ref.size * 4)
        dev.call(fn, dev.upload(raw).ptr, out.ptr, nb)
        got = dev.read(out, np.float32, ref.size)
        assert np.array_equal(got.view(np.uint32), ref.astype(np.float32).view(np.uint32))


@pytest.mark.gpu
@pytest.mark.parametrize("fused", [False, True])
@pytest.mark.parametrize("name,N", MODELS)
def test_golden_decode_gpu(e4b, name, N, fused):
    img = e4b.synth.build_model(e4b.config.get(name))
    eng = e4b.Engine(img, 0, record=True, fused=fused)
    try:
        ids = eng.generate([int(t) for t in G[f"{name}_prompt"]], N)
        h = eng.read_hidden()
    finally:
        eng.close()
    want, margins = [int(t) for t in G[f"{name}_ids"]], G[f"{name}_margins"]
    for i, (a, b) in enumerate(zip(ids, want)):
        if a != b:
            assert margins[i] < TIE, (i, a, b, margins[i])
            break
    ref = G[f"{name}_final_hidden"].astype(np.float64)
    if ids == want:
        assert np.linalg.norm(h - ref) / np.linalg.norm(ref) < 1e-2

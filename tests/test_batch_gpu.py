"""Batched MoE decode (BatchEngine: B sequences in lockstep, grouped experts,
tensor-core GEMMs) against the oracle run on each sequence separately."""
import numpy as np
import pytest

from oracle.model import OracleModel

pytestmark = pytest.mark.gpu
TIE = 5e-3


@pytest.mark.parametrize("B", [1, 3, 9])
def test_batched_moe_decode_matches_oracle(e4b, models, B):
    buf = models("tiny_moe")
    cfg = e4b.config.get("tiny_moe")
    P, N = 10, 8
    prompts = np.stack([e4b.synth.prompt_ids(P, cfg.vocab, seed=100 + b) for b in range(B)])
    eng = e4b.BatchEngine(buf, B, 0)
    try:
        ids = eng.generate(prompts, N)
        h = eng.read_hidden()
        assert eng.dev.status() == 0
    finally:
        eng.close()
    for b in range(B):
        ref = OracleModel(buf)
        rids, margins, recs = ref.generate([int(t) for t in prompts[b]], N, record=True)
        got = [int(t) for t in ids[b]]
        for i, (x, y) in enumerate(zip(got, rids)):
            if x != y:
                assert margins[i] < TIE, (b, i, x, y, margins[i])
                break
        if got == rids:
            href = recs[-1]["hidden"][-1]
            assert np.linalg.norm(h[b] - href) / np.linalg.norm(href) < 1e-2


@pytest.mark.parametrize("V,N,n", [(3000, 512, 11), (1000, 768, 64), (520, 256, 70), (4, 256, 1), (1000, 768, 1),
                                   (520, 256, 30)])
def test_batched_lmhead_rows(e4b, dev, V, N, n):
    """e4b_q6k_lmhead_rows (tensor cores, x as f16 hi + lo) against the oracle q6_K matvec per row;
    V % 8 == 0 takes the staged kernel, other V the direct one."""
    from oracle import ops as O
    w = e4b.synth.quant_q6_K(e4b.synth.normal_f32(V * N, 41 + V, "lmrows", 0.02))
    x = np.random.default_rng(42).standard_normal((n, N)).astype(np.float32)
    y = dev.alloc(n * V * 4)
    scr = dev.alloc(2 * ((n + 7) // 8 * 8) * N * 2)
    dev.call("e4b_q6k_lmhead_rows", dev.upload(w).ptr, dev.upload(x).ptr, scr.ptr, y.ptr, N, V,
             np.float32(30.0), n)
    dev.sync()
    got = dev.read(y, np.float32, n * V).reshape(n, V)
    for r in range(n):
        ref = O.softcap(O.q6k_matvec(w, x[r], V, N), 30.0)
        assert np.max(np.abs(got[r] - ref)) / np.max(np.abs(ref)) < 2e-5

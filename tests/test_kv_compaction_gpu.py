"""Long-context KV budget compaction (src/engine-a4b.js:589-657): the
attention-mass score pass (e4b_attn_score, kernels/attnos.wgsl:82-97), the
slot gather (e4b_kvgather, kernels/kvgather.wgsl), and Engine.generate_long
(probe step, compaction to the budget, decode with recompaction) against the
oracle's restatement (oracle/model.py generate_long) on pinned models."""
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


def test_kvgather_bit_exact(e4b, dev):
    rng = np.random.default_rng(5)
    slots, KVH, HD = 300, 4, 256
    k = rng.standard_normal((slots, KVH, HD)).astype(np.float16)
    v = rng.standard_normal((slots, KVH, HD)).astype(np.float16)
    keep = np.sort(rng.choice(slots, 77, replace=False)).astype(np.uint32)
    bk, bv = dev.upload(k), dev.upload(v)
    dk, dv = dev.alloc(k.nbytes), dev.alloc(v.nbytes)
    dev.call("e4b_kvgather", dev.upload(keep).ptr, len(keep), bk.ptr, bv.ptr, dk.ptr, dv.ptr, KVH, HD, slots)
    dev.sync()
    n = len(keep) * KVH * HD
    assert np.array_equal(dev.read(dk, np.uint16, n), k[keep].view(np.uint16).reshape(-1))
    assert np.array_equal(dev.read(dv, np.uint16, n), v[keep].view(np.uint16).reshape(-1))


def test_attn_score_op(e4b, dev):
    """One score pass on seeded q, K and the LSE of those logits: each head's
    probabilities added to the running scores, against float64."""
    rng = np.random.default_rng(9)
    QH, KVH, HD, slots, n = 16, 4, 256, 300, 211
    q = (rng.standard_normal((QH, HD)) * 0.1).astype(np.float32)
    k = rng.standard_normal((slots, KVH, HD)).astype(np.float16)
    s = np.einsum("hd,thd->ht", q.astype(np.float64), k[:n][:, np.arange(QH) // (QH // KVH)].astype(np.float64))
    lse = (s.max(1) + np.log(np.exp(s - s.max(1, keepdims=True)).sum(1))).astype(np.float32)
    prev = rng.random((QH, slots)).astype(np.float32)
    params = np.zeros(8, np.uint32)
    params[4], params[5] = n - 1, n
    sc = dev.upload(prev)
    dev.call("e4b_attn_score", dev.upload(q).ptr, dev.upload(k).ptr, dev.upload(lse).ptr, dev.upload(params).ptr,
             sc.ptr, QH, KVH, HD, np.float32(1.0), slots)
    dev.sync()
    got = dev.read(sc, np.float32, QH * slots).reshape(QH, slots)
    ref = prev.astype(np.float64)
    ref[:, :n] += np.exp(s - lse[:, None].astype(np.float64))
    assert np.max(np.abs(got - ref)) < 2e-5 * max(1.0, np.max(np.abs(ref)))
    assert dev.status() == 0


@pytest.mark.parametrize("name,tol", [("tiny", 1e-2), ("a4b_heads", 5e-2)])
def test_scores_match_oracle(e4b, name, tol):
    """Mass accumulated over a prefill's steps: the GPU's per-slot scores of
    every counted (global) cache equal the oracle's within the f16-storage
    noise of the two paths (of the largest mass: 1e-2 for the dense model; 5e-2
    for the small MoE model, where near-tied expert choices move single
    positions' hidden states by up to ~1e-1 in its deeper layers)."""
    from oracle.model import OracleModel
    cfg, img, prompt, _ = pin_cases.build(name)
    eng = e4b.Engine(img, 0, kv_budget=8, kv_decap=16, kv_protect=2)
    try:
        eng.prefill([int(t) for t in prompt])
        eng.dev.sync()
        got = {L.i: eng.dev.read(L.score, np.float32, cfg.q_heads * L.slots).reshape(cfg.q_heads, L.slots)
               for L in eng.layers if getattr(L, "score", None) is not None}
        assert eng.dev.status() == 0
    finally:
        eng.close()
    m = OracleModel(img)
    m.scoring = True
    for pos, t in enumerate(prompt):
        m.step(int(t), pos)
    assert set(got) == set(m.scores) and got
    P = len(prompt)
    for l, sc in got.items():
        ref = m.scores[l][:, :P]
        assert np.max(np.abs(sc[:, :P] - ref)) <= tol * np.max(ref), l
        assert np.all(sc[:, P:] == 0)
        # column sums: each step adds a probability distribution per head
        assert np.allclose(sc[:, :P].sum(axis=1), P, rtol=1e-4)


@pytest.mark.parametrize("name,P,n_new,budget,decap,protect", [
    ("tiny", 48, 30, 24, 40, 4),
    ("a4b_heads", 28, 20, 16, 24, 4),
])
def test_generate_long_matches_oracle(e4b, name, P, n_new, budget, decap, protect):
    """Prompt longer than the recompaction threshold: probe, compaction to the
    budget, then several recompactions while decoding; greedy ids equal the
    oracle's generate_long (the MoE case on its transformers-pinned prompt)."""
    from oracle.model import OracleModel
    cfg, img, pinned, _ = pin_cases.build(name)
    prompt = [int(t) for t in (pinned if len(pinned) == P else e4b.synth.prompt_ids(P, cfg.vocab, seed=77))]
    eng = e4b.Engine(img, 0, kv_budget=budget, kv_decap=decap, kv_protect=protect)
    try:
        ids = eng.generate_long(prompt, n_new)
        kv = eng.kv_count
        assert eng.dev.status() == 0
    finally:
        eng.close()
    ref = OracleModel(img).generate_long(prompt, n_new, budget, decap, protect)
    assert ids == ref
    assert kv <= decap

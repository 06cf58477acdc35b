"""CPU checks of the oracle and of the GGUF / block-format tooling.

Pins: the python `gguf` package (an independent implementation of the GGUF
container and of the Q4_0 / Q6_K block formats) decodes our blocks to the same
f32 values as the oracle, encodes Q4_0 to the same bytes as our generator, and
reads our files to the same tensors.
"""
import os
import tempfile

import gguf as gguf_pkg
import numpy as np
import pytest

from oracle import gguf_min, ops as O
from oracle.model import OracleModel


def test_q4_0_quantizer_matches_gguf_package(e4b):
    x = e4b.synth.normal_f32(1 << 16, 7, "qtest", 0.02)
    edge = np.zeros(32 * 6, np.float32)
    edge[0] = -1.0                      # extreme negative sets d
    edge[40] = 0.25                     # ties in magnitude: first index wins
    edge[41] = -0.25
    edge[64:96] = 3.0                   # constant block
    edge[100] = 1e-30                   # tiny scale
    edge[160:192] = np.linspace(-2, 2, 32)
    for v in (x, edge):
        ours = e4b.synth.quant_q4_0(v)
        ref = gguf_pkg.quants.quantize(v.reshape(-1, 32), gguf_pkg.GGMLQuantizationType.Q4_0).reshape(-1)
        assert np.array_equal(ours, ref)


def test_q4_0_dequant_bit_exact_vs_gguf_package(e4b):
    raw = e4b.synth.quant_q4_0(e4b.synth.normal_f32(1 << 14, 3, "dq", 0.02))
    ref = gguf_pkg.quants.dequantize(raw.reshape(-1, 18), gguf_pkg.GGMLQuantizationType.Q4_0).reshape(-1)
    assert np.array_equal(O.deq_q40(raw).view(np.uint32), ref.astype(np.float32).view(np.uint32))


def test_q6k_dequant_bit_exact_vs_gguf_package(e4b):
    x = e4b.synth.normal_f32(256 * 64, 5, "q6", 0.02)
    x[:256] = 0.0                       # all-zero block
    raw = e4b.synth.quant_q6_K(x)
    ref = gguf_pkg.quants.dequantize(raw.reshape(-1, 210), gguf_pkg.GGMLQuantizationType.Q6_K).reshape(-1)
    ours = O.deq_q6k(raw)
    assert np.array_equal(ours.view(np.uint32), ref.astype(np.float32).view(np.uint32))
    # the C row decoder (used for embedding rows) agrees too, with mult = 1
    rows = O.q6k_row(raw, 3, 256 * 4, 1.0)     # row 3 of a [.., 1024] matrix = blocks 12..15
    assert np.array_equal(rows, ours[12 * 256:16 * 256])
    # quantisation error is what a 6-bit code allows
    assert np.sqrt(np.mean((ours[256:] - x[256:]) ** 2)) < 0.03 * np.std(x)


def test_gguf_readers_agree(e4b):
    cfg = e4b.config.tiny_moe()
    path = tempfile.mktemp(suffix=".gguf")
    try:
        img = e4b.synth.build_model(cfg, path=path)
        ref = gguf_pkg.GGUFReader(path)
        ours = e4b.gguf.open_gguf(path)
        mem = e4b.gguf.open_gguf(np.asarray(img))
        orc = gguf_min.open_gguf(path)
        assert len(ref.tensors) == len(ours.tensors) == len(orc.tensors)
        for t in ref.tensors:
            a = np.asarray(t.data).reshape(-1).view(np.uint8)
            assert np.array_equal(a, ours.fetch(t.name))
            assert np.array_equal(a, mem.fetch(t.name))
            assert np.array_equal(a, orc.fetch(t.name))
            assert list(t.shape) == ours.tensors[t.name].dims
        assert ours.data_start % 32 == 0
        back = e4b.ModelConfig.from_kv(ours.kv).as_dict()
        want = cfg.as_dict()
        assert abs(back.pop("eps") - want.pop("eps")) < 1e-12     # stored as f32
        assert back == want
    finally:
        os.remove(path)


def test_synth_is_deterministic_and_stream_separated(e4b):
    a = e4b.synth.build_model(e4b.config.tiny())
    b = e4b.synth.build_model(e4b.config.tiny())
    assert np.array_equal(a, b)
    g = e4b.gguf.open_gguf(a)
    assert not np.array_equal(g.fetch("blk.0.attn_q.weight")[:1024], g.fetch("blk.1.attn_q.weight")[:1024])
    w = O.deq_q40(g.fetch("blk.0.ffn_up.weight"))
    assert abs(float(w.std()) - 0.02) < 0.002 and abs(float(w.mean())) < 1e-3


def test_oracle_q40_matvec_vs_dequant(e4b):
    rows, n_in = 37, 704                # 704 = 22 blocks: rows are not 16-byte aligned
    raw = e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, 1, "mv", 0.02))
    x = np.random.default_rng(0).standard_normal(n_in).astype(np.float32)
    y = O.q40mv(raw, x, rows, n_in)
    ref = O.deq_q40(raw).reshape(rows, n_in).astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)


def test_oracle_q6k_matvec_vs_dequant(e4b):
    rows, n_in = 9, 512
    raw = e4b.synth.quant_q6_K(e4b.synth.normal_f32(rows * n_in, 2, "mv6", 0.02))
    x = np.random.default_rng(1).standard_normal(n_in).astype(np.float32)
    y = O.q6k_matvec(raw, x, rows, n_in)
    ref = O.deq_q6k(raw).reshape(rows, n_in).astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)


def _split_attention(q, k, v, valid, chunk):
    """Chunked online softmax (the attsplit/attcomb decomposition) in numpy."""
    parts = []
    for c0 in range(0, len(k), chunk):
        idx = [t for t in valid if c0 <= t < c0 + chunk]
        if not idx:
            continue
        s = k[idx] @ q
        m = s.max()
        p = np.exp(s - m)
        parts.append((m, p.sum(), p @ v[idx]))
    M = max(m for m, _, _ in parts)
    den = sum(l * np.exp(m - M) for m, l, _ in parts)
    o = sum(oc * np.exp(m - M) for m, _, oc in parts) / den
    return o, M + np.log(den)


@pytest.mark.parametrize("L,chunk", [(1, 64), (100, 64), (4096, 64), (333, 128)])
def test_split_kv_merge_equals_dense(L, chunk):
    rng = np.random.default_rng(L)
    q = rng.standard_normal(64)
    k = rng.standard_normal((L, 64))
    v = rng.standard_normal((L, 64))
    k[rng.integers(L)] = 8 * q / np.linalg.norm(q)       # planted sharp peak
    valid = list(range(L))
    o, lse = _split_attention(q, k, v, valid, chunk)
    s = k @ q
    ref_lse = np.log(np.sum(np.exp(s - s.max()))) + s.max()
    ref = (np.exp(s - ref_lse)) @ v
    np.testing.assert_allclose(o, ref, rtol=1e-10, atol=1e-12)
    assert abs(lse - ref_lse) < 1e-10


@pytest.mark.parametrize("window,slack", [(16, 8), (512, 512), (5, 1), (7, 0)])
def test_ring_slot_rule_sound_and_complete(window, slack):
    """The sliding ring's invariants (specs/KVRing.tla SoundRec / Complete): for
    every query position, the attended slots hold exactly the positions of the
    window, once each."""
    ring = window + slack
    for qp in range(0, 3 * ring + 5):
        n = min(qp + 1, ring)
        ps = O.ring_positions(qp, ring)[:n]
        written = {t: p for t, p in enumerate(ps)}         # slot t holds position ps (p = t mod ring, <= qp)
        for t, p in written.items():
            assert p % ring == t and p <= qp and p > qp - ring
        attended = sorted(p for p in ps if p <= qp and p + window > qp)
        assert attended == list(range(max(0, qp - window + 1), qp + 1))


def test_router_ties_pick_lowest_index():
    wr = np.zeros((8, 4), np.float32)
    wr[[1, 3, 5], 0] = 1.0                               # three equal top scores
    idx, w = O.router_topk(np.array([1, 0, 0, 0], np.float32), wr, np.ones(8, np.float32), 4)
    assert list(idx[:3]) == [1, 3, 5] and idx[3] == 0
    assert abs(float(w.sum()) - 1.0) < 1e-6


def test_argmax_ties_lowest_index():
    x = np.array([0, 3, 1, 3, 3], np.float32)
    assert O.argmax_first(x) == 1


def test_oracle_decode_runs_all_graphs(models):
    for name in ("tiny", "tiny_ple", "tiny_moe"):
        m = OracleModel(models(name))
        ids, margins, recs = m.generate([1, 2, 3, 4], 3, record=True)
        assert len(ids) == 3 and all(0 <= t < 4096 for t in ids)
        assert np.isfinite(recs[-1]["hidden"]).all()


def test_fragment_order_permutation():
    """batch.xfo_perm is a permutation within every 32-element block and puts
    MMA lane t's B-fragment values -- the k indices its q4_0 A fragment uses
    (odd blocks 4t..4t+3, even blocks 2+4t..5+4t or {0, 1, 14, 15} for t = 3,
    and the same + 16) -- at halves 8t..8t+7 as [j0, j2, j1, j3, +16 ...]."""
    import importlib
    e4b = importlib.import_module("e4b-webgpu_b200")
    n = 128
    pos = e4b.batch.xfo_perm(n)
    assert sorted(pos.tolist()) == list(range(n))
    for b in range(n // 32):
        assert set(pos[32 * b:32 * b + 32].tolist()) == set(range(32 * b, 32 * b + 32))
        for t in range(4):
            if b & 1:
                j = [4 * t, 4 * t + 1, 4 * t + 2, 4 * t + 3]
            elif t < 3:
                j = [2 + 4 * t, 3 + 4 * t, 4 + 4 * t, 5 + 4 * t]
            else:
                j = [0, 1, 14, 15]
            order = [j[0], j[2], j[1], j[3], j[0] + 16, j[2] + 16, j[1] + 16, j[3] + 16]
            for slot, jj in enumerate(order):
                assert pos[32 * b + jj] == 32 * b + 8 * t + slot
    x = np.arange(n, dtype=np.float32)
    assert np.array_equal(e4b.batch.from_xfo(e4b.batch.to_xfo(x)), x)


def mvtest_x(n):
    """The reference's synthetic q40mv known-answer input (resident-a4b.html:421-456,
    "mvtest"): x[i] = ((13 i + 5) mod 17 - 8) / 8, exact in f16."""
    i = np.arange(n)
    return (((i * 13 + 5) % 17 - 8) / 8).astype(np.float32)


def mvtest_exact(raw, x, rows, n_in):
    """Row results by the KAT's own rule: per 32-weight block, d x sum((lo - 8) x_j +
    (hi - 8) x_{j+16}) over the 16 bytes, in float64."""
    b = raw.reshape(rows, n_in // 32, 18)
    d = b[:, :, :2].copy().view(np.float16).astype(np.float64)[..., 0]
    nib = b[:, :, 2:].astype(np.int64)
    xb = x.astype(np.float64).reshape(n_in // 32, 32)
    blk = (((nib & 15) - 8) * xb[None, :, :16]).sum(-1) + (((nib >> 4) - 8) * xb[None, :, 16:]).sum(-1)
    terms = d * blk
    return terms.sum(-1), np.abs(terms).sum(-1)


def test_oracle_q40mv_reference_kat(e4b):
    """The reference's mvtest at its shape (2112-wide down projection, x as
    above): the oracle's q4_0 matvec equals the exact per-block sum to f32
    accumulation error."""
    rows, n_in = 64, 2112
    raw = e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, 5, "mvtest", 0.02))
    x = mvtest_x(n_in)
    assert np.array_equal(x.astype(np.float16).astype(np.float32), x)
    exact, mag = mvtest_exact(raw, x, rows, n_in)
    got = O.q40mv(raw, x, rows, n_in)
    assert np.all(np.abs(got - exact) <= 1e-6 * mag)


def test_budget_keep_rule():
    """compactAll's choice (src/engine-a4b.js:589-603): the protected most recent
    slots always, the rest by accumulated mass summed over heads, ties to the
    lower slot, result ascending."""
    from oracle import ops as O
    sc = np.zeros((2, 12), np.float32)
    sc[0, :10] = [0.5, 0.1, 0.9, 0.1, 0.3, 0.9, 0.0, 0.2, 0.4, 0.1]
    sc[1, :10] = [0.0, 0.0, 0.0, 0.0, 0.6, 0.0, 0.0, 0.0, 0.0, 0.0]
    keep = O.budget_keep(sc, 10, 5, 2)          # slots 8, 9 protected; 3 of 0..7 by mass
    assert keep.tolist() == [2, 4, 5, 8, 9]     # masses 0.9 (2), 0.9 (4), 0.9 (5): ties keep the lower slots
    assert O.budget_keep(sc, 10, 12, 2).tolist() == list(range(10))

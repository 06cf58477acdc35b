"""Causal prefill attention (e4b_attn_prefill) for a chunk of npos positions of
nseq sequences whose K/V are already in the caches, against a float64 softmax
reference per query (its own position and slot rule) and against the decode
attention (e4b_attdec_seq) run once per position on the same caches: linear,
windowed and wrapping ring caches, GQA groups of 1, 4 and 8, shared K=V,
partial position blocks."""
import numpy as np
import pytest

from test_attdec_gpu import reference, valid_slots

pytestmark = pytest.mark.gpu
F32 = np.float32

CASES = [  # QH, KVH, HD, mode, pos0, npos, window, ring, cache_slots, keqv, nseq
    (16, 4, 256, 2, 100, 37, 0, 0, 192, False, 3),     # global linear cache, 16 positions per block
    (8, 1, 256, 2, 0, 20, 0, 0, 64, False, 2),         # GQA 8, prefill from position 0
    (16, 4, 256, 2, 60, 70, 0, 0, 192, True, 2),       # shared K=V (k_eq_v global layer)
    (8, 2, 256, 0, 300, 33, 96, 0, 384, False, 2),     # windowed linear cache
    (16, 4, 256, 1, 700, 33, 128, 160, 192, False, 2), # ring that has wrapped (33 = ring - window + 1)
    (16, 4, 256, 1, 10, 30, 128, 160, 192, False, 1),  # ring before it wraps
    (4, 4, 128, 2, 5, 64, 0, 0, 128, False, 2),        # GQA 1, HD 128
]


def params_for(pos, kv):
    p = np.zeros(8, np.uint32)
    p[0], p[1], p[4], p[5] = pos, pos + 1, kv, kv + 1
    return p


@pytest.mark.parametrize("case", CASES)
def test_attn_prefill(e4b, dev, case):
    QH, KVH, HD, mode, pos0, npos, window, ring, slots_n, keqv, nseq = case
    G = QH // KVH
    rng = np.random.default_rng(pos0 + npos + HD + mode)
    q = (rng.standard_normal((npos * nseq, QH, HD)) * 0.2).astype(F32)
    kc = rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    vc = kc if keqv else rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    bq, bk = dev.upload(q), dev.upload(kc)
    bv = bk if keqv else dev.upload(vc)
    bp = dev.upload(params_for(pos0, pos0))
    out = dev.alloc(npos * nseq * QH * HD * 2)
    dev.call("e4b_attn_prefill", bq.ptr, bk.ptr, bv.ptr, bp.ptr, out.ptr, QH, KVH, HD, window, mode, ring,
             np.float32(1.0), slots_n, nseq, npos)
    dev.sync()
    assert dev.status() == 0
    got = dev.read(out, np.float16, npos * nseq * QH * HD).reshape(npos, nseq, QH, HD).astype(np.float64)
    maxch = (slots_n + 63) // 64
    po, pm = dev.alloc(nseq * QH * maxch * HD * 4), dev.alloc(nseq * QH * maxch * 8)
    dec = dev.alloc(nseq * QH * HD * 2)
    for p in range(npos):
        qp = pos0 + p
        _, slots = valid_slots(mode, qp, qp + 1, window, ring)
        qrow = q[p * nseq:(p + 1) * nseq]
        ref = reference(qrow, kc, vc, slots, G)
        scale = max(1.0, np.max(np.abs(ref)))
        assert np.max(np.abs(got[p] - ref)) <= 2e-3 * scale, p
        # the decode kernel on the same caches at this position
        dev.call("e4b_attdec_seq", bq.ptr + p * nseq * QH * HD * 4, bk.ptr, bv.ptr, dev.upload(params_for(qp, qp)).ptr,
                 po.ptr, pm.ptr, dec.ptr, QH, KVH, HD, window, mode, ring, maxch, np.float32(1.0), slots_n, nseq, 0)
        dev.sync()
        d = dev.read(dec, np.float16, nseq * QH * HD).reshape(nseq, QH, HD).astype(np.float64)
        assert np.max(np.abs(got[p] - d)) <= 2e-3 * scale, p
    assert dev.status() == 0


def test_attn_prefill_rejects_ring_overwrite(e4b, dev):
    kc = dev.alloc(192 * 4 * 256 * 2)
    q = dev.alloc(64 * 16 * 256 * 4)
    out = dev.alloc(64 * 16 * 256 * 2)
    with pytest.raises(e4b.E4BError, match="overwrite"):
        dev.call("e4b_attn_prefill", q.ptr, kc.ptr, kc.ptr, dev.upload(params_for(0, 0)).ptr, out.ptr, 16, 4, 256,
                 128, 1, 160, np.float32(1.0), 192, 1, 34)

"""Batched tensor-core decode attention (e4b_attdec_seq) against a float64
softmax-attention reference over the valid slots (kernels/attsplit.wgsl +
attcomb.wgsl semantics), for linear, windowed and ring caches, GQA groups of
4 and 8, shared K=V caches, and against the reference-granularity
attsplit_seq + attcomb_seq pair."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
F32 = np.float32


def valid_slots(mode, qp, length, window, ring):
    """Slot rule of the f16 caches: which slots a query at qp attends."""
    if mode == 1:
        n = min(qp + 1, ring)
        out = []
        for t in range(n):
            ps = qp - ((qp + ring - t) % ring)
            if ps <= qp and ps + window > qp:
                out.append(t)
        return n, out
    n = length
    if mode == 0 and window > 0 and length > window:
        return n, list(range(length - window, length))
    return n, list(range(length))


def reference(q, kc, vc, slots, G):
    nseq, QH, HD = q.shape
    out = np.zeros((nseq, QH, HD))
    for b in range(nseq):
        for h in range(QH):
            kvh = h // G
            K = kc[b, slots, kvh].astype(np.float64)
            V = vc[b, slots, kvh].astype(np.float64)
            s = K @ q[b, h].astype(np.float64)
            p = np.exp(s - s.max())
            out[b, h] = p @ V / p.sum()
    return out


CASES = [  # QH, KVH, HD, mode, qp, length, window, ring, cache_slots, keqv
    (16, 4, 256, 2, 200, 201, 0, 0, 256, False),
    (16, 4, 256, 2, 63, 64, 0, 0, 128, True),
    (8, 2, 256, 0, 300, 301, 96, 0, 320, False),
    (8, 1, 128, 2, 1, 2, 0, 0, 64, False),
    (16, 4, 256, 1, 700, 0, 128, 160, 192, False),
    (16, 4, 256, 1, 90, 0, 128, 160, 192, False),
    (4, 4, 64, 2, 130, 131, 0, 0, 192, False),
]


@pytest.mark.parametrize("case", CASES)
@pytest.mark.parametrize("nseq", [1, 5])
def test_attdec_matches_reference(e4b, dev, case, nseq):
    QH, KVH, HD, mode, qp, length, window, ring, slots_n, keqv = case
    G = QH // KVH
    rng = np.random.default_rng(qp + 7 * nseq + HD)
    q = rng.standard_normal((nseq, QH, HD)).astype(F32) * 0.2
    kc = rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    vc = kc if keqv else rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    n, slots = valid_slots(mode, qp, length, window, ring)
    params = np.zeros(8, np.uint32)
    params[0], params[1], params[5] = qp, length, length
    maxch = (slots_n + 63) // 64
    bk = dev.upload(kc)
    bv = bk if keqv else dev.upload(vc)
    po, pm = dev.alloc(nseq * QH * maxch * HD * 4), dev.alloc(nseq * QH * maxch * 8)
    out = dev.alloc(nseq * QH * HD * 2)
    bq, bp = dev.upload(q), dev.upload(params)
    dev.call("e4b_attdec_seq", bq.ptr, bk.ptr, bv.ptr, bp.ptr, po.ptr, pm.ptr, out.ptr, QH, KVH, HD, window, mode,
             ring, maxch, np.float32(1.0), slots_n, nseq, 0)
    dev.sync()
    assert dev.status() == 0
    got = dev.read(out, np.float16, nseq * QH * HD).reshape(nseq, QH, HD).astype(np.float64)
    ref = reference(q, kc, vc, slots, G)
    assert np.max(np.abs(got - ref)) <= 2e-3 * max(1.0, np.max(np.abs(ref)))
    # the reference-granularity pair on the same inputs (64-slot chunks)
    out2 = dev.alloc(nseq * QH * HD * 2)
    dev.call("e4b_attsplit_seq", bq.ptr, bk.ptr, bv.ptr, bp.ptr, po.ptr, pm.ptr, QH, KVH, HD, window, mode, ring, 64,
             maxch, np.float32(1.0), slots_n, nseq)
    dev.call("e4b_attcomb_seq", po.ptr, pm.ptr, out2.ptr, None, None, QH, HD, maxch, nseq, 0)
    dev.sync()
    got2 = dev.read(out2, np.float16, nseq * QH * HD).reshape(nseq, QH, HD).astype(np.float64)
    assert np.max(np.abs(got - got2)) <= 2e-3 * max(1.0, np.max(np.abs(ref)))


def test_attdec_fragment_order(e4b, dev):
    QH, KVH, HD, nseq, slots_n = 16, 4, 256, 2, 128
    rng = np.random.default_rng(3)
    q = rng.standard_normal((nseq, QH, HD)).astype(F32) * 0.2
    kc = rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    vc = rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    params = np.zeros(8, np.uint32)
    params[0], params[1] = 99, 100
    maxch = 2
    res = {}
    for xfo in (0, 1):
        po, pm = dev.alloc(nseq * QH * maxch * HD * 4), dev.alloc(nseq * QH * maxch * 8)
        out = dev.alloc(nseq * QH * HD * 2)
        dev.call("e4b_attdec_seq", dev.upload(q).ptr, dev.upload(kc).ptr, dev.upload(vc).ptr, dev.upload(params).ptr,
                 po.ptr, pm.ptr, out.ptr, QH, KVH, HD, 0, 2, 0, maxch, np.float32(1.0), slots_n, nseq, xfo)
        dev.sync()
        res[xfo] = dev.read(out, np.uint16, nseq * QH * HD).reshape(nseq, QH * HD)
    assert np.array_equal(e4b.batch.to_xfo(res[0]), res[1])


@pytest.mark.parametrize("grid_cap", [1, 2, 3])
@pytest.mark.parametrize("keqv", [False, True])
def test_attdec_many_items_per_cta(e4b, dev, grid_cap, keqv):
    """The stage ring wraps many times: nseq 4 x 4 KV heads x 32 chunks = 512
    items on 1..3 CTAs (>= 170 items per CTA), so every stage is reused by
    both warp groups in turn."""
    QH, KVH, HD, nseq, slots_n = 16, 4, 256, 4, 2048
    G = QH // KVH
    rng = np.random.default_rng(11 + grid_cap)
    q = rng.standard_normal((nseq, QH, HD)).astype(F32) * 0.2
    kc = rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    vc = kc if keqv else rng.standard_normal((nseq, slots_n, KVH, HD)).astype(np.float16)
    params = np.zeros(8, np.uint32)
    params[0], params[1], params[5] = slots_n - 1, slots_n, slots_n
    maxch = slots_n // 64
    bk = dev.upload(kc)
    bv = bk if keqv else dev.upload(vc)
    po, pm = dev.alloc(nseq * QH * maxch * HD * 4), dev.alloc(nseq * QH * maxch * 8)
    out = dev.alloc(nseq * QH * HD * 2)
    dev.call("e4b_set_option", b"attn_grid_cap", grid_cap)
    try:
        dev.call("e4b_attdec_seq", dev.upload(q).ptr, bk.ptr, bv.ptr, dev.upload(params).ptr, po.ptr, pm.ptr, out.ptr,
                 QH, KVH, HD, 0, 2, 0, maxch, np.float32(1.0), slots_n, nseq, 0)
        dev.sync()
    finally:
        dev.call("e4b_set_option", b"attn_grid_cap", 0)
    assert dev.status() == 0
    got = dev.read(out, np.float16, nseq * QH * HD).reshape(nseq, QH, HD).astype(np.float64)
    ref = reference(q, kc, vc, list(range(slots_n)), G)
    assert np.max(np.abs(got - ref)) <= 2e-3 * max(1.0, np.max(np.abs(ref)))

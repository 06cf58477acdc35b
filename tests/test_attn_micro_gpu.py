"""benchmark config 3: split-KV decode attention microbenchmark shapes -- GQA 8
query / 2 KV heads, head_dim 256, f16 K/V/q drawn N(0,1), one planted key per
sequence with q.k scaled x8 (a sharp softmax peak), KV lengths 4096 / 8192 /
32768 at batch 1 and 16, sliding-window (512) and global masking.  The fp32
output and LSE of attsplit_seq + attcomb_seq (kernels/attsplit.wgsl +
attcomb.wgsl) and the f16 output of the tensor-core attdec_seq are compared
with a dense float64 softmax reference."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
QH, KVH, HD, W = 8, 2, 256, 512
SCALE = 1.0 / 16.0


def make(nseq, kv, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((nseq, QH, HD)).astype(np.float16)
    kc = rng.standard_normal((nseq, kv, KVH, HD)).astype(np.float16)
    vc = rng.standard_normal((nseq, kv, KVH, HD)).astype(np.float16)
    planted = rng.integers(0, kv, nseq)
    for b in range(nseq):
        # the planted key of KV head 0 is 8 x head 0's query: q.k = 8 |q|^2, a sharp peak
        kc[b, planted[b], 0] = (8 * q[b, 0].astype(np.float32)).astype(np.float16)
    return q, kc, vc, planted


def reference(q, kc, vc, lo):
    nseq = q.shape[0]
    out = np.zeros((nseq, QH, HD))
    lse = np.zeros((nseq, QH))
    for b in range(nseq):
        for h in range(QH):
            K = kc[b, lo:, h // (QH // KVH)].astype(np.float64)
            V = vc[b, lo:, h // (QH // KVH)].astype(np.float64)
            s = (K @ q[b, h].astype(np.float64)) * SCALE
            m = s.max()
            p = np.exp(s - m)
            out[b, h] = p @ V / p.sum()
            lse[b, h] = m + np.log(p.sum())
    return out, lse


@pytest.mark.parametrize("kv", [4096, 8192, 32768])
@pytest.mark.parametrize("nseq", [1, 16])
@pytest.mark.parametrize("window", [0, W])
def test_attention_microbench_shapes(e4b, dev, kv, nseq, window):
    q, kc, vc, planted = make(nseq, kv, kv + nseq + window)
    qf = q.astype(np.float32)
    params = np.zeros(8, np.uint32)
    params[0], params[1], params[5] = kv - 1, kv, kv
    mode = 0 if window else 2
    lo = kv - window if window else 0
    maxch = kv // 64
    bq, bk, bv, bp = dev.upload(qf), dev.upload(kc), dev.upload(vc), dev.upload(params)
    po, pm = dev.alloc(nseq * QH * maxch * HD * 4), dev.alloc(nseq * QH * maxch * 8)
    of, lse = dev.alloc(nseq * QH * HD * 4), dev.alloc(nseq * QH * 4)
    dev.call("e4b_attsplit_seq", bq.ptr, bk.ptr, bv.ptr, bp.ptr, po.ptr, pm.ptr, QH, KVH, HD, window, mode, 0, 64,
             maxch, np.float32(SCALE), kv, nseq)
    dev.call("e4b_attcomb_seq", po.ptr, pm.ptr, None, of.ptr, lse.ptr, QH, HD, maxch, nseq, 0)
    oh = dev.alloc(nseq * QH * HD * 2)
    dev.call("e4b_attdec_seq", bq.ptr, bk.ptr, bv.ptr, bp.ptr, po.ptr, pm.ptr, oh.ptr, QH, KVH, HD, window, mode, 0,
             maxch, np.float32(SCALE), kv, nseq, 0)
    dev.sync()
    assert dev.status() == 0
    ref, rlse = reference(qf, kc, vc, lo)
    got = dev.read(of, np.float32, nseq * QH * HD).reshape(nseq, QH, HD)
    glse = dev.read(lse, np.float32, nseq * QH).reshape(nseq, QH)
    assert np.max(np.abs(got - ref)) <= 1e-4 * max(1.0, np.abs(ref).max())
    assert np.max(np.abs(glse - rlse)) <= 1e-4 * max(1.0, np.abs(rlse).max())
    gh = dev.read(oh, np.float16, nseq * QH * HD).reshape(nseq, QH, HD).astype(np.float64)
    assert np.max(np.abs(gh - ref)) <= 2e-3 * max(1.0, np.abs(ref).max())
    # the planted key dominates where it is inside the window
    for b in range(nseq):
        if planted[b] >= lo:
            v = vc[b, planted[b], 0].astype(np.float64)
            assert np.corrcoef(ref[b, 0], v)[0, 1] > 0.99

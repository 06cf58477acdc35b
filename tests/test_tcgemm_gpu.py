"""The batched-prefill q4_0 GEMM on the tcgen05 tensor cores (e4b_q40gemm)
against a float64 product of the exactly dequantised weights (the oracle's
q4_0 decode, kernels/q40sg.wgsl with TPREC=f32): f32 outputs within 2e-5 of
the sum of |terms| (f32 summation order), the fused gate|up + GeGLU within one
f16 ulp of the GeGLU of that reference (plus the f32 bound through gelu);
dense and grouped (per-group weight matrices over row ranges, empty groups),
partial weight and token tiles, aligned and unaligned q4_0 rows (IN % 256)."""
import numpy as np
import pytest

from oracle import ops as O

pytestmark = pytest.mark.gpu
F32 = np.float32


def q40(e4b, rows, n_in, seed):
    return e4b.synth.quant_q4_0(e4b.synth.normal_f32(rows * n_in, seed, f"tc{rows}x{n_in}", 0.02))


def gelu64(g):
    t = np.clip(np.sqrt(2 / np.pi) * (g + 0.044715 * g ** 3), -20, 20)
    return 0.5 * g * (1 + np.tanh(t))


def run(e4b, dev, x, raw, IN, OUT, groups, offsets, epi):
    M = x.shape[0]
    bx, bw = dev.upload(x), dev.upload(raw)
    bo = dev.upload(np.asarray(offsets, np.uint32)) if offsets is not None else None
    if epi == 0:
        y = dev.alloc(M * OUT * 4)
        dev.call("e4b_q40gemm", bx.ptr, bw.ptr, y.ptr, None, bo.ptr if bo else None, IN, OUT, M, groups, 0)
        dev.sync()
        assert dev.status() == 0
        return dev.read(y, F32, M * OUT).reshape(M, OUT)
    yh = dev.alloc(M * OUT * 2)
    dev.call("e4b_q40gemm", bx.ptr, bw.ptr, None, yh.ptr, bo.ptr if bo else None, IN, OUT, M, groups, 1)
    dev.sync()
    assert dev.status() == 0
    return dev.read(yh, np.float16, M * OUT).reshape(M, OUT)


def reference(x, raw, IN, rows, groups, offsets):
    """float64 W x per row, and the bound sum |W||x| per output."""
    W = O.deq_q40(raw).astype(np.float64).reshape(groups, rows, IN)
    xs = x.astype(np.float64)
    M = x.shape[0]
    y = np.zeros((M, rows))
    bound = np.zeros((M, rows))
    offs = offsets if offsets is not None else [0, M]
    for g in range(groups):
        r0, r1 = offs[g], offs[g + 1]
        if r1 > r0:
            y[r0:r1] = xs[r0:r1] @ W[g].T
            bound[r0:r1] = np.abs(xs[r0:r1]) @ np.abs(W[g]).T
    return y, bound


CASES = [  # IN, OUT, M, group sizes (None: dense)
    (2816, 640, 300, None),          # aligned rows (IN % 256 == 0), partial weight and token tiles
    (704, 256, 257, None),           # unaligned rows (396 bytes), expert-down width
    (2112, 384, 512, None),          # unaligned rows (1188 bytes), A4B dense down width
    (2048, 128, 40, None),           # one partial token tile
    (2816, 256, None, [300, 0, 17, 513, 1]),   # grouped: empty groups, several token tiles
    (704, 384, None, [64, 200, 0, 0, 300]),
]


@pytest.mark.parametrize("case", CASES)
def test_q40gemm_matches_exact_reference(e4b, dev, case):
    IN, OUT, M, sizes = case
    groups = 1 if sizes is None else len(sizes)
    offsets = None if sizes is None else np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32)
    if sizes is not None:
        M = int(offsets[-1])
    rng = np.random.default_rng(IN + OUT + M)
    x = rng.standard_normal((M, IN)).astype(np.float16)
    raw = np.concatenate([q40(e4b, OUT, IN, 10 + g) for g in range(groups)])
    got = run(e4b, dev, x, raw, IN, OUT, groups, offsets, 0).astype(np.float64)
    ref, bound = reference(x, raw, IN, OUT, groups, None if offsets is None else offsets.tolist())
    err = np.abs(got - ref)
    assert np.all(err <= 2e-5 * bound + 1e-30), float(np.max(err / (bound + 1e-30)))


@pytest.mark.parametrize("case", [(2816, 200, 260, None), (2816, 192, None, [100, 0, 300, 5]), (2048, 64, 256, None)])
def test_q40gemm_geglu(e4b, dev, case):
    IN, FF, M, sizes = case
    groups = 1 if sizes is None else len(sizes)
    offsets = None if sizes is None else np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint32)
    if sizes is not None:
        M = int(offsets[-1])
    rng = np.random.default_rng(IN + FF + M + 1)
    x = rng.standard_normal((M, IN)).astype(np.float16)
    raw = np.concatenate([q40(e4b, 2 * FF, IN, 30 + g) for g in range(groups)])
    got = run(e4b, dev, x, raw, IN, FF, groups, offsets, 1).astype(np.float64)
    ref, bound = reference(x, raw, IN, 2 * FF, groups, None if offsets is None else offsets.tolist())
    g, u = ref[:, :FF], ref[:, FF:]
    r = gelu64(g) * u
    # f32 summation noise of g and u carried through gelu(g)*u, then one f16 rounding
    dg, du = 2e-5 * bound[:, :FF], 2e-5 * bound[:, FF:]
    slope = np.abs(gelu64(g + 1e-3) - gelu64(g - 1e-3)) / 2e-3 + 1.2
    tol = slope * dg * np.abs(u) + np.abs(gelu64(g)) * du + np.abs(r) * 2.0 ** -10 + 2.0 ** -24
    assert np.all(np.abs(got - r) <= 1.01 * tol)


def test_q40gemm_rejects_bad_shapes(e4b, dev):
    x = dev.alloc(64 * 96 * 2)
    w = dev.alloc(64 * 96 // 32 * 18)
    y = dev.alloc(64 * 64 * 4)
    with pytest.raises(e4b.E4BError, match="multiple of 64"):
        dev.call("e4b_q40gemm", x.ptr, w.ptr, y.ptr, None, None, 96, 64, 64, 1, 0)
    with pytest.raises(e4b.E4BError, match="offsets"):
        dev.call("e4b_q40gemm", x.ptr, w.ptr, y.ptr, None, None, 64, 64, 64, 2, 0)

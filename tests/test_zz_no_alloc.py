"""The allocation-free argmax (e4b_argmax_static) against the scratch-taking
e4b_argmax on the same inputs, two calls in a row each (the second call reuses
the library's fixed partials array)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _run(dev, name, x_buf, N, parts, part_buf=None):
    out = dev.alloc(8, "amax")
    if part_buf is None:
        dev.call(name, x_buf.ptr, out.ptr, N, parts)
    else:
        dev.call(name, x_buf.ptr, part_buf.ptr, out.ptr, N, parts)
    dev.sync()
    res = dev.read(out, np.uint32, 2)
    dev.free(out)
    return int(res[0]), int(res[1])


@pytest.mark.parametrize("N,parts", [(262144, 256), (4096, 7), (100003, 4096)])
def test_static_argmax_matches_scratch_argmax(e4b, dev, N, parts):
    rng = np.random.default_rng(N)
    xs = [rng.standard_normal(N).astype(np.float32) for _ in range(2)]
    xs[1][[5, N // 2, N - 1]] = np.float32(50.0)          # tie: lowest index wins
    part = dev.alloc(2 * parts * 4, "part")
    for x in xs:
        xb = dev.upload(x, "x")
        ref = _run(dev, "e4b_argmax", xb, N, parts, part)
        got1 = _run(dev, "e4b_argmax_static", xb, N, parts)
        got2 = _run(dev, "e4b_argmax_static", xb, N, parts)
        assert got1 == ref and got2 == ref
        assert ref[0] == int(np.argmax(x))
        dev.free(xb)
    dev.free(part)


def test_static_argmax_rejects_too_many_parts(e4b, dev):
    xb = dev.upload(np.zeros(64, np.float32), "x")
    out = dev.alloc(8, "amax")
    with pytest.raises(e4b.E4BError, match="parts"):
        dev.call("e4b_argmax_static", xb.ptr, out.ptr, 64, 4097)
    dev.free(out)
    dev.free(xb)

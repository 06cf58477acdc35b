"""CPU ORACLE -- TEST INFRASTRUCTURE ONLY.

Minimal GGUF v3 parser for the oracle, written independently of the product's
loader so the two can be checked against each other (and both against the python
`gguf` package's reader).  Layout per src/gguf.js:17-83 / the GGUF v3 spec.
"""
from __future__ import annotations

import os
import struct

import numpy as np

_BLK = {0: (4, 1), 1: (2, 1), 30: (2, 1), 2: (18, 32), 6: (22, 32), 8: (34, 32), 12: (144, 256), 14: (210, 256)}
_FMT = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class Gguf:
    def __init__(self, buf, kv, tensors, data_start):
        self.buf, self.kv, self.tensors, self.data_start = buf, kv, tensors, data_start

    def fetch(self, name):
        ttype, dims, off = self.tensors[name]
        bb, be = _BLK[ttype]
        n = int(np.prod(dims)) // be * bb
        return np.frombuffer(self.buf, dtype=np.uint8, count=n, offset=self.data_start + off)

    def f32(self, name):
        assert self.tensors[name][0] == 0, name
        return self.fetch(name).view(np.float32)


def _val(b, off, t):
    if t == 8:
        (n,) = struct.unpack_from("<Q", b, off)
        return bytes(b[off + 8:off + 8 + n]).decode(), off + 8 + n
    if t == 9:
        et, n = struct.unpack_from("<IQ", b, off)
        off += 12
        out = []
        for _ in range(n):
            v, off = _val(b, off, et)
            out.append(v)
        return out, off
    f = _FMT[t]
    return struct.unpack_from(f, b, off)[0], off + struct.calcsize(f)


def open_gguf(src):
    if isinstance(src, (str, os.PathLike)):
        src = np.memmap(src, dtype=np.uint8, mode="r")
    b = memoryview(src).cast("B")
    assert bytes(b[:4]) == b"GGUF"
    ver, nt, nkv = struct.unpack_from("<IQQ", b, 4)
    assert ver == 3
    off, kv, tensors = 24, {}, {}
    for _ in range(nkv):
        k, off = _val(b, off, 8)
        (t,) = struct.unpack_from("<I", b, off)
        kv[k], off = _val(b, off + 4, t)
    for _ in range(nt):
        name, off = _val(b, off, 8)
        (nd,) = struct.unpack_from("<I", b, off)
        dims = struct.unpack_from(f"<{nd}Q", b, off + 4)
        off += 4 + 8 * nd
        ttype, toff = struct.unpack_from("<IQ", b, off)
        off += 12
        tensors[name] = (ttype, dims, toff)
    align = int(kv.get("general.alignment", 32))
    return Gguf(b, kv, tensors, (off + align - 1) // align * align)

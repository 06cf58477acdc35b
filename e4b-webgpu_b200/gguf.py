"""GGUF v3 reader and writer.

The reader mirrors the reference's `openGGUF` (src/gguf.js:17-83): it parses the
header, the key/value table and the tensor table, applies `general.alignment`
(default 32) to find the data start, and hands out each tensor's raw bytes.  The
block type table is the reference's (src/gguf.js:3-9): Q4_0 = 18 bytes per 32
weights, Q6_K = 210 bytes per 256.  Tensor bytes are returned UNCHANGED: the
decode kernels consume the q4_0 / q6_K blocks exactly as they sit in the file,
so the loader does no repacking (unlike src/engine-a4b.js:29-73).

The writer produces the synthetic models the tests and the benchmark run on.
It writes to a path or to an in-memory buffer (a numpy uint8 array), which the
reader accepts as well, so a multi-GB synthetic model never has to touch disk.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, field

import numpy as np

GGML_F32 = 0
GGML_F16 = 1
GGML_Q4_0 = 2
GGML_Q5_0 = 6
GGML_Q8_0 = 8
GGML_Q4_K = 12
GGML_Q6_K = 14
GGML_BF16 = 30

# [block bytes, block elements]  (src/gguf.js:5-9)
TYPE_SIZES = {
    GGML_F32: (4, 1), GGML_F16: (2, 1), GGML_BF16: (2, 1),
    GGML_Q4_0: (18, 32), GGML_Q5_0: (22, 32), GGML_Q8_0: (34, 32),
    GGML_Q4_K: (144, 256), GGML_Q6_K: (210, 256),
}

# GGUF value types
_T_U8, _T_I8, _T_U16, _T_I16, _T_U32, _T_I32, _T_F32, _T_BOOL, _T_STR, _T_ARR, _T_U64, _T_I64, _T_F64 = range(13)
_SCALAR_FMT = {_T_U8: "<B", _T_I8: "<b", _T_U16: "<H", _T_I16: "<h", _T_U32: "<I", _T_I32: "<i",
               _T_F32: "<f", _T_BOOL: "<?", _T_U64: "<Q", _T_I64: "<q", _T_F64: "<d"}


class GGUFError(ValueError):
    pass


def tensor_bytes(ttype: int, dims) -> int:
    """Byte size of a tensor (src/gguf.js:11-15)."""
    if ttype not in TYPE_SIZES:
        raise GGUFError(f"unsupported ggml type {ttype}")
    bb, be = TYPE_SIZES[ttype]
    n = 1
    for d in dims:
        n *= int(d)
    if dims and int(dims[0]) % be:
        raise GGUFError(f"row length {dims[0]} is not a whole number of type-{ttype} blocks ({be})")
    return (n // be) * bb


@dataclass
class TensorInfo:
    name: str
    dims: list          # ggml order: dims[0] is the fastest-varying (row length)
    type: int
    offset: int         # relative to the data start

    @property
    def nbytes(self) -> int:
        return tensor_bytes(self.type, self.dims)


@dataclass
class GGUFFile:
    kv: dict
    tensors: dict
    data_start: int
    buf: memoryview = field(repr=False)
    version: int = 3

    def fetch(self, name: str) -> np.ndarray:
        """Raw bytes of one tensor as a uint8 view (no copy)."""
        t = self.tensors.get(name)
        if t is None:
            raise GGUFError("no tensor " + name)
        start = self.data_start + t.offset
        end = start + t.nbytes
        if end > len(self.buf):
            raise GGUFError(f"tensor {name} runs past the end of the file")
        return np.frombuffer(self.buf, dtype=np.uint8, count=t.nbytes, offset=start)

    def f32(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        if t.type != GGML_F32:
            raise GGUFError(f"{name} is type {t.type}, not F32")
        return self.fetch(name).view(np.float32)


def _read_value(b: memoryview, off: int, t: int):
    if t == _T_STR:
        (n,) = struct.unpack_from("<Q", b, off)
        off += 8
        s = bytes(b[off:off + n]).decode("utf-8")
        return s, off + n
    if t == _T_ARR:
        et, n = struct.unpack_from("<IQ", b, off)
        off += 12
        if et in _SCALAR_FMT and et != _T_STR:
            fmt = _SCALAR_FMT[et]
            sz = struct.calcsize(fmt)
            out = [struct.unpack_from(fmt, b, off + i * sz)[0] for i in range(n)]
            return out, off + n * sz
        out = []
        for _ in range(n):
            v, off = _read_value(b, off, et)
            out.append(v)
        return out, off
    fmt = _SCALAR_FMT.get(t)
    if fmt is None:
        raise GGUFError(f"bad gguf value type {t}")
    (v,) = struct.unpack_from(fmt, b, off)
    return v, off + struct.calcsize(fmt)


def open_gguf(src) -> GGUFFile:
    """Parse a GGUF v3 file from a path, bytes-like object or uint8 array."""
    if isinstance(src, (str, os.PathLike)):
        data = np.memmap(src, dtype=np.uint8, mode="r")
    else:
        data = src
    b = memoryview(data).cast("B")
    if bytes(b[0:4]) != b"GGUF":
        raise GGUFError("not GGUF")
    version, n_tensors, n_kv = struct.unpack_from("<IQQ", b, 4)
    if version != 3:
        raise GGUFError(f"unsupported GGUF version {version}")
    off = 24
    kv = {}
    for _ in range(n_kv):
        k, off = _read_value(b, off, _T_STR)
        (t,) = struct.unpack_from("<I", b, off)
        off += 4
        v, off = _read_value(b, off, t)
        if not k.startswith("tokenizer."):     # src/gguf.js:58 drops these too
            kv[k] = v
    align = int(kv.get("general.alignment", 32))
    tensors = {}
    for _ in range(n_tensors):
        name, off = _read_value(b, off, _T_STR)
        (nd,) = struct.unpack_from("<I", b, off)
        off += 4
        dims = list(struct.unpack_from(f"<{nd}Q", b, off))
        off += 8 * nd
        ttype, toff = struct.unpack_from("<IQ", b, off)
        off += 12
        tensors[name] = TensorInfo(name, dims, ttype, toff)
    data_start = (off + align - 1) // align * align
    return GGUFFile(kv=kv, tensors=tensors, data_start=data_start, buf=b, version=version)


# ---------------------------------------------------------------- writer

def _enc_str(s: str) -> bytes:
    e = s.encode("utf-8")
    return struct.pack("<Q", len(e)) + e


def _enc_kv(key: str, val) -> bytes:
    out = _enc_str(key)
    if isinstance(val, bool):
        return out + struct.pack("<I?", _T_BOOL, val)
    if isinstance(val, int):
        return out + struct.pack("<II", _T_U32, val) if 0 <= val < 2**32 else out + struct.pack("<Iq", _T_I64, val)
    if isinstance(val, float):
        return out + struct.pack("<If", _T_F32, val)
    if isinstance(val, str):
        return out + struct.pack("<I", _T_STR) + _enc_str(val)
    if isinstance(val, (list, tuple)):
        if all(isinstance(v, bool) for v in val):
            return out + struct.pack("<IIQ", _T_ARR, _T_BOOL, len(val)) + b"".join(struct.pack("<?", v) for v in val)
        if all(isinstance(v, int) for v in val):
            return out + struct.pack("<IIQ", _T_ARR, _T_I32, len(val)) + b"".join(struct.pack("<i", v) for v in val)
        if all(isinstance(v, float) for v in val):
            return out + struct.pack("<IIQ", _T_ARR, _T_F32, len(val)) + b"".join(struct.pack("<f", v) for v in val)
    raise GGUFError(f"cannot encode kv {key}={val!r}")


class GGUFWriter:
    """Collects kv pairs and tensors, then lays out a GGUF v3 image.

    Tensors are registered with their ggml dims and type; their bytes are
    produced by a callback into the final buffer, so multi-GB models are
    generated in place without intermediate copies.
    """

    def __init__(self, alignment: int = 32):
        self.alignment = alignment
        self.kv = {"general.alignment": alignment}
        self.tensors = []       # (name, dims, type, fill)

    def add_kv(self, key: str, val):
        self.kv[key] = val

    def add_tensor(self, name: str, dims, ttype: int, fill):
        """fill(out_uint8_view) writes exactly tensor_bytes(ttype, dims) bytes."""
        self.tensors.append((name, [int(d) for d in dims], ttype, fill))

    def build(self, path: str | None = None) -> np.ndarray:
        head = bytearray(b"GGUF")
        head += struct.pack("<IQQ", 3, len(self.tensors), len(self.kv))
        for k, v in self.kv.items():
            head += _enc_kv(k, v)
        offsets = []
        cur = 0
        for name, dims, ttype, _ in self.tensors:
            cur = (cur + self.alignment - 1) // self.alignment * self.alignment
            offsets.append(cur)
            head += _enc_str(name) + struct.pack("<I", len(dims))
            head += struct.pack(f"<{len(dims)}Q", *dims) + struct.pack("<IQ", ttype, cur)
            cur += tensor_bytes(ttype, dims)
        data_start = (len(head) + self.alignment - 1) // self.alignment * self.alignment
        total = data_start + cur
        if path is None:
            out = np.zeros(total, dtype=np.uint8)
        else:
            out = np.memmap(path, dtype=np.uint8, mode="w+", shape=(total,))
        out[:len(head)] = np.frombuffer(bytes(head), dtype=np.uint8)
        for (name, dims, ttype, fill), o in zip(self.tensors, offsets):
            n = tensor_bytes(ttype, dims)
            fill(out[data_start + o: data_start + o + n])
        if path is not None:
            out.flush()
        return out

"""ctypes binding of libe4b_b200.so, generated from include/e4b_b200.h.

Every `E4B_API` prototype in the header becomes a typed ctypes function, so the
Python host and the C ABI cannot drift apart.  The library is required: if it
is missing or the CUDA runtime cannot open a device, calls fail loudly -- there
is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
HEADER = os.path.join(os.path.dirname(_HERE), "include", "e4b_b200.h")
LIBPATH = os.path.join(_HERE, "libe4b_b200.so")

_CTYPE = {
    "int": ctypes.c_int, "float": ctypes.c_float, "int64_t": ctypes.c_int64, "size_t": ctypes.c_size_t,
    "uint32_t": ctypes.c_uint32, "double": ctypes.c_double, "unsigned long long": ctypes.c_ulonglong,
}

_PROTO = re.compile(r"E4B_API\s+([\w\s\*]+?)\s*\b(e4b_\w+)\s*\(([^)]*)\)\s*;", re.S)


def _arg_type(decl: str):
    decl = " ".join(decl.replace("const ", "").split())
    if "**" in decl:
        return ctypes.POINTER(ctypes.c_void_p)
    if decl.startswith("char*") or decl.startswith("char *"):
        return ctypes.c_char_p
    if "*" in decl:
        return ctypes.c_void_p
    base = decl.rsplit(" ", 1)[0] if " " in decl else decl
    if base not in _CTYPE:
        raise TypeError(f"unmapped C type in header: {decl!r}")
    return _CTYPE[base]


def parse_header(path: str = HEADER) -> dict:
    """name -> (restype, [argtypes]) for every E4B_API prototype."""
    src = open(path).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    out = {}
    for ret, name, args in _PROTO.findall(src):
        ret = " ".join(ret.replace("const ", "").split())
        restype = ctypes.c_char_p if ret == "char*" or ret == "char *" else _CTYPE.get(ret, ctypes.c_int)
        argl = [a.strip() for a in args.split(",") if a.strip() and a.strip() != "void"]
        out[name] = (restype, [_arg_type(a) for a in argl])
    return out


class E4BError(RuntimeError):
    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed ({code}): {msg}")
        self.code = code


_LIB = None
PROTOS = None


def _nccl_path():
    """The NCCL build the expert-parallel exchange opens: E4B_NCCL_LIB, else the
    nvidia-nccl wheel's (the one a CUDA-enabled framework in this process would
    load, so both share one copy), else the loader's libnccl.so.2."""
    if os.environ.get("E4B_NCCL_LIB"):
        return os.environ["E4B_NCCL_LIB"]
    import importlib.util
    spec = importlib.util.find_spec("nvidia")
    for base in (spec.submodule_search_locations or []) if spec else []:
        cand = os.path.join(base, "nccl", "lib", "libnccl.so.2")
        if os.path.exists(cand):
            return cand
    return ""


def lib():
    """Load libe4b_b200.so and type every function the header declares."""
    global _LIB, PROTOS
    if _LIB is None:
        path = _nccl_path()
        if path:
            os.environ.setdefault("E4B_NCCL_LIB", path)
        if not os.path.exists(LIBPATH):
            raise RuntimeError(f"{LIBPATH} is missing: build it with __graft_entry__.build() "
                               "(the decode path has no CPU fallback)")
        L = ctypes.CDLL(LIBPATH)
        PROTOS = parse_header()
        for name, (res, args) in PROTOS.items():
            fn = getattr(L, name)          # AttributeError here = header/library mismatch
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB

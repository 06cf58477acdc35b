"""CPU checks of the C ABI: the library loads, exports every symbol the header
declares, and rejects bad arguments without touching a GPU."""
import ctypes
import re
import subprocess

import pytest


def _header_names(e4b):
    return sorted(e4b._lib.parse_header().keys())


def test_header_declares_operator_set(e4b):
    names = set(_header_names(e4b))
    ops = {"q40mv", "q40gu", "q40moedown", "moecomb", "q6k_embed", "q6k_lmhead", "rmsnorm", "rmsacc", "rmsacc3",
           "a4btail", "routertop", "router", "top8", "headprep", "rope", "kvwrite", "attsplit", "attcomb",
           "geglumul", "geglusl", "geglub", "pleprep", "plegatemv", "plemul", "argmax", "feedtok"}
    assert {"e4b_" + o for o in ops} <= names
    assert {"e4b_plan_begin", "e4b_plan_end", "e4b_plan_launch", "e4b_alloc", "e4b_upload"} <= names


def test_library_exports_every_header_symbol(e4b):
    lib = e4b.lib()
    out = subprocess.run(["nm", "-D", "--defined-only", e4b._lib.LIBPATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (e4b_\w+)", out))
    missing = [n for n in _header_names(e4b) if n not in exported]
    assert not missing, missing
    for n in _header_names(e4b):
        assert getattr(lib, n) is not None
    # nothing exported that the header does not declare
    assert exported <= set(_header_names(e4b))


def test_null_context_is_rejected(e4b):
    lib = e4b.lib()
    assert lib.e4b_sync(None) == -1
    assert lib.e4b_q40mv(None, None, None, None, None, 32, 1, 0, 0, 0, 1, 1) == -1
    assert lib.e4b_last_error(None) == b"null context"


def test_create_fails_cleanly_without_gpu(e4b):
    lib = e4b.lib()
    h = ctypes.c_void_p()
    rc = lib.e4b_create(0, ctypes.byref(h))
    if rc == 0:
        lib.e4b_destroy(h)
        pytest.skip("a CUDA device is present")
    assert rc == -2 and not h.value
    with pytest.raises(e4b.E4BError):
        e4b.Device(0)


def test_dense_plan_struct_layout_matches_header(e4b, tmp_path):
    """The ctypes mirrors of e4b_dense_layer / e4b_dense_model have the C layout."""
    from importlib import import_module
    eng = import_module("e4b-webgpu_b200.engine")
    structs = {"e4b_dense_layer": eng.DenseLayer, "e4b_dense_model": eng.DenseModel}
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "e4b_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for f, _ in py._fields_:
            lines.append(f'  printf("{cname} {f} %zu\\n", offsetof({cname}, {f}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    inc = e4b._lib.HEADER.rsplit("/", 1)[0]
    subprocess.run(["gcc", "-I", inc, str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {}
    for ln in out:
        if ln:
            cname, field, val = ln.split()
            got[(cname, field)] = int(val)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for f, _ in py._fields_:
            assert got[(cname, f)] == getattr(py, f).offset, (cname, f)

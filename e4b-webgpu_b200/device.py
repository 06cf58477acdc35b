"""Device context and buffers over the C ABI (replaces src/gpu.js:4-50).

`Device` owns one e4b_ctx (one CUDA device + stream).  `Buffer` is a device
allocation with a byte size; `Device.call(name, ...)` runs any C-ABI function
on the context and raises E4BError with the library's message on failure.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import E4BError, lib


class Buffer:
    __slots__ = ("dev", "ptr", "nbytes", "name")

    def __init__(self, dev: "Device", ptr: int, nbytes: int, name: str = ""):
        self.dev, self.ptr, self.nbytes, self.name = dev, ptr, nbytes, name

    def at(self, offset_bytes: int) -> int:
        """Device address `offset_bytes` into the buffer."""
        assert 0 <= offset_bytes <= self.nbytes
        return self.ptr + offset_bytes

    def __int__(self):
        return self.ptr

    def __repr__(self):
        return f"Buffer({self.name!r}, {self.nbytes} B @ {self.ptr:#x})"


_RUNTIME = {"e4b_create", "e4b_destroy", "e4b_device_info", "e4b_alloc", "e4b_free", "e4b_host_alloc",
            "e4b_host_free", "e4b_upload", "e4b_download", "e4b_upload_async", "e4b_download_async", "e4b_memset",
            "e4b_copy", "e4b_sync", "e4b_event_record", "e4b_event_elapsed", "e4b_set_pdl", "e4b_device_status",
            "e4b_plan_begin", "e4b_plan_end", "e4b_plan_launch", "e4b_plan_destroy", "e4b_set_workspace",
            "e4b_set_option", "e4b_dense_plan_create", "e4b_dense_plan_destroy",
            "e4b_dense_plan_trace", "e4b_dense_plan_phases", "e4b_nccl_init", "e4b_nccl_destroy",
            "e4b_ep_exchange", "e4b_ep_exchange2_async", "e4b_ep_join", "e4b_ep_allgather", "e4b_ipc_handle",
            "e4b_ipc_open", "e4b_ipc_close", "e4b_side_begin", "e4b_side_end", "e4b_join"}


def _ptr(x):
    if x is None:
        return None
    if isinstance(x, Buffer):
        return x.ptr
    return int(x)


class Device:
    # C-ABI functions that enqueue kernels, with the number of kernels each launches
    KERNELS = {"e4b_argmax": 2, "e4b_argmax_static": 2, "e4b_argmax_rows": 2, "e4b_q6k_lmhead_rows": 2,
               "e4b_q6k_lmhead_tiles": 2, "e4b_attdec_seq": 2}

    def __init__(self, device: int = 0):
        self.kernel_launches = 0
        self.L = lib()
        h = ctypes.c_void_p()
        rc = self.L.e4b_create(device, ctypes.byref(h))
        if rc != 0 or not h.value:
            raise E4BError("e4b_create", rc, f"cannot open CUDA device {device} (no GPU, or driver error)")
        self.ctx = h
        self.index = device
        self.buffers = []
        sm, ma, mi, mem = ctypes.c_int(), ctypes.c_int(), ctypes.c_int(), ctypes.c_size_t()
        self.call("e4b_device_info", ctypes.byref(sm), ctypes.byref(ma), ctypes.byref(mi), ctypes.byref(mem))
        self.sm_count, self.cc, self.total_mem = sm.value, (ma.value, mi.value), mem.value

    # ---- calls
    def call(self, name: str, *args):
        conv = [(_ptr(a) if isinstance(a, Buffer) else a) for a in args]
        rc = getattr(self.L, name)(self.ctx, *conv)
        if rc != 0:
            raise E4BError(name, rc, self.last_error())
        if name == "e4b_set_workspace":
            self.has_workspace = bool(conv[0])
        if name not in _RUNTIME:
            n = self.KERNELS.get(name, 1)
            if name == "e4b_routertop" and getattr(self, "has_workspace", False):
                n = 2          # split-K scores + per-token top-K
            if name == "e4b_q6k_lmhead_tiles" and args[-1] == 1:
                n = 1          # one token: the GEMV alone, no activation split
            self.kernel_launches += n
        return rc

    def last_error(self) -> str:
        m = self.L.e4b_last_error(self.ctx)
        return m.decode() if m else ""

    # ---- memory
    def alloc(self, nbytes: int, name: str = "", zero: bool = True) -> Buffer:
        p = ctypes.c_void_p()
        self.call("e4b_alloc", ctypes.c_size_t(max(int(nbytes), 16)), ctypes.byref(p))
        b = Buffer(self, p.value, int(nbytes), name)
        self.buffers.append(b)
        if zero:
            self.memset(b, 0)
        return b

    def upload(self, arr: np.ndarray, name: str = "") -> Buffer:
        a = np.ascontiguousarray(arr)
        b = self.alloc(a.nbytes, name, zero=False)
        self.write(b, a)
        return b

    def write(self, buf, arr: np.ndarray, offset: int = 0):
        a = np.ascontiguousarray(arr)
        dst = _ptr(buf) + offset
        self.call("e4b_upload", ctypes.c_void_p(dst), a.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(a.nbytes))

    def read(self, buf, dtype, count: int, offset: int = 0) -> np.ndarray:
        out = np.empty(count, dtype=dtype)
        src = _ptr(buf) + offset
        self.call("e4b_download", out.ctypes.data_as(ctypes.c_void_p), ctypes.c_void_p(src), ctypes.c_size_t(out.nbytes))
        return out

    def memset(self, buf, value: int = 0, nbytes: int | None = None):
        n = buf.nbytes if nbytes is None else nbytes
        self.call("e4b_memset", ctypes.c_void_p(_ptr(buf)), value, ctypes.c_size_t(max(n, 0)))

    def free(self, buf: Buffer):
        self.call("e4b_free", ctypes.c_void_p(buf.ptr))
        self.buffers.remove(buf)

    def sync(self):
        self.call("e4b_sync")

    def status(self) -> int:
        st = ctypes.c_uint32()
        self.call("e4b_device_status", ctypes.byref(st))
        return st.value

    def close(self):
        if self.ctx:
            for b in list(self.buffers):
                self.L.e4b_free(self.ctx, ctypes.c_void_p(b.ptr))
            self.buffers.clear()
            self.L.e4b_destroy(self.ctx)
            self.ctx = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

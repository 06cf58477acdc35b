"""The Python host's C-ABI calls checked on the CPU: a stand-in device accepts
every call only if the header declares the function and each argument converts
to the declared ctypes type (the conversion a real call performs), and answers
the out-parameters (allocations, events, plan handles) with placeholders.  The
engines then run their whole host side -- weight upload, per-token plan
recording and replay, generate, close -- for the dense graph (per-operator and
fused), the batched MoE graph, and expert parallelism over NCCL and over peer
memory, so an argument-count or type mistake on any path shows here rather than
on a GPU."""
import ctypes
import importlib

import numpy as np
import pytest


@pytest.fixture(scope="module")
def pkg(e4b):
    return e4b


def make_device(e4b):
    """A Device subclass (so the engines accept it) that checks and answers calls."""
    dev_mod = importlib.import_module("e4b-webgpu_b200.device")
    lib_mod = importlib.import_module("e4b-webgpu_b200._lib")
    protos = lib_mod.parse_header()

    class StandInDevice(dev_mod.Device):
        def __init__(self):
            self.kernel_launches = 0
            self.L = lib_mod.lib()
            self.ctx = ctypes.c_void_p(1)
            self.index = 0
            self.buffers = []
            self.sm_count, self.cc, self.total_mem = 148, (10, 0), 180 << 30
            self.names = []
            self._next = 1 << 32
            self._host = []

        def _fake_ptr(self, n):
            p = self._next
            self._next += (int(n) + 255) // 256 * 256 + 256
            return p

        def call(self, name, *args):
            assert name in protos, f"{name} is not declared in the header"
            _, argtypes = protos[name]
            conv = [(dev_mod._ptr(a) if isinstance(a, dev_mod.Buffer) else a) for a in args]
            assert len(conv) + 1 == len(argtypes), f"{name}: {len(conv)} arguments, header has {len(argtypes) - 1}"
            for i, (a, t) in enumerate(zip(conv, argtypes[1:])):
                try:
                    t.from_param(a)
                except Exception as exc:              # the conversion a real call would reject
                    raise AssertionError(f"{name} argument {i}: {a!r} does not convert to {t}: {exc}")
            self.names.append(name)
            out = conv[-1] if conv else None
            if name in ("e4b_alloc", "e4b_ipc_open"):
                out._obj.value = self._fake_ptr(conv[0].value if name == "e4b_alloc" else 64)
            elif name == "e4b_host_alloc":
                buf = ctypes.create_string_buffer(conv[0].value)
                self._host.append(buf)
                out._obj.value = ctypes.addressof(buf)
            elif name == "e4b_download":
                ctypes.memset(conv[0], 0, conv[2].value)
            elif name in ("e4b_device_status",):
                out._obj.value = 0
            elif name in ("e4b_plan_end", "e4b_dense_plan_create"):
                out._obj.value = 1
            elif name == "e4b_event_elapsed":
                out._obj.value = 1.0
            elif name == "e4b_ipc_handle":
                ctypes.memset(out, 7, 64)
            if name not in dev_mod._RUNTIME:
                self.kernel_launches += self.KERNELS.get(name, 1)
            return 0

        def close(self):
            self.buffers.clear()

    return StandInDevice()


def test_dense_engine_host_calls(pkg):
    cfg = pkg.config.get("tiny_ple")
    img = pkg.synth.build_model(cfg)
    for fused in (False, True):
        dev = make_device(pkg)
        eng = pkg.Engine(img, dev, fused=fused)
        ids = eng.generate([1, 2, 3], 4)
        assert len(ids) == 4
        eng.close()
        assert ("e4b_dense_plan_create" in dev.names) == fused


@pytest.mark.parametrize("ep,transport", [(None, "nccl"), ((2, 0), "nccl"), ((2, 1), "p2p")])
def test_batch_engine_host_calls(pkg, ep, transport):
    cfg = pkg.config.get("tiny_moe")
    img = pkg.synth.build_model(cfg)
    dev = make_device(pkg)
    epx = None if ep is None else (ep[0], ep[1], bytes(128))
    eng = pkg.BatchEngine(img, 3, dev, ep=epx, zipf=1.1 if ep else None, ep_transport=transport)
    ids = eng.generate(np.zeros((3, 4), np.uint32), 3)
    assert ids.shape == (3, 3)
    if ep is not None:
        assert eng.exchange_time(7) >= 0.0
    eng.close()
    want = {None: {"e4b_expgroup"}, "nccl": {"e4b_ep_exchange2_async", "e4b_ep_join", "e4b_ep_exchange"},
            "p2p": {"e4b_ipc_handle", "e4b_ipc_open", "e4b_ep_push", "e4b_ep_wait", "e4b_ep_push_back",
                    "e4b_ipc_close"}}[None if ep is None else transport]
    assert want <= set(dev.names), want - set(dev.names)
    if transport == "p2p":
        assert not {"e4b_ep_exchange", "e4b_ep_exchange2_async"} & set(dev.names)

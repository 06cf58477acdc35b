"""B200-native (sm_100a) per-token decode path of Verilean/e4b-webgpu.

The reference's WGSL operators (q40mv, q40gu, q40moedown, q6k, rmsacc3,
a4btail, routertop, headprep, attsplit/attcomb, pleprep, argmax2, ...) are
CUDA kernels in libe4b_b200.so behind the C ABI of include/e4b_b200.h; this
package is the Python host (ctypes) that mirrors the reference's engine API.
The package directory name contains a hyphen, so import it with
``importlib.import_module("e4b-webgpu_b200")``.
"""
from . import config, gguf, ops, synth  # noqa: F401
from ._lib import E4BError, lib  # noqa: F401
from .config import ModelConfig  # noqa: F401
from .device import Buffer, Device  # noqa: F401
from .engine import DeviceStatusError, Engine  # noqa: F401
from .batch import BatchEngine  # noqa: F401

__all__ = ["Engine", "DeviceStatusError", "BatchEngine", "Device", "Buffer", "ModelConfig", "E4BError", "config", "gguf", "ops", "synth", "lib"]

"""Seeded synthetic GGUF models.

Every linear weight is N(0, 0.02) fp32 quantised to q4_0; the tied token
embedding / LM head and the per-layer-embedding table are q6_K; norm weights,
layer scales, router input scales and per-expert scales are 1.0 (f32); the
router is f32 N(0, 0.02).  Each tensor draws from its own generator stream
(keyed by its name), so adding a tensor never shifts another one's values.
The generator and quantisers are host C (csrc/synth.c) running on all cores.

Tensor names follow the reference's GGUF names where it has them
(src/engine-a4b.js:141-214); the per-layer-embedding tensors (which the
reference only has in safetensors form, src/engine.js:122-134) use
llama.cpp gemma3n-style names (see `build_model`).
"""
from __future__ import annotations

import ctypes
import os
import zlib

import numpy as np

from . import gguf
from .config import ModelConfig

_HERE = os.path.dirname(os.path.abspath(__file__))
_SYNTH = None


def synth_lib():
    global _SYNTH
    if _SYNTH is None:
        path = os.path.join(_HERE, "libe4b_synth.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run __graft_entry__.build() first")
        lib = ctypes.CDLL(path)
        u8p = ctypes.POINTER(ctypes.c_uint8)
        f32p = ctypes.POINTER(ctypes.c_float)
        lib.e4b_synth_q4_0.argtypes = [u8p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]
        lib.e4b_synth_q6_K.argtypes = [u8p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]
        lib.e4b_synth_normal_f32.argtypes = [f32p, ctypes.c_int64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float]
        lib.e4b_quant_q4_0.argtypes = [f32p, u8p, ctypes.c_int64]
        lib.e4b_quant_q6_K.argtypes = [f32p, u8p, ctypes.c_int64]
        lib.e4b_synth_threads.restype = ctypes.c_int
        _SYNTH = lib
    return _SYNTH


def _u8p(a: np.ndarray):
    assert a.dtype == np.uint8 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))


def _f32p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def stream_of(name: str) -> int:
    return zlib.crc32(name.encode()) | (len(name) << 32)


def normal_f32(n: int, seed: int, name: str, std: float) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    synth_lib().e4b_synth_normal_f32(_f32p(out), n, seed, stream_of(name), std)
    return out


def quant_q4_0(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    assert x.size % 32 == 0
    out = np.empty(x.size // 32 * 18, dtype=np.uint8)
    synth_lib().e4b_quant_q4_0(_f32p(x), _u8p(out), x.size // 32)
    return out


def quant_q6_K(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    assert x.size % 256 == 0
    out = np.empty(x.size // 256 * 210, dtype=np.uint8)
    synth_lib().e4b_quant_q6_K(_f32p(x), _u8p(out), x.size // 256)
    return out


def _fill_q40(seed, name, std):
    def f(out):
        synth_lib().e4b_synth_q4_0(_u8p(out), out.size // 18, seed, stream_of(name), std)
    return f


def _fill_q6k(seed, name, std):
    def f(out):
        synth_lib().e4b_synth_q6_K(_u8p(out), out.size // 210, seed, stream_of(name), std)
    return f


def _fill_const(v):
    def f(out):
        out.view(np.float32)[:] = np.float32(v)
    return f


def _fill_normal(seed, name, std):
    def f(out):
        o = out.view(np.float32)
        synth_lib().e4b_synth_normal_f32(_f32p(o), o.size, seed, stream_of(name), std)
    return f


def _fill_shifted(seed, name, val, std):
    def f(out):
        o = out.view(np.float32)
        synth_lib().e4b_synth_normal_f32(_f32p(o), o.size, seed, stream_of(name), std)
        o += np.float32(val)
    return f


def build_model(cfg: ModelConfig, seed: int = 0, std: float = 0.02, path: str | None = None,
                vec_std: float = 0.0, router_std: float | None = None) -> np.ndarray:
    """Build a synthetic GGUF image for `cfg` (in memory, or at `path`); returns the uint8 buffer.
    vec_std > 0 draws every f32 vector (norm weights, router / expert / layer
    scales) as its constant + N(0, vec_std) instead of the constant, so a test
    can tell the vectors apart; router_std (default: std) is the router
    weights' deviation -- larger values give peaked routing with fewer near-tied
    expert choices.  The benchmark models keep the defaults."""
    w = gguf.GGUFWriter()
    for k, v in cfg.to_kv().items():
        w.add_kv(k, v)
    H, V = cfg.hidden, cfg.vocab
    Q4, Q6, F32 = gguf.GGML_Q4_0, gguf.GGML_Q6_K, gguf.GGML_F32

    def lin(name, n_in, n_out):
        w.add_tensor(name, [n_in, n_out], Q4, _fill_q40(seed, name, std))

    def vec(name, n, val=1.0):
        w.add_tensor(name, [n], F32, _fill_const(val) if vec_std <= 0 else _fill_shifted(seed, name, val, vec_std))

    w.add_tensor("token_embd.weight", [H, V], Q6, _fill_q6k(seed, "token_embd.weight", std))
    vec("output_norm.weight", H)
    if cfg.ple_dim:
        PD, L = cfg.ple_dim, cfg.layers
        w.add_tensor("per_layer_token_embd.weight", [L * PD, V], Q6,
                     _fill_q6k(seed, "per_layer_token_embd.weight", std))
        lin("per_layer_model_proj.weight", H, L * PD)
        vec("per_layer_proj_norm.weight", PD)
    for l in range(cfg.layers):
        p = f"blk.{l}."
        hd = cfg.head_dim
        vec(p + "attn_norm.weight", H)
        lin(p + "attn_q.weight", H, cfg.q_heads * hd)
        lin(p + "attn_k.weight", H, cfg.kv_heads * hd)
        if not cfg.keqv(l):
            lin(p + "attn_v.weight", H, cfg.kv_heads * hd)
        vec(p + "attn_q_norm.weight", hd)
        vec(p + "attn_k_norm.weight", hd)
        lin(p + "attn_output.weight", cfg.q_heads * hd, H)
        vec(p + "post_attention_norm.weight", H)
        vec(p + "ffn_norm.weight", H)
        lin(p + "ffn_gate.weight", H, cfg.ff)
        lin(p + "ffn_up.weight", H, cfg.ff)
        lin(p + "ffn_down.weight", cfg.ff, H)
        vec(p + "post_ffw_norm.weight", H)
        vec(p + "layer_output_scale.weight", 1)
        if cfg.ple_dim:
            lin(p + "inp_gate.weight", H, cfg.ple_dim)
            lin(p + "proj.weight", cfg.ple_dim, H)
            vec(p + "post_norm.weight", H)
        if cfg.moe:
            E, EF = cfg.experts, cfg.expert_ff
            vec(p + "post_ffw_norm_1.weight", H)
            vec(p + "post_ffw_norm_2.weight", H)
            vec(p + "pre_ffw_norm_2.weight", H)
            vec(p + "ffn_gate_inp.scale", H)
            vec(p + "ffn_down_exps.scale", E)
            w.add_tensor(p + "ffn_gate_inp.weight", [H, E], F32,
                         _fill_normal(seed, p + "ffn_gate_inp.weight", std if router_std is None else router_std))
            w.add_tensor(p + "ffn_gate_up_exps.weight", [H, 2 * EF, E], Q4,
                         _fill_q40(seed, p + "ffn_gate_up_exps.weight", std))
            w.add_tensor(p + "ffn_down_exps.weight", [EF, H, E], Q4,
                         _fill_q40(seed, p + "ffn_down_exps.weight", std))
    return w.build(path)


def prompt_ids(n: int, vocab: int, seed: int = 0) -> np.ndarray:
    """Uniform token ids in [0, vocab) from numpy's default_rng(seed)."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)

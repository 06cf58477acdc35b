"""Models of the transformers parity pin (made by tests/golden/make_pin.py,
checked by tests/test_pin_transformers.py and tests/test_pin_gpu.py).

Small synthetic Gemma-4 graphs that together cover every operator on the
decode path, built by e4b-webgpu_b200/synth.py with non-constant norm weights
and scales (vec_std), so a swapped or missing vector shows.
"""
from __future__ import annotations

import dataclasses
import functools
import importlib

VEC_STD = 0.15
ROUTER_STD = 1.0      # peaked routing: few near-tied expert choices for f16 storage to flip
SEED = 0

CASES = {
    # dense, two global layers, every RoPE pair rotating at theta 1e4 (benchmark config 1's shape)
    "tiny": dict(base="tiny", P=16, N=8, seed=102),
    # dense + per-layer embeddings; sliding ring (window 16 in 24 slots) wraps; partial-RoPE global layer last
    "tiny_ple": dict(base="tiny_ple", sliding=[True, True, True, False], P=32, N=8, seed=104),
    # MoE, top-4 of 16 experts, a k_eq_v global layer
    "tiny_moe": dict(base="tiny_moe", P=32, N=8, seed=103),
    # the E4B layer geometry (8q/2kv x 256, 4 sliding : 1 global, PLE 256) at hidden 512
    "e4b_heads": dict(base="e4b", hidden=512, layers=5, ff=1024, vocab=4096, window=16, ring_slack=8,
                      sliding=[True, True, True, True, False], max_ctx=1024, P=28, N=8, seed=101),
    # the A4B layer geometry (16q/4kv x 256, 5 sliding : 1 k_eq_v global, top-8 experts) at hidden 512
    "a4b_heads": dict(base="a4b", hidden=512, layers=6, ff=384, vocab=4096, experts=32, expert_ff=192, window=16,
                      ring_slack=8, sliding=[True, True, True, True, True, False], max_ctx=1024, P=28, N=8, seed=100),
    # benchmark config 2 at full width (hidden 2048, FF 16384, vocab 262144, PLE, window 512): one
    # 4 sliding : 1 global period of its 35 layers
    "e4b_5l": dict(base="e4b", layers=5, sliding=[True, True, True, True, False], max_ctx=1024, P=16, N=8,
                   seed=105),
    # benchmark config 4 at full width (hidden 2816, 128 experts top-8, vocab 262144): a sliding
    # and a k_eq_v global layer of its 30
    "a4b_2l": dict(base="a4b", layers=2, sliding=[True, False], max_ctx=1024, P=16, N=8, seed=106),
}
# hidden states stored at these many positions (first and last) for the full-width cases
FEW_POSITIONS = {"e4b_5l", "a4b_2l"}


def _pkg():
    return importlib.import_module("e4b-webgpu_b200")


def config(name: str):
    spec = dict(CASES[name])
    base = spec.pop("base")
    for k in ("P", "N", "seed"):
        spec.pop(k)
    return dataclasses.replace(_pkg().config.get(base), name=f"pin_{name}", **spec)


@functools.lru_cache(maxsize=None)
def build(name: str):
    """(config, GGUF image, prompt ids, new tokens) of a pin case (built once
    per process; the image is shared, not to be modified)."""
    e4b = _pkg()
    cfg = config(name)
    img = e4b.synth.build_model(cfg, seed=SEED, vec_std=VEC_STD, router_std=ROUTER_STD)
    prompt = e4b.synth.prompt_ids(CASES[name]["P"], cfg.vocab, seed=CASES[name]["seed"])
    return cfg, img, prompt, CASES[name]["N"]

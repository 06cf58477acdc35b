"""Model configurations for the decode path.

A config is read from GGUF key/values the way the reference reads its model
config (src/engine-a4b.js:100-116); `to_kv()` writes the same keys for the
synthetic models.  Layer types follow the reference: sliding-window layers use
a ring KV cache of `window + ring_slack` slots with full RoPE at theta 10k, global
layers use a linear cache with partial RoPE (a quarter of the pairs rotate) at
theta 1M (src/engine-a4b.js:328-347).

Named shapes (benchmark configs):
  tiny      2L, H=512, 4q/1kv x 128, FF 2048, V 4096, all layers global
  e4b       35L, H=2048, 8q/2kv x 256, FF 16384, V 262144, PLE 256/layer,
            4 sliding (W=512) : 1 global
  a4b       30L, H=2816, 16q/4kv x 256, 128 experts top-8, expert FF 704,
            dense FF 2112, V 262144, 5 sliding (W=1024) : 1 global (k_eq_v)
Test-only shapes (small, exercise every operator the big ones use):
  tiny_ple  tiny + PLE + sliding ring layers + a global partial-RoPE layer
  tiny_moe  small MoE with a k_eq_v global layer
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field, asdict


@dataclass
class ModelConfig:
    name: str
    arch: str                   # "dense" (E4B graph, optional PLE) or "moe" (A4B graph)
    hidden: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    ff: int                     # dense GeGLU hidden
    vocab: int
    eps: float = 1e-6
    softcap: float = 30.0
    window: int = 0             # sliding window (0: no sliding layers)
    sliding: list = field(default_factory=list)   # per-layer: True = sliding
    ring_slack: int = 512       # sliding ring = window + slack (src/engine-a4b.js:343)
    theta_sliding: float = 10000.0
    theta_global: float = 1000000.0
    rope_frac_global: float = 0.25
    ple_dim: int = 0            # per-layer-embedding width (0: none)
    experts: int = 0
    topk: int = 0
    expert_ff: int = 0
    keqv_global: bool = False   # global layers reuse the K projection for V
    max_ctx: int = 8192         # KV capacity of global layers

    # ---- derived ----
    def is_sliding(self, l: int) -> bool:
        return bool(self.sliding[l]) if self.sliding else False

    def keqv(self, l: int) -> bool:
        return self.keqv_global and not self.is_sliding(l)

    def rope_angles(self, l: int) -> int:
        half = self.head_dim // 2
        return half if self.is_sliding(l) else int(math.floor(self.rope_frac_global * self.head_dim / 2))

    def theta(self, l: int) -> float:
        return self.theta_sliding if self.is_sliding(l) else self.theta_global

    def ring(self, l: int) -> int:
        return self.window + self.ring_slack if self.is_sliding(l) else 1

    def kv_slots(self, l: int) -> int:
        return self.ring(l) if self.is_sliding(l) else self.max_ctx

    def qkv_rows(self, l: int) -> int:
        kv = self.kv_heads * self.head_dim
        return self.q_heads * self.head_dim + kv * (1 if self.keqv(l) else 2)

    @property
    def q_dim(self) -> int:
        return self.q_heads * self.head_dim

    @property
    def moe(self) -> bool:
        return self.arch == "moe"

    def to_kv(self) -> dict:
        a = "gemma4."
        kv = {
            "general.architecture": "gemma4",
            "general.name": self.name,
            "e4b.arch": self.arch,
            a + "embedding_length": self.hidden,
            a + "block_count": self.layers,
            a + "attention.head_count": self.q_heads,
            a + "attention.head_count_kv": [self.kv_heads] * self.layers,
            a + "attention.key_length": self.head_dim,
            a + "attention.key_length_swa": self.head_dim,
            a + "feed_forward_length": self.ff,
            a + "vocab_size": self.vocab,
            a + "attention.layer_norm_rms_epsilon": float(self.eps),
            a + "final_logit_softcapping": float(self.softcap),
            a + "attention.sliding_window": self.window,
            a + "attention.sliding_window_pattern": [bool(self.is_sliding(l)) for l in range(self.layers)],
            a + "rope.freq_base_swa": float(self.theta_sliding),
            a + "rope.freq_base": float(self.theta_global),
            a + "rope.partial_rotary_factor": float(self.rope_frac_global),
            a + "embedding_length_per_layer_input": self.ple_dim,
            a + "expert_count": self.experts,
            a + "expert_used_count": self.topk,
            a + "expert_feed_forward_length": self.expert_ff,
            a + "attention.k_eq_v_global": bool(self.keqv_global),
            "e4b.ring_slack": self.ring_slack,
            "e4b.max_ctx": self.max_ctx,
        }
        return kv

    @classmethod
    def from_kv(cls, kv: dict) -> "ModelConfig":
        a = "gemma4."
        L = int(kv[a + "block_count"])
        kvh = kv[a + "attention.head_count_kv"]
        kvh = int(kvh[0]) if isinstance(kvh, list) else int(kvh)
        return cls(
            name=str(kv.get("general.name", "gguf")),
            arch=str(kv.get("e4b.arch", "moe" if int(kv.get(a + "expert_count", 0)) else "dense")),
            hidden=int(kv[a + "embedding_length"]), layers=L,
            q_heads=int(kv[a + "attention.head_count"]), kv_heads=kvh,
            head_dim=int(kv[a + "attention.key_length"]),
            ff=int(kv[a + "feed_forward_length"]), vocab=int(kv[a + "vocab_size"]),
            eps=float(kv[a + "attention.layer_norm_rms_epsilon"]),
            softcap=float(kv[a + "final_logit_softcapping"]),
            window=int(kv.get(a + "attention.sliding_window", 0)),
            sliding=[bool(x) for x in kv.get(a + "attention.sliding_window_pattern", [False] * L)],
            ring_slack=int(kv.get("e4b.ring_slack", 512)),
            theta_sliding=float(kv.get(a + "rope.freq_base_swa", 10000.0)),
            theta_global=float(kv.get(a + "rope.freq_base", 1000000.0)),
            rope_frac_global=float(kv.get(a + "rope.partial_rotary_factor", 0.25)),
            ple_dim=int(kv.get(a + "embedding_length_per_layer_input", 0)),
            experts=int(kv.get(a + "expert_count", 0)), topk=int(kv.get(a + "expert_used_count", 0)),
            expert_ff=int(kv.get(a + "expert_feed_forward_length", 0)),
            keqv_global=bool(kv.get(a + "attention.k_eq_v_global", False)),
            max_ctx=int(kv.get("e4b.max_ctx", 8192)),
        )

    def as_dict(self) -> dict:
        return asdict(self)


def _pattern(L: int, period: int) -> list:
    """Sliding everywhere except every `period`-th layer (index % period == period-1)."""
    return [(l % period) != period - 1 for l in range(L)]


def tiny() -> ModelConfig:
    # benchmark config 1: all-global layers, RoPE theta 10000 with every pair rotating.
    return ModelConfig(name="tiny", arch="dense", hidden=512, layers=2, q_heads=4, kv_heads=1,
                       head_dim=128, ff=2048, vocab=4096, window=0, sliding=[False, False],
                       theta_global=10000.0, rope_frac_global=1.0, max_ctx=1024)


def e4b() -> ModelConfig:
    return ModelConfig(name="e4b", arch="dense", hidden=2048, layers=35, q_heads=8, kv_heads=2,
                       head_dim=256, ff=16384, vocab=262144, window=512, sliding=_pattern(35, 5),
                       ple_dim=256, max_ctx=2048)


def a4b() -> ModelConfig:
    return ModelConfig(name="a4b", arch="moe", hidden=2816, layers=30, q_heads=16, kv_heads=4,
                       head_dim=256, ff=2112, vocab=262144, window=1024, sliding=_pattern(30, 6),
                       experts=128, topk=8, expert_ff=704, keqv_global=True, max_ctx=4096)


def tiny_ple() -> ModelConfig:
    # sliding rings of 24 slots (wrap early), one global layer, PLE width 256
    return ModelConfig(name="tiny_ple", arch="dense", hidden=512, layers=4, q_heads=4, kv_heads=2,
                       head_dim=128, ff=1024, vocab=4096, window=16, ring_slack=8,
                       sliding=[True, True, False, True], ple_dim=256, max_ctx=1024)


def tiny_moe() -> ModelConfig:
    return ModelConfig(name="tiny_moe", arch="moe", hidden=512, layers=3, q_heads=4, kv_heads=2,
                       head_dim=128, ff=384, vocab=4096, window=16, ring_slack=8,
                       sliding=[True, True, False], experts=16, topk=4, expert_ff=192,
                       keqv_global=True, max_ctx=1024)


CONFIGS = {"tiny": tiny, "e4b": e4b, "a4b": a4b, "tiny_ple": tiny_ple, "tiny_moe": tiny_moe}


def get(name: str) -> ModelConfig:
    if name not in CONFIGS:
        raise KeyError(f"unknown config {name!r}; known: {sorted(CONFIGS)}")
    return CONFIGS[name]()

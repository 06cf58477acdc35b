"""Regenerate tests/golden/golden.npz (run from the repository root:
`python tests/golden/make_golden.py`).

Contents:
  * q40_raw / q40_deq, q6k_raw / q6k_deq: seeded q4_0 and q6_K blocks and their
    f32 dequantisation by the python `gguf` package (an independent decoder of
    the GGML block formats), including edge blocks (all-zero, extreme scales);
  * for the `tiny` (benchmark config 1: 32-token prompt from seed 0, 32 greedy
    tokens) and `tiny_ple` models built by e4b-webgpu_b200/synth.py: the sha256
    of the GGUF image, the prompt, the oracle's greedy ids and top-2 margins, the
    per-step per-layer hidden-state norms of the prompt steps, and the final
    hidden state.
"""
import hashlib
import importlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main():
    import gguf as gguf_pkg
    import __graft_entry__
    __graft_entry__.build()
    e4b = importlib.import_module("e4b-webgpu_b200")
    from oracle.model import OracleModel

    out = {}
    x = e4b.synth.normal_f32(32 * 64, 11, "golden_q40", 0.02)
    x[:32] = 0.0
    x[32] = -1.0
    x[64:96] = np.linspace(-3.0, 3.0, 32)
    raw = e4b.synth.quant_q4_0(x)
    out["q40_raw"] = raw
    out["q40_deq"] = gguf_pkg.quants.dequantize(raw.reshape(-1, 18), gguf_pkg.GGMLQuantizationType.Q4_0).reshape(-1)
    y = e4b.synth.normal_f32(256 * 8, 12, "golden_q6k", 0.02)
    y[:256] = 0.0
    y[256:512] *= 1e3
    raw6 = e4b.synth.quant_q6_K(y)
    out["q6k_raw"] = raw6
    out["q6k_deq"] = gguf_pkg.quants.dequantize(raw6.reshape(-1, 210), gguf_pkg.GGMLQuantizationType.Q6_K).reshape(-1)

    for name, P, N in (("tiny", 32, 32), ("tiny_ple", 20, 24)):
        cfg = e4b.config.get(name)
        img = np.asarray(e4b.synth.build_model(cfg))
        prompt = e4b.synth.prompt_ids(P, cfg.vocab, seed=0)
        ids, margins, recs = OracleModel(img).generate(prompt, N, record=True)
        out[f"{name}_sha256"] = np.frombuffer(hashlib.sha256(img.tobytes()).digest(), np.uint8)
        out[f"{name}_prompt"] = np.asarray(prompt, np.int64)
        out[f"{name}_ids"] = np.asarray(ids, np.int64)
        out[f"{name}_margins"] = np.asarray(margins, np.float64)
        out[f"{name}_hidden_norms"] = np.array([np.linalg.norm(r["hidden"], axis=1) for r in recs[:P]], np.float64)
        out[f"{name}_final_hidden"] = np.asarray(recs[-1]["hidden"][-1], np.float32)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()

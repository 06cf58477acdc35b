"""Regenerate the transformers parity fixtures tests/golden/pin_<case>.npz
(run from the repository root: `python tests/golden/make_pin.py`).

The reference makes its golden vectors with transformers on the CPU in f32
(goldens/gen.py: AutoModelForCausalLM, model.generate(do_sample=False), per-layer
hidden states).  This script runs the same implementation of the same
architecture -- transformers' Gemma4ForCausalLM, eager attention, f32, CPU --
on the synthetic models of tests/golden/pin_cases.py: each GGUF image is read
and its q4_0 / q6_K / f32 tensors dequantised by the python `gguf` package (an
implementation independent of this repository), loaded into the transformers
modules by name, and run.

Per case the fixture holds: the prompt; the greedy ids of model.generate; the
top-2 logit margin of every greedy step; every layer's output hidden state at
the positions in `pos`; the 16 largest logits (ids and values) at every
position of the teacher-forced sequence prompt + ids[:-1]; the sha256 of the
GGUF image; the library versions.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)

import pin_cases  # noqa: E402

TOPN = 16


def gguf_tensors(img) -> dict:
    """name -> f32 torch tensor, decoded by the `gguf` package."""
    import gguf
    import torch
    fd, path = tempfile.mkstemp(suffix=".gguf")
    os.close(fd)
    try:
        np.asarray(img).tofile(path)
        r = gguf.GGUFReader(path)
        return {t.name: torch.from_numpy(np.array(gguf.quants.dequantize(t.data, t.tensor_type), dtype=np.float32))
                for t in r.tensors}
    finally:
        os.unlink(path)


def transformers_model(cfg, img):
    """Gemma4ForCausalLM (f32, eager attention, CPU) holding the GGUF's weights."""
    import torch
    from transformers import Gemma4ForCausalLM, Gemma4TextConfig
    W = gguf_tensors(img)
    L = cfg.layers
    types = ["sliding_attention" if cfg.is_sliding(l) else "full_attention" for l in range(L)]
    rope = {"full_attention": {"rope_type": "proportional", "partial_rotary_factor": cfg.rope_frac_global,
                               "rope_theta": cfg.theta_global}}
    if "sliding_attention" in types:
        rope["sliding_attention"] = {"rope_type": "default", "rope_theta": cfg.theta_sliding}
    tc = Gemma4TextConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.ff, num_hidden_layers=L,
        num_attention_heads=cfg.q_heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
        global_head_dim=cfg.head_dim, num_global_key_value_heads=cfg.kv_heads,
        hidden_activation="gelu_pytorch_tanh", rms_norm_eps=cfg.eps, sliding_window=max(cfg.window, 1),
        layer_types=types, final_logit_softcapping=cfg.softcap, rope_parameters=rope,
        vocab_size_per_layer_input=cfg.vocab, hidden_size_per_layer_input=cfg.ple_dim or 0,
        attention_k_eq_v=cfg.keqv_global, num_kv_shared_layers=0, enable_moe_block=bool(cfg.moe),
        num_experts=cfg.experts or None, top_k_experts=cfg.topk or None,
        moe_intermediate_size=cfg.expert_ff or None, tie_word_embeddings=True, max_position_embeddings=4096)
    tc._attn_implementation = "eager"
    model = Gemma4ForCausalLM(tc).eval()
    sd = {"model.embed_tokens.weight": W["token_embd.weight"], "model.norm.weight": W["output_norm.weight"]}
    if cfg.ple_dim:
        sd["model.embed_tokens_per_layer.weight"] = W["per_layer_token_embd.weight"]
        sd["model.per_layer_model_projection.weight"] = W["per_layer_model_proj.weight"]
        sd["model.per_layer_projection_norm.weight"] = W["per_layer_proj_norm.weight"]
    names = {
        "input_layernorm.weight": "attn_norm.weight", "self_attn.q_proj.weight": "attn_q.weight",
        "self_attn.k_proj.weight": "attn_k.weight", "self_attn.v_proj.weight": "attn_v.weight",
        "self_attn.q_norm.weight": "attn_q_norm.weight", "self_attn.k_norm.weight": "attn_k_norm.weight",
        "self_attn.o_proj.weight": "attn_output.weight",
        "post_attention_layernorm.weight": "post_attention_norm.weight",
        "pre_feedforward_layernorm.weight": "ffn_norm.weight", "mlp.gate_proj.weight": "ffn_gate.weight",
        "mlp.up_proj.weight": "ffn_up.weight", "mlp.down_proj.weight": "ffn_down.weight",
        "post_feedforward_layernorm.weight": "post_ffw_norm.weight", "layer_scalar": "layer_output_scale.weight",
        "per_layer_input_gate.weight": "inp_gate.weight", "per_layer_projection.weight": "proj.weight",
        "post_per_layer_input_norm.weight": "post_norm.weight",
        "router.proj.weight": "ffn_gate_inp.weight", "router.scale": "ffn_gate_inp.scale",
        "router.per_expert_scale": "ffn_down_exps.scale", "experts.gate_up_proj": "ffn_gate_up_exps.weight",
        "experts.down_proj": "ffn_down_exps.weight", "post_feedforward_layernorm_1.weight": "post_ffw_norm_1.weight",
        "post_feedforward_layernorm_2.weight": "post_ffw_norm_2.weight",
        "pre_feedforward_layernorm_2.weight": "pre_ffw_norm_2.weight",
    }
    own = model.state_dict()
    for l in range(L):
        for ours_name, gguf_name in names.items():
            k, g = f"model.layers.{l}.{ours_name}", f"blk.{l}.{gguf_name}"
            if k in own and g in W:
                sd[k] = W[g].reshape(own[k].shape)
    unset = sorted(k for k in own if k not in sd and k != "lm_head.weight")
    if unset:
        raise RuntimeError(f"transformers parameters without a GGUF tensor: {unset}")
    model.load_state_dict(sd, strict=False)
    model.lm_head.weight = model.model.embed_tokens.weight
    return model


def run_case(name: str) -> dict:
    import torch
    cfg, img, prompt, n_new = pin_cases.build(name)
    model = transformers_model(cfg, img)
    ids_in = torch.tensor([[int(t) for t in prompt]])
    with torch.no_grad():
        gen = model.generate(ids_in, max_new_tokens=n_new, do_sample=False, output_scores=False,
                             return_dict_in_generate=True, pad_token_id=None, eos_token_id=None)
    ids = gen.sequences[0, len(prompt):].numpy().astype(np.int64)
    seq = [int(t) for t in prompt] + [int(t) for t in ids[:-1]]
    hs = {}
    hooks = [layer.register_forward_hook(
        lambda mod, args, out, l=l: hs.__setitem__(l, (out[0] if isinstance(out, tuple) else out).detach()))
        for l, layer in enumerate(model.model.layers)]
    try:
        with torch.no_grad():
            logits = model(torch.tensor([seq]), use_cache=False).logits[0].numpy()
    finally:
        for h in hooks:
            h.remove()
    P, T = len(prompt), len(seq)
    pos = np.array(sorted({0, T - 1} if name in pin_cases.FEW_POSITIONS else {0, P // 2, P - 1, T - 1}), np.int64)
    hidden = np.stack([np.stack([hs[l][0, p].numpy() for l in range(cfg.layers)]) for p in pos]).astype(np.float32)
    top_i = np.argsort(-logits, axis=1, kind="stable")[:, :TOPN]
    top_v = np.take_along_axis(logits, top_i, axis=1)
    steps = logits[P - 1:]
    srt = np.sort(steps, axis=1)
    if not np.array_equal(steps.argmax(1), ids):
        raise RuntimeError(f"{name}: teacher-forced argmax differs from generate()")
    import gguf
    import transformers
    return {
        "sha256": np.frombuffer(hashlib.sha256(np.asarray(img).tobytes()).digest(), np.uint8),
        "prompt": np.asarray(prompt, np.int64), "ids": ids, "margins": (srt[:, -1] - srt[:, -2]).astype(np.float32),
        "pos": pos, "hidden": hidden, "top_ids": top_i.astype(np.int32), "top_logits": top_v.astype(np.float32),
        "versions": np.array([f"transformers {transformers.__version__}", f"torch {torch.__version__}",
                              f"gguf {getattr(gguf, '__version__', 'unknown')}"]),
    }


def main():
    names = sys.argv[1:] or sorted(pin_cases.CASES)
    for name in names:
        out = run_case(name)
        path = os.path.join(HERE, f"pin_{name}.npz")
        np.savez_compressed(path, **out)
        print(f"{path}: ids {out['ids'].tolist()}  min margin {out['margins'].min():.3g}  "
              f"{os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()

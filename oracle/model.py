"""CPU ORACLE -- TEST INFRASTRUCTURE ONLY.

Token-by-token decode of a GGUF model with the reference's graphs, in numpy:

  * "moe"   -- the A4B layer (src/engine-a4b.js:424-463): qkv -> headprep ->
               attention -> o -> rmsacc3 -> router top-k -> dense gate/up GeGLU +
               expert-slot gate/up GeGLU -> dense down + slot-combined expert down
               -> a4btail (post norms, residual, layer scale, next input norm).
  * "dense" -- the E4B layer (src/engine.js:292-323 with the q4_0 / q6_K weights of
               this build; semantics NOTES/arch-spec.md 2.2): qkv -> headprep ->
               attention -> o -> residual -> pre-FFN norm -> gate/up GeGLU ->
               down -> residual -> [PLE gate GEMV * gelu * per-layer input ->
               PLE projection -> post norm -> residual] -> layer scale.  The
               per-layer inputs are prepared per token as in src/engine.js:282-290
               and kernels/pleprep.wgsl:15-46.

Embedding: q6_K row x sqrt(H) (kernels/q6k.wgsl MODE 0); LM head: tied q6_K
matvec + softcap 30 (q6k.wgsl MODE 1); greedy argmax, ties to the lowest index.
The KV caches are f16 with the reference's slot rules (sliding ring slot
pos % RING, global slot = running count).  Records every layer's hidden state,
the logits' top-2 margin and the greedy ids.
"""
from __future__ import annotations

import math

import numpy as np

from . import gguf_min
from . import ops

F32 = np.float32


class OracleModel:
    def __init__(self, src, ternary=None):
        """ternary: {layer: {"gu" | "down": (planes, scales)}}: those layers' experts
        in the ternary format (kernels/t2gu.wgsl, kernels/t2moedown.wgsl)."""
        self.ternary = ternary or {}
        self.g = gguf_min.open_gguf(src)
        kv = self.g.kv
        a = "gemma4."
        self.H = int(kv[a + "embedding_length"])
        self.L = int(kv[a + "block_count"])
        self.QH = int(kv[a + "attention.head_count"])
        kvh = kv[a + "attention.head_count_kv"]
        self.KVH = int(kvh[0] if isinstance(kvh, list) else kvh)
        self.HD = int(kv[a + "attention.key_length"])
        self.FF = int(kv[a + "feed_forward_length"])
        self.V = int(kv[a + "vocab_size"])
        self.eps = float(kv[a + "attention.layer_norm_rms_epsilon"])
        self.cap = float(kv[a + "final_logit_softcapping"])
        self.W = int(kv.get(a + "attention.sliding_window", 0))
        self.sliding = [bool(x) for x in kv.get(a + "attention.sliding_window_pattern", [False] * self.L)]
        self.slack = int(kv.get("e4b.ring_slack", 512))
        self.th_s = float(kv.get(a + "rope.freq_base_swa", 10000.0))
        self.th_g = float(kv.get(a + "rope.freq_base", 1000000.0))
        self.frac = float(kv.get(a + "rope.partial_rotary_factor", 0.25))
        self.PD = int(kv.get(a + "embedding_length_per_layer_input", 0))
        self.E = int(kv.get(a + "expert_count", 0))
        self.K = int(kv.get(a + "expert_used_count", 0))
        self.EF = int(kv.get(a + "expert_feed_forward_length", 0))
        self.keqv_g = bool(kv.get(a + "attention.k_eq_v_global", False))
        self.max_ctx = int(kv.get("e4b.max_ctx", 8192))
        self.moe = self.E > 0
        self.scoring = False        # accumulate attention mass of the counted (global) caches
        self.reset()

    # ---- per-layer geometry (same rules as the reference: src/engine-a4b.js:328-347)
    def keqv(self, l):
        return self.keqv_g and not self.sliding[l]

    def ring(self, l):
        return self.W + self.slack

    def angles(self, l):
        return self.HD // 2 if self.sliding[l] else int(math.floor(self.frac * self.HD / 2))

    def theta(self, l):
        return self.th_s if self.sliding[l] else self.th_g

    def t(self, name):
        return self.g.fetch(name)

    def cat(self, *names):
        """Row-concatenated weights of same-IN linears (cached: no per-step copy)."""
        if not hasattr(self, "_cat"):
            self._cat = {}
        if names not in self._cat:
            self._cat[names] = np.concatenate([self.t(n) for n in names])
        return self._cat[names]

    def f(self, name):
        return self.g.f32(name)

    def reset(self):
        self.kc, self.vc = [], []
        for l in range(self.L):
            n = self.ring(l) if self.sliding[l] else self.max_ctx
            dt = np.float16 if ops.STORE_F16 else F32
            self.kc.append(np.zeros((n, self.KVH, self.HD), dt))
            self.vc.append(np.zeros((n, self.KVH, self.HD), dt))
        self.kv_count = 0
        self.reset_scores()

    def reset_scores(self):
        self.scores = {l: np.zeros((self.QH, self.max_ctx), F32) for l in range(self.L) if not self.sliding[l]}

    # ---- one token
    def step(self, tok: int, pos: int, record: bool = False):
        H, eps = self.H, self.eps
        p = "blk.{}."
        x = ops.q6k_row(self.t("token_embd.weight"), tok, H, F32(math.sqrt(H)))
        h = x
        ple = None
        if self.PD:
            ple = self.ple_inputs(tok, x)
        hidden = []
        xn = ops.f16r(ops.rmsnorm(h, self.f("blk.0.attn_norm.weight"), eps))
        slot_g = self.kv_count
        for l in range(self.L):
            b = p.format(l)
            QH, KVH, HD = self.QH, self.KVH, self.HD
            keqv = self.keqv(l)
            rows = QH * HD + KVH * HD * (1 if keqv else 2)
            wqkv = self.cat(*([b + "attn_q.weight", b + "attn_k.weight"] + ([] if keqv else [b + "attn_v.weight"])))
            qkv = ops.q40mv(wqkv, xn, rows, H)
            q, k, v = ops.headprep(qkv, self.f(b + "attn_q_norm.weight"), self.f(b + "attn_k_norm.weight"),
                                   pos, QH, KVH, HD, self.angles(l), self.theta(l), eps, keqv)
            if self.sliding[l]:
                slot, cm = pos % self.ring(l), 1
            else:
                slot, cm = slot_g, 2
            self.kc[l][slot] = k
            self.vc[l][slot] = v
            att = ops.decode_attention(q, self.kc[l], self.vc[l], pos, KVH, self.W, self.ring(l), cm, slot_g + 1)
            if self.scoring and cm == 2:
                self.scores[l][:, :slot_g + 1] += ops.attention_mass(q, self.kc[l], slot_g + 1, KVH)
            t = ops.q40mv(self.t(b + "attn_output.weight"), att.reshape(-1), H, QH * HD)
            nxt = self.f(p.format(l + 1) + "attn_norm.weight") if l + 1 < self.L else None
            mul = float(self.f(b + "layer_output_scale.weight")[0])
            if self.moe:
                h, xn = self.moe_ffn(b, h, t, nxt, mul)
            else:
                h, xn = self.dense_ffn(b, l, h, t, nxt, mul, ple)
            hidden.append(h.copy())
        self.kv_count += 1
        xf = ops.rmsnorm(h, self.f("output_norm.weight"), eps)
        logits = ops.softcap(ops.q6k_matvec(self.t("token_embd.weight"), xf, self.V, H), self.cap)
        nxt_tok = ops.argmax_first(logits)
        if record:
            return nxt_tok, {"hidden": np.stack(hidden), "logits": logits, "final": xf}
        return nxt_tok, None

    def ple_inputs(self, tok, x0):
        """pleIn[l] = (rms(Wp.x0 * H^-1/2)_l * norm + q6k_row_l * sqrt(PD)) * sqrt(1/2)
        (src/engine.js:282-290; kernels/pleprep.wgsl:15-46)."""
        H, L, PD = self.H, self.L, self.PD
        proj = ops.q40mv(self.t("per_layer_model_proj.weight"), x0, L * PD, H) * F32(1.0 / math.sqrt(H))
        ident = ops.q6k_row(self.t("per_layer_token_embd.weight"), tok, L * PD, F32(math.sqrt(PD)))
        nw = self.f("per_layer_proj_norm.weight")
        out = np.empty((L, PD), F32)
        for l in range(L):
            blk = proj[l * PD:(l + 1) * PD].astype(F32)
            out[l] = (blk * ops.rms_inv(blk, self.eps) * nw + ident[l * PD:(l + 1) * PD]) * F32(math.sqrt(0.5))
        return out

    def dense_ffn(self, b, l, h, t, nxt, mul, ple):
        H, FF, eps = self.H, self.FF, self.eps
        last_res = self.PD == 0
        h = ops.rmsacc(t, self.f(b + "post_attention_norm.weight"), h, eps)
        x2 = ops.f16r(ops.rmsnorm(h, self.f(b + "ffn_norm.weight"), eps))
        wgu = self.cat(b + "ffn_gate.weight", b + "ffn_up.weight")
        g = ops.geglu_rows(ops.q40mv(wgu, x2, 2 * FF, H), FF)
        t = ops.q40mv(self.t(b + "ffn_down.weight"), g, H, FF)
        h = ops.rmsacc(t, self.f(b + "post_ffw_norm.weight"), h, eps, mul if last_res else 1.0)
        if self.PD:
            PD = self.PD
            pg = ops.q40mv(self.t(b + "inp_gate.weight"), ops.f16r(h), PD, H)
            pg = ops.f16r(ops.gelu_tanh(pg) * ple[l])
            t = ops.q40mv(self.t(b + "proj.weight"), pg, H, PD)
            h = ops.rmsacc(t, self.f(b + "post_norm.weight"), h, eps, mul)
        xn = ops.f16r(ops.rmsnorm(h, nxt, eps)) if nxt is not None else None
        return h, xn

    def moe_ffn(self, b, h, t, nxt, mul):
        H, FF, EF, E, K, eps = self.H, self.FF, self.EF, self.E, self.K, self.eps
        rs = (self.f(b + "ffn_gate_inp.scale").astype(np.float64) * (1.0 / math.sqrt(H))).astype(F32)
        hB, normed, router_in, moe_in = ops.rmsacc3(t, self.f(b + "post_attention_norm.weight"),
                                                    self.f(b + "ffn_norm.weight"), rs,
                                                    self.f(b + "pre_ffw_norm_2.weight"), h, eps)
        wr = self.f(b + "ffn_gate_inp.weight").reshape(E, H)
        idx, w = ops.router_topk(router_in, wr, self.f(b + "ffn_down_exps.scale"), K)
        wgu = self.cat(b + "ffn_gate.weight", b + "ffn_up.weight")
        gd = ops.geglu_rows(ops.q40mv(wgu, normed, 2 * FF, H), FF)
        t2 = self.ternary.get(int(b.split(".")[1]))
        if t2 is not None:
            slots = ops.t2gu(moe_in, t2["gu"][0].reshape(-1), t2["gu"][1], idx, H, EF)
            t1 = ops.q40mv(self.t(b + "ffn_down.weight"), gd, H, FF)
            m = ops.t2moedown(slots, t2["down"][0].reshape(-1), t2["down"][1], idx, w, EF, H)
        else:
            gue = self.t(b + "ffn_gate_up_exps.weight")
            per = 2 * EF * H // 32 * 18
            slots = np.stack([ops.geglu_rows(ops.q40mv(gue[int(e) * per:(int(e) + 1) * per], moe_in, 2 * EF, H), EF)
                              for e in idx])
            t1 = ops.q40mv(self.t(b + "ffn_down.weight"), gd, H, FF)
            m = ops.moe_down(slots, self.t(b + "ffn_down_exps.weight"), idx, w, EF, H)
        wn = nxt if nxt is not None else self.f(b + "attn_norm.weight")
        h, xn = ops.a4btail(t1, self.f(b + "post_ffw_norm_1.weight"), m, self.f(b + "post_ffw_norm_2.weight"),
                            self.f(b + "post_ffw_norm.weight"), hB, wn, eps, mul, nxt is not None)
        self.last_topk = (idx, w)
        return h, xn

    # ---- long context (src/engine-a4b.js:589-657)
    def compact(self, budget, protect):
        """compactAll: every counted (global) cache keeps the slots
        ops.budget_keep picks from its accumulated scores, gathered to the front
        (kernels/kvgather.wgsl); scores reset; the count becomes the kept length."""
        n = self.kv_count
        kept = n
        for l, sc in self.scores.items():
            keep = ops.budget_keep(sc, n, budget, protect)
            self.kc[l][:len(keep)] = self.kc[l][keep]
            self.vc[l][:len(keep)] = self.vc[l][keep]
            kept = len(keep)
        self.reset_scores()
        self.kv_count = kept

    def generate_long(self, prompt, n_new, budget, decap, protect):
        """generateLong: prefill (no scores), a scored probe step and a
        compaction when the prompt exceeds `decap`, then decode in runs of 8
        with scores accumulating, recompacting whenever the count would pass
        `decap`.  Returns the greedy ids."""
        self.reset()
        self.scoring = False
        tok = None
        for pos, t in enumerate(prompt):
            tok, _ = self.step(int(t), pos)
        pos = len(prompt)
        ids = [tok]
        self.scoring = True
        if self.kv_count > decap:
            tok, _ = self.step(int(ids[-1]), pos)
            pos += 1
            ids.append(tok)
            self.compact(budget, protect)
        while len(ids) < n_new:
            if self.kv_count + 8 > decap:
                self.compact(budget, protect)
            for _ in range(min(8, n_new - len(ids))):
                tok, _ = self.step(int(ids[-1]), pos)
                pos += 1
                ids.append(tok)
        self.scoring = False
        return ids[:n_new]

    # ---- driver (src/engine-a4b.js:826-847 generateFast semantics)
    def generate(self, prompt, n_new, record=False):
        """Token-by-token prefill of `prompt`, then greedy decode; returns
        (ids, margins, records) with len(ids) == n_new."""
        self.reset()
        recs, ids, margins = [], [], []
        tok = None
        for pos, t in enumerate(prompt):
            tok, r = self.step(int(t), pos, record)
            if record:
                recs.append(r)
        pos = len(prompt)
        ids.append(tok)
        if record:
            margins.append(_margin(recs[-1]["logits"]))
        while len(ids) < n_new:
            tok, r = self.step(int(ids[-1]), pos, record)
            pos += 1
            ids.append(tok)
            if record:
                recs.append(r)
                margins.append(_margin(r["logits"]))
        return ids, margins, recs


def _margin(logits):
    top = np.partition(logits, -2)[-2:]
    return float(abs(top[1] - top[0]))

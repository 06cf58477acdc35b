"""Per-token decode engine (host side).

Mirrors the reference engines' public surface -- `loadEngineA4B()` /
`loadEngine()` returning {step, decodeChunk, generateFast, argmaxFast,
readHidden, ...} (src/engine-a4b.js:75-857, src/engine.js:10-485) -- on top of
the C-ABI kernels:

  load     GGUF -> config from kv (src/engine-a4b.js:100-116) -> every q4_0 /
           q6_K tensor uploaded UNCHANGED; same-IN linears (q|k|v, gate|up) are
           placed back to back in one allocation (byte concatenation, no repack).
  encode   one token's operator sequence (src/engine-a4b.js:424-463, 683-693 for
           "moe"; src/engine.js:282-337 for "dense" with q4_0 / q6_K weights).
  plan     the token sequence recorded once as a CUDA graph and replayed
           (src/engine-a4b.js:800-818); the token id, positions and the greedy
           token ring advance on the device (kernels/feedtok.wgsl), so a decode
           chunk is `count` graph launches with no host work in between.
"""
from __future__ import annotations

import ctypes
import math
from types import SimpleNamespace

import numpy as np

from . import gguf, ops
from .config import ModelConfig
from .device import Device

F32 = np.float32
RING_CAP = 16384        # greedy-token ring (src/engine-a4b.js:250 uses 1024)
ARGMAX_PARTS = 256
STATUS_EVERY = 32       # tokens between reads of the device status word in prefill / decode_chunk


class DeviceStatusError(RuntimeError):
    """A device-side check or bounded wait failed (the status word is nonzero)."""


class DenseLayer(ctypes.Structure):
    """e4b_dense_layer (include/e4b_b200.h)"""
    _fields_ = [(n, ctypes.c_void_p) for n in ("qkv", "o", "gu", "down", "ple_gate", "ple_proj", "attn_norm",
                                               "q_norm", "k_norm", "post_attn", "ffn_norm", "post_ffw",
                                               "post_norm")] + \
        [("scale", ctypes.c_float), ("theta", ctypes.c_float), ("kcache", ctypes.c_void_p),
         ("vcache", ctypes.c_void_p)] + \
        [(n, ctypes.c_int) for n in ("sliding", "ring", "slots", "rope_angles", "keqv", "qkv_rows")]


class DenseModel(ctypes.Structure):
    """e4b_dense_model (include/e4b_b200.h)"""
    _fields_ = [(n, ctypes.c_int) for n in ("layers", "hidden", "q_heads", "kv_heads", "head_dim", "ff", "vocab",
                                            "ple_dim", "window")] + \
        [("eps", ctypes.c_float)] + \
        [(n, ctypes.c_void_p) for n in ("token_embd", "ple_table", "ple_proj_w", "ple_norm", "out_norm")] + \
        [("layer", ctypes.POINTER(DenseLayer))] + \
        [(n, ctypes.c_void_p) for n in ("params", "hidden_out", "xf", "dump")]


def fused_supported(c: ModelConfig) -> bool:
    """Shapes the fused token kernel takes (e4b_dense_plan_create checks the same)."""
    return (not c.moe and c.hidden % 256 == 0 and c.hidden <= 4096 and c.q_dim % 256 == 0 and c.ff % 256 == 0
            and c.head_dim % 64 == 0 and (c.ple_dim == 0 or (c.ple_dim % 256 == 0 and c.ple_dim <= 4096)))


class Engine:
    def __init__(self, src, device: int | Device = 0, *, chunk: int = 64, record: bool = False,
                 fused: bool | None = None, kv_budget: int | None = None, kv_decap: int | None = None,
                 kv_protect: int = 64, ternary: dict | None = None):
        """fused: run each token's layers as one persistent kernel (dense graph
        only; None = whenever the model's shapes allow it).  kv_budget: long
        context with budget compaction of the counted (global) caches
        (src/engine-a4b.js:16-21, 589-657): every decode step accumulates the
        attention mass of their slots, compact_all() keeps kv_budget of them
        (the kv_protect most recent plus the highest mass), generate_long()
        recompacts whenever the count would pass kv_decap (default kv_budget +
        128).  Runs on the per-operator path.  ternary: the expert tensors in the
        ternary format ({layer: {"gu" | "down": (planes, scales)}}, from
        ternary.ternarize_model) decoded by e4b_t2gu / e4b_t2moedown
        (src/engine-a4b.js:338-340, 442-454)."""
        self.ternary = ternary
        self.kv_budget = kv_budget
        self.kv_decap = kv_decap if kv_decap is not None else (kv_budget + 128 if kv_budget else None)
        self.kv_protect = kv_protect
        self.kv_count = 0
        if kv_budget is not None:
            if fused:
                raise ValueError("budget compaction runs on the per-operator path (fused=False)")
            fused = False
            if not (0 < kv_protect <= kv_budget < self.kv_decap):
                raise ValueError(f"need 0 < kv_protect <= kv_budget < kv_decap ({kv_protect}, {kv_budget}, "
                                 f"{self.kv_decap})")
        self.g = gguf.open_gguf(src)
        self.cfg = ModelConfig.from_kv(self.g.kv)
        self.dev = device if isinstance(device, Device) else Device(device)
        self.own_dev = not isinstance(device, Device)
        self.chunk = chunk
        self.record = record
        self.plan = None
        self.plan_mode = None
        self.weight_bytes = 0
        if fused is None:
            fused = fused_supported(self.cfg)
        if fused and not fused_supported(self.cfg):
            raise ValueError(f"model {self.cfg.name!r} has shapes the fused token kernel does not take")
        self.fused = bool(fused)
        self.emb_tiles = None                # tile-packed LM head table (the batched engine makes its own)
        self._load_weights()
        self._alloc_activations()
        self.dense_plan = self._create_dense_plan() if self.fused else None
        # the fused path's LM head streams a tile-packed copy of the q6_K table
        # (one contiguous bulk copy per 16 rows x superblock; the warp-MMA GEMV)
        if self.fused:
            H, V = self.cfg.hidden, self.cfg.vocab
            self.emb_tiles = self.dev.alloc(int(self.dev.L.e4b_q6k_packed_bytes(H, V)), "lmHeadTiles")
            self.dev.call("e4b_q6k_pack_tiles", self.emb, self.emb_tiles, H, V)

    # ------------------------------------------------------------ loading
    def _raw(self, name: str):
        t = self.g.fetch(name)
        self.weight_bytes += t.nbytes
        return self.dev.upload(t, name)

    def _cat(self, names):
        """Upload same-IN linears back to back (rows concatenate in memory)."""
        parts = [self.g.fetch(n) for n in names]
        total = sum(p.nbytes for p in parts)
        buf = self.dev.alloc(total, "+".join(names), zero=False)
        off = 0
        for p in parts:
            self.dev.write(buf, p, off)
            off += p.nbytes
        self.weight_bytes += total
        return buf

    def _f32(self, name: str, scale: float | None = None):
        a = self.g.f32(name)
        if scale is not None:   # host fold, like the reference's router-scale fold (src/engine-a4b.js:174-179)
            a = (a.astype(np.float64) * scale).astype(F32)
        return self.dev.upload(np.ascontiguousarray(a, dtype=F32), name)

    def _load_weights(self):
        c = self.cfg
        H = c.hidden
        self.emb = self._raw("token_embd.weight")
        self.out_norm = self._f32("output_norm.weight")
        if c.ple_dim:
            self.ple_table = self._raw("per_layer_token_embd.weight")
            self.ple_proj_w = self._raw("per_layer_model_proj.weight")
            self.ple_norm = self._f32("per_layer_proj_norm.weight")
        self.layers = []
        for l in range(c.layers):
            p = f"blk.{l}."
            L = SimpleNamespace(i=l, sliding=c.is_sliding(l), keqv=c.keqv(l))
            L.attn_norm = self._f32(p + "attn_norm.weight")
            L.qkv = self._cat([p + "attn_q.weight", p + "attn_k.weight"] + ([] if L.keqv else [p + "attn_v.weight"]))
            L.qkv_rows = c.qkv_rows(l)
            L.q_norm = self._f32(p + "attn_q_norm.weight")
            L.k_norm = self._f32(p + "attn_k_norm.weight")
            L.o = self._raw(p + "attn_output.weight")
            L.post_attn = self._f32(p + "post_attention_norm.weight")
            L.ffn_norm = self._f32(p + "ffn_norm.weight")
            L.gu = self._cat([p + "ffn_gate.weight", p + "ffn_up.weight"])
            L.down = self._raw(p + "ffn_down.weight")
            L.post_ffw = self._f32(p + "post_ffw_norm.weight")
            L.scale = float(self.g.f32(p + "layer_output_scale.weight")[0])
            if c.ple_dim:
                L.inp_gate = self._raw(p + "inp_gate.weight")
                L.proj = self._raw(p + "proj.weight")
                L.post_norm = self._f32(p + "post_norm.weight")
            if c.moe:
                L.post_ffw1 = self._f32(p + "post_ffw_norm_1.weight")
                L.post_ffw2 = self._f32(p + "post_ffw_norm_2.weight")
                L.pre_ffw2 = self._f32(p + "pre_ffw_norm_2.weight")
                L.router_s = self._f32(p + "ffn_gate_inp.scale", 1.0 / math.sqrt(H))
                L.wr = self._f32(p + "ffn_gate_inp.weight")
                L.pes = self._f32(p + "ffn_down_exps.scale")
                L.gu_exps = self._raw(p + "ffn_gate_up_exps.weight")
                L.down_exps = self._raw(p + "ffn_down_exps.weight")
                t2 = (getattr(self, "ternary", None) or {}).get(l)
                if t2 is not None:
                    L.gu_t2 = self.dev.upload(np.ascontiguousarray(t2["gu"][0]), f"guT2_{l}")
                    L.gu_t2s = self.dev.upload(np.ascontiguousarray(t2["gu"][1]), f"guT2s_{l}")
                    L.down_t2 = self.dev.upload(np.ascontiguousarray(t2["down"][0]), f"downT2_{l}")
                    L.down_t2s = self.dev.upload(np.ascontiguousarray(t2["down"][1]), f"downT2s_{l}")
            L.angles = c.rope_angles(l)
            L.theta = c.theta(l)
            L.ring = c.ring(l)
            L.slots = c.kv_slots(l)
            L.cachemode = 1 if L.sliding else 2
            kvb = L.slots * c.kv_heads * c.head_dim * 2 * getattr(self, "nseq", 1)
            L.kc = self.dev.alloc(kvb, f"kcache{l}")
            L.vc = self.dev.alloc(kvb, f"vcache{l}")
            L.max_chunks = (L.slots + self.chunk - 1) // self.chunk
            self.layers.append(L)

    def _alloc_activations(self):
        c, d = self.cfg, self.dev
        H, FF, QD = c.hidden, c.ff, c.q_dim
        maxrows = max(c.qkv_rows(l) for l in range(c.layers))
        maxch = max(L.max_chunks for L in self.layers)
        A = SimpleNamespace()
        A.params = d.alloc(32, "params")
        A.hidden = d.alloc(H * 4, "hidden")
        A.hidden_b = d.alloc(H * 4, "hiddenB")
        A.normed = d.alloc(H * 2, "normed")
        A.qkv = d.alloc(maxrows * 4, "qkv")
        A.q = d.alloc(QD * 4, "qPrep")
        A.attn = d.alloc(QD * 2, "attnOut")
        A.part_o = d.alloc(c.q_heads * maxch * c.head_dim * 4, "partO")
        A.part_ml = d.alloc(c.q_heads * maxch * 2 * 4, "partML")
        A.tmp = d.alloc(H * 4, "tmp")
        A.geglu = d.alloc(FF * 2, "geglu")
        A.xf = d.alloc(H * 4, "xfinal")
        A.logits = d.alloc(c.vocab * 4, "logits")
        A.amax_part = d.alloc(ARGMAX_PARTS * 8, "amaxPart")
        A.amax = d.alloc(16, "amax")
        A.ring = d.alloc(RING_CAP * 4, "tokRing")
        if c.ple_dim:
            A.ple_proj = d.alloc(c.layers * c.ple_dim * 4, "pleProj")
            A.ple_in = d.alloc(c.layers * c.ple_dim * 4, "pleIn")
            A.hraw = d.alloc(H * 2, "hraw")
            A.ple_g = d.alloc(c.ple_dim * 2, "pleGate")
        if c.moe:
            A.router_in = d.alloc(H * 4, "routerIn")
            A.moe_in = d.alloc(H * 2, "moeIn")
            A.topk_idx = d.alloc(c.topk * 4, "topkIdx")
            A.topk_w = d.alloc(c.topk * 4, "topkW")
            A.geglu_slots = d.alloc(c.topk * c.expert_ff * 2, "gegluSlots")
            A.moe_out = d.alloc(H * 4, "moeOut")
        if self.record:
            A.dump = d.alloc(c.layers * H * 4, "hiddenDump")
        if self.kv_budget is not None:
            A.lse = d.alloc(c.q_heads * 4, "lse")
            glob = [L for L in self.layers if L.cachemode == 2]
            smax = max([L.slots for L in glob], default=1)
            A.keep = d.alloc(smax * 4, "kvKeep")
            A.kscr = d.alloc(smax * c.kv_heads * c.head_dim * 2, "kvScratchK")
            A.vscr = d.alloc(smax * c.kv_heads * c.head_dim * 2, "kvScratchV")
            for L in glob:
                L.score = d.alloc(c.q_heads * L.slots * 4, f"score{L.i}")
        self.A = A
        ws = int(d.L.e4b_workspace_bytes())
        A.ws = d.alloc(ws, "workspace")
        d.call("e4b_set_workspace", A.ws.ptr, ctypes.c_size_t(ws))
        # pinned per-step parameter slots (host -> device copies stay async)
        self.host_params_n = 8192
        p = ctypes.c_void_p()
        d.call("e4b_host_alloc", ctypes.c_size_t(self.host_params_n * 32), ctypes.byref(p))
        self.host_params = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint32)),
                                                 shape=(self.host_params_n, 8))
        self._host_params_ptr = p.value
        self._hp_next = 0
        p2 = ctypes.c_void_p()
        d.call("e4b_host_alloc", ctypes.c_size_t(64), ctypes.byref(p2))
        self.host_tok = np.ctypeslib.as_array(ctypes.cast(p2, ctypes.POINTER(ctypes.c_uint32)), shape=(16,))
        self._host_tok_ptr = p2.value

    def _create_dense_plan(self) -> int:
        """Describe the dense model to e4b_dense_plan_create (fused token kernel)."""
        c, A = self.cfg, self.A
        lay = (DenseLayer * c.layers)()
        for L in self.layers:
            e = lay[L.i]
            e.qkv, e.o, e.gu, e.down = L.qkv.ptr, L.o.ptr, L.gu.ptr, L.down.ptr
            if c.ple_dim:
                e.ple_gate, e.ple_proj, e.post_norm = L.inp_gate.ptr, L.proj.ptr, L.post_norm.ptr
            e.attn_norm, e.q_norm, e.k_norm = L.attn_norm.ptr, L.q_norm.ptr, L.k_norm.ptr
            e.post_attn, e.ffn_norm, e.post_ffw = L.post_attn.ptr, L.ffn_norm.ptr, L.post_ffw.ptr
            e.scale, e.theta = L.scale, L.theta
            e.kcache, e.vcache = L.kc.ptr, L.vc.ptr
            e.sliding, e.ring, e.slots = int(L.sliding), L.ring, L.slots
            e.rope_angles, e.keqv, e.qkv_rows = L.angles, int(L.keqv), L.qkv_rows
        m = DenseModel()
        m.layers, m.hidden, m.q_heads, m.kv_heads = c.layers, c.hidden, c.q_heads, c.kv_heads
        m.head_dim, m.ff, m.vocab, m.ple_dim, m.window = c.head_dim, c.ff, c.vocab, c.ple_dim, c.window
        m.eps = c.eps
        m.token_embd, m.out_norm = self.emb.ptr, self.out_norm.ptr
        if c.ple_dim:
            m.ple_table, m.ple_proj_w, m.ple_norm = self.ple_table.ptr, self.ple_proj_w.ptr, self.ple_norm.ptr
        m.layer = lay
        m.params, m.hidden_out, m.xf = A.params.ptr, A.hidden.ptr, A.xf.ptr
        m.dump = A.dump.ptr if self.record else None
        h = ctypes.c_int()
        self.dev.call("e4b_dense_plan_create", ctypes.byref(m), ctypes.byref(h))
        return h.value

    # ------------------------------------------------------------ one token
    def encode_forward(self):
        """Enqueue one token (src/engine-a4b.js:683-693)."""
        c, d, A = self.cfg, self.dev, self.A
        H, V = c.hidden, c.vocab
        if self.fused:
            d.call("e4b_dense_plan_run", self.dense_plan)
            d.call("e4b_q6k_lmhead_tiles", self.emb_tiles, A.xf, None, A.logits, H, V, ctypes.c_float(c.softcap), 1)
            ops.argmax(d, A.logits, A.amax_part, A.amax, N=V, PARTS=ARGMAX_PARTS)
            ops.feedtok(d, A.amax, A.params, A.ring, RING_CAP=RING_CAP)
            return
        ops.q6k_embed(d, self.emb, A.params, None, A.hidden, N=H, ROWS=V, MULT=float(F32(math.sqrt(H))))
        if c.ple_dim:
            L, PD = c.layers, c.ple_dim
            ops.q40mv(d, A.hidden, self.ple_proj_w, None, A.ple_proj, IN=H, OUT=L * PD, XF16=0)
            ops.pleprep(d, self.ple_table, A.params, None, A.ple_proj, self.ple_norm, A.ple_in, PD=PD, LAYERS=L,
                        ROWS=V, MULT=float(F32(math.sqrt(PD))), PROJ_SCALE=float(F32(1.0 / math.sqrt(H))), EPS=c.eps)
        ops.rmsnorm(d, A.hidden, self.layers[0].attn_norm, None, None, A.normed, DIM=H, EPS=c.eps, F16OUT=1)
        for L in self.layers:
            self._encode_attention(L)
            if c.moe:
                self._encode_moe_ffn(L)
            else:
                self._encode_dense_ffn(L)
            if self.record:
                d.call("e4b_copy", A.dump.at(L.i * H * 4), A.hidden.ptr, ctypes.c_size_t(H * 4))
        ops.rmsnorm(d, A.hidden, self.out_norm, A.xf, None, None, DIM=H, EPS=c.eps, F16OUT=0)
        ops.q6k_lmhead(d, self.emb, A.xf, A.logits, N=H, OUT=V, SOFTCAP=c.softcap)
        ops.argmax(d, A.logits, A.amax_part, A.amax, N=V, PARTS=ARGMAX_PARTS)
        ops.feedtok(d, A.amax, A.params, A.ring, RING_CAP=RING_CAP)

    def _encode_attention(self, L):
        c, d, A = self.cfg, self.dev, self.A
        H = c.hidden
        ops.q40mv(d, A.normed, L.qkv, None, A.qkv, IN=H, OUT=L.qkv_rows, XF16=1)
        ops.headprep(d, A.qkv, L.q_norm, L.k_norm, A.params, L.kc, L.vc, A.q, QH=c.q_heads, KVH=c.kv_heads,
                     HEAD_DIM=c.head_dim, ROPE_ANGLES=L.angles, THETA=L.theta, EPS=c.eps, KEQV=int(L.keqv),
                     CACHEMODE=L.cachemode, RING=L.ring, SLOTS=L.slots)
        ops.attsplit(d, A.q, L.kc, L.vc, A.params, A.part_o, A.part_ml, Q_HEADS=c.q_heads, KV_HEADS=c.kv_heads,
                     HEAD_DIM=c.head_dim, WINDOW=c.window if L.sliding else 0, CACHEMODE=L.cachemode, RING=L.ring,
                     CS=self.chunk, CHUNKS=L.max_chunks)
        scoring = self.kv_budget is not None and L.cachemode == 2
        ops.attcomb(d, A.part_o, A.part_ml, A.attn, None, A.lse if scoring else None, Q_HEADS=c.q_heads,
                    HEAD_DIM=c.head_dim, CHUNKS=L.max_chunks)
        if scoring:      # the mass pass of kernels/attnos.wgsl:82-97 (SCORE=1 on global layers)
            d.call("e4b_attn_score", A.q, L.kc, A.lse, A.params, L.score, c.q_heads, c.kv_heads, c.head_dim,
                   ctypes.c_float(1.0), L.slots)
        ops.q40mv(d, A.attn, L.o, None, A.tmp, IN=c.q_dim, OUT=H, XF16=1)

    def _next_norm(self, L):
        return self.layers[L.i + 1].attn_norm if L.i + 1 < self.cfg.layers else None

    def _encode_dense_ffn(self, L):
        """src/engine.js:308-322 (post-attn residual, pre-FFN norm, GeGLU FFN, PLE block)."""
        c, d, A = self.cfg, self.dev, self.A
        H, FF = c.hidden, c.ff
        ops.rmsaccn(d, A.tmp, L.post_attn, A.hidden, L.ffn_norm, A.normed, DIM=H, EPS=c.eps, MUL=1.0, NORM2=1)
        ops.q40gu(d, None, None, None, None, A.normed, L.gu, A.geglu, IN=H, FF=0, FF2=FF, K=0)
        ops.q40mv(d, A.geglu, L.down, None, A.tmp, IN=FF, OUT=H, XF16=1)
        nxt = self._next_norm(L)
        if c.ple_dim:
            PD = c.ple_dim
            ops.rmsaccn(d, A.tmp, L.post_ffw, A.hidden, None, A.hraw, DIM=H, EPS=c.eps, MUL=1.0, NORM2=0)
            ops.plegatemv(d, A.hraw, L.inp_gate, A.ple_in, A.ple_g, IN=H, OUT=PD, OFF=L.i * PD)
            ops.q40mv(d, A.ple_g, L.proj, None, A.tmp, IN=PD, OUT=H, XF16=1)
            last_w = L.post_norm
        else:
            last_w = L.post_ffw
        if nxt is not None:
            ops.rmsaccn(d, A.tmp, last_w, A.hidden, nxt, A.normed, DIM=H, EPS=c.eps, MUL=L.scale, NORM2=1)
        else:
            ops.rmsacc(d, A.tmp, last_w, A.hidden, DIM=H, EPS=c.eps, MUL=L.scale)

    def _encode_moe_ffn(self, L):
        """src/engine-a4b.js:437-462."""
        c, d, A = self.cfg, self.dev, self.A
        H, FF, EF, K = c.hidden, c.ff, c.expert_ff, c.topk
        ops.rmsacc3(d, A.tmp, L.post_attn, L.ffn_norm, L.router_s, L.pre_ffw2, A.hidden, A.normed, A.router_in,
                    A.moe_in, A.hidden_b, DIM=H, EPS=c.eps)
        ops.routertop(d, A.router_in, L.wr, L.pes, A.topk_idx, A.topk_w, H=H, E=c.experts, K=K)
        if getattr(L, "gu_t2", None) is not None:
            # ternary experts (src/engine-a4b.js:442-454): dense branch q4_0, expert slots t2
            ops.q40gu(d, None, None, None, None, A.normed, L.gu, A.geglu, IN=H, FF=0, FF2=FF, K=0)
            d.call("e4b_t2gu", A.moe_in, L.gu_t2, L.gu_t2s, A.topk_idx, A.geglu_slots, H, EF, K, c.experts)
            ops.q40mv(d, A.geglu, L.down, None, A.tmp, IN=FF, OUT=H, XF16=1)
            d.call("e4b_t2moedown", A.geglu_slots, L.down_t2, L.down_t2s, A.topk_idx, A.topk_w, A.moe_out, EF, H, K,
                   c.experts)
        else:
            ops.q40gu(d, A.moe_in, L.gu_exps, A.topk_idx, A.geglu_slots, A.normed, L.gu, A.geglu, IN=H, FF=EF,
                      FF2=FF, K=K)
            ops.q40mv(d, A.geglu, L.down, None, A.tmp, IN=FF, OUT=H, XF16=1)
            ops.q40moedown(d, A.geglu_slots, L.down_exps, A.topk_idx, A.topk_w, A.moe_out, IN=EF, OUT=H, K=K)
        nxt = self._next_norm(L)
        ops.a4btail(d, A.tmp, L.post_ffw1, A.moe_out, L.post_ffw2, L.post_ffw, A.hidden_b,
                    nxt if nxt is not None else L.attn_norm, A.normed, A.hidden, H=H, EPS=c.eps, MUL=L.scale,
                    NEXT=int(nxt is not None))

    # ------------------------------------------------------------ plan
    def build_plan(self):
        """Record encode_forward() once as a replayable CUDA graph.  If the
        driver refuses to record the fused (cooperative) kernel into a graph,
        tokens are enqueued kernel by kernel instead (plan_mode "direct")."""
        if self.plan_mode is None:
            n0 = self.dev.kernel_launches
            self.dev.call("e4b_plan_begin")
            err = None
            try:
                self.encode_forward()
            except Exception as e:      # recorded below; capture must still be ended
                err = e
            p = ctypes.c_int()
            try:
                self.dev.call("e4b_plan_end", ctypes.byref(p))
            except Exception as e:
                err = err or e
            self.kernels_per_token = self.dev.kernel_launches - n0
            if err is None:
                self.plan, self.plan_mode = p.value, "graph"
            elif self.fused:
                self.plan_mode, self.plan_error = "direct", str(err)
                self.dev.sync()
            else:
                raise err
        return self.plan

    def run_token(self, count: int = 1):
        """Enqueue `count` tokens (graph replays, or direct launches)."""
        self.build_plan()
        if self.plan_mode == "graph":
            self.dev.call("e4b_plan_launch", self.plan, count)
        else:
            for _ in range(count):
                self.encode_forward()

    # ------------------------------------------------------------ host API
    def set_params(self, token: int, pos: int, ring_index: int | None = None, sync_slot: bool = False,
                   kv: int | None = None):
        """Queue [pos, pos+1, token, 0, kvCount, kvCount+1, ringIndex, 0] (src/engine-a4b.js:697-698);
        kvCount = pos unless given (budget compaction decouples the two)."""
        if self._hp_next >= self.host_params_n:
            self.dev.sync()
            self._hp_next = 0
        i = self._hp_next
        self._hp_next += 1
        ri = pos if ring_index is None else ring_index
        kc = pos if kv is None else kv
        self.host_params[i] = (pos, pos + 1, token, 0, kc, kc + 1, ri, 0)
        self.dev.call("e4b_upload_async", self.A.params.ptr, ctypes.c_void_p(self._host_params_ptr + i * 32),
                      ctypes.c_size_t(32))

    def step(self, token: int, pos: int):
        """One token at `pos` (src/engine-a4b.js:695-705); the result stays on the device."""
        if self.kv_budget is not None:
            self.set_params(token, pos, kv=self.kv_count)
            self.kv_count += 1
        else:
            self.set_params(token, pos)
        self.run_token(1)

    def argmax_fast(self) -> int:
        """src/engine-a4b.js:781-784"""
        return int(self.dev.read(self.A.amax, np.uint32, 1)[0])

    def check_status(self, where: str):
        """Read (and clear) the device status word; raise if a device-side check
        or a bounded wait failed since the last read, so a failing kernel stops
        the run at once instead of being relaunched for every later token."""
        st = self.dev.status()
        if st:
            raise DeviceStatusError(f"{where}: device status word {st:#x} "
                                    "(1 = index out of range, 2 = a bounded device wait timed out)")

    # ------------------------------------------------------------ long context
    def reset_scores(self):
        for L in self.layers:
            if getattr(L, "score", None) is not None:
                self.dev.memset(L.score, 0)

    def compact_all(self):
        """compactAll (src/engine-a4b.js:589-617): per counted (global) cache,
        mass[t] = sum over heads of the accumulated scores; keep the kv_protect
        most recent slots and the highest-mass others up to kv_budget (ties:
        lower slot), ascending; gather them to the front (e4b_kvgather through
        scratch, kernels/kvgather.wgsl); reset the scores; the count and the
        device parameters' kvCount become the kept length."""
        if self.kv_budget is None:
            raise RuntimeError("compact_all needs an Engine built with kv_budget")
        c, d, A = self.cfg, self.dev, self.A
        d.sync()
        n = self.kv_count
        kept = n
        row = c.kv_heads * c.head_dim * 2
        for L in self.layers:
            if getattr(L, "score", None) is None:
                continue
            sc = d.read(L.score, F32, c.q_heads * L.slots).reshape(c.q_heads, L.slots)
            mass = sc[:, :n].astype(np.float64).sum(axis=0)
            prot = min(self.kv_protect, n)
            cand = np.argsort(-mass[:n - prot], kind="stable")
            keep = np.sort(np.concatenate([cand[:max(self.kv_budget - prot, 0)],
                                           np.arange(n - prot, n)])).astype(np.uint32)
            d.write(A.keep, keep)
            d.call("e4b_kvgather", A.keep, len(keep), L.kc, L.vc, A.kscr, A.vscr, c.kv_heads, c.head_dim, L.slots)
            d.call("e4b_copy", ctypes.c_void_p(L.kc.ptr), ctypes.c_void_p(A.kscr.ptr), ctypes.c_size_t(len(keep) * row))
            d.call("e4b_copy", ctypes.c_void_p(L.vc.ptr), ctypes.c_void_p(A.vscr.ptr), ctypes.c_size_t(len(keep) * row))
            d.memset(L.score, 0)
            kept = len(keep)
        self.kv_count = kept
        p = d.read(A.params, np.uint32, 8)
        p[4], p[5] = kept, kept + 1
        d.write(A.params, p)
        self.check_status("compact_all")

    def generate_long(self, prompt, n_new: int, eos=None):
        """generateLong (src/engine-a4b.js:622-657): prefill; if the prompt
        exceeds kv_decap, one scored probe step then a compaction; then greedy
        decode in runs of 8 tokens with scores accumulating, recompacting when
        the count would pass kv_decap.  Returns n_new ids (cut at eos)."""
        if self.kv_budget is None:
            raise RuntimeError("generate_long needs an Engine built with kv_budget")
        self.kv_count = 0
        P = len(prompt)
        assert P >= 1 and P + n_new <= RING_CAP
        self.prefill(prompt)
        self.reset_scores()                 # the reference's prefill does not score
        done = 1
        if self.kv_count > self.kv_decap:
            self.decode_chunk(1)            # probe: scored step on the full cache
            self.kv_count += 1
            done = 2
            self.compact_all()
        while done < n_new:
            if self.kv_count + 8 > self.kv_decap:
                self.compact_all()
            n = min(8, n_new - done)
            self.decode_chunk(n)
            self.kv_count += n
            done += n
        self.dev.sync()
        ids = [int(x) for x in self.read_ring(P - 1, n_new)]
        if eos:
            for i, t in enumerate(ids):
                if t in eos:
                    return ids[:i + 1]
        return ids

    def decode_chunk(self, count: int, check_every: int = STATUS_EVERY):
        """`count` greedy tokens continuing from the device-side parameters
        (src/engine-a4b.js:786-823); the status word is read every
        `check_every` tokens (0: only by the caller)."""
        step = count if check_every <= 0 else check_every
        done = 0
        while done < count:
            n = min(step, count - done)
            self.run_token(n)
            done += n
            if check_every > 0:
                self.check_status(f"decode_chunk (token {done} of {count})")

    def read_ring(self, start: int, n: int) -> np.ndarray:
        return self.dev.read(self.A.ring, np.uint32, n, offset=start * 4)

    def read_hidden(self) -> np.ndarray:
        """src/engine-a4b.js:850-852"""
        return self.dev.read(self.A.hidden, F32, self.cfg.hidden)

    def read_dump(self) -> np.ndarray:
        assert self.record
        return self.dev.read(self.A.dump, F32, self.cfg.layers * self.cfg.hidden).reshape(self.cfg.layers, -1)

    def read_logits(self) -> np.ndarray:
        return self.dev.read(self.A.logits, F32, self.cfg.vocab)

    def prefill(self, prompt):
        """Token-by-token prefill (the reference's generateFast path, src/engine-a4b.js:828)."""
        if self._hp_next:
            self.dev.sync()          # pinned parameter slots are reused from the start
            self._hp_next = 0
        for pos, t in enumerate(prompt):
            self.step(int(t), pos)
            if (pos + 1) % STATUS_EVERY == 0 or pos + 1 == len(prompt):
                self.check_status(f"prefill (position {pos})")

    def generate(self, prompt, n_new: int, eos=None):
        """generateFast (src/engine-a4b.js:826-847): prefill, then greedy decode
        with the token id fed back on the device; returns n_new ids (cut at eos)."""
        P = len(prompt)
        assert P >= 1 and P + n_new <= RING_CAP
        self.prefill(prompt)
        if n_new > 1:
            self.decode_chunk(n_new - 1)
        self.dev.sync()
        ids = [int(x) for x in self.read_ring(P - 1, n_new)]
        if eos:
            for i, t in enumerate(ids):
                if t in eos:
                    return ids[:i + 1]
        return ids

    def close(self):
        if self.dense_plan is not None:
            self.dev.call("e4b_dense_plan_destroy", self.dense_plan)
            self.dense_plan = None
        if self.own_dev:
            self.dev.close()

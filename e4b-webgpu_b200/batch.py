"""Batched decode of B sequences in lockstep (benchmark configs 4/5: A4B-shaped
MoE at batch 1/16/64).

All B sequences share the position block (same prompt length, one token per
step each); every sequence has its own KV cache region.  Per layer
(src/engine-a4b.js:424-463 per token, batched as the reference's grouped path
src/engine-a4b.js:467-585 does for prefill):

  q|k|v        e4b_q40mm          (tensor-core GEMM, tokens as columns)
  head prep    e4b_headprep_seq   (per-sequence cache)
  attention    e4b_attdec_seq     (split-KV on the tensor cores + combine)
  o            e4b_q40mm
  norms        e4b_rmsacc3        (rows = B)
  router       e4b_routertop      (batch = B)
  dense FFN    e4b_q40gumm + e4b_q40mm
  experts      e4b_expgroup -> e4b_q40gugrp -> e4b_q40downgrp
  tail         e4b_a4btail_wacc   (expert combine + a4btail, rows = B)

Every f16 activation that feeds a q4_0 GEMM (normed rows, attention output,
MoE input, GeGLU outputs) is kept in fragment order (xfo_perm), written so
by its producer.

then the final norm, e4b_q6k_lmhead_tiles (on a tile-packed copy of the
q6_K embedding), e4b_argmax_rows and
e4b_feedtok_rows (each sequence's greedy token fed back on the device).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np

from . import ops
from .engine import Engine, RING_CAP, ARGMAX_PARTS, F32, STATUS_EVERY

C = ctypes.c_void_p


def xfo_perm(n: int) -> np.ndarray:
    """Fragment order of an f16 activation row of n elements (n % 32 == 0):
    element i is stored at half xfo_perm(n)[i].  Inside each 32-element block
    the 8 values MMA lane t reads (indices 4t..4t+3 in odd blocks, 2+4t..5+4t or
    {0, 1, 14, 15} for t = 3 in even blocks, and the same + 16) are contiguous
    at halves 8t..8t+7 in the order [j0, j2, j1, j3, j0+16, j2+16, j1+16, j3+16]."""
    assert n % 32 == 0
    pos = np.empty(n, np.int64)
    for i in range(n):
        b, j = divmod(i, 32)
        hi, jj = divmod(j, 16)
        if b & 1:
            t, r = divmod(jj, 4)
        elif 2 <= jj < 14:
            t, r = divmod(jj - 2, 4)
        else:
            t, r = 3, (jj if jj < 2 else jj - 12)
        slot = {0: 0, 1: 2, 2: 1, 3: 3}[r]
        pos[i] = 32 * b + 8 * t + 4 * hi + slot
    return pos


def nccl_unique_id(dev) -> bytes:
    """A fresh NCCL unique id (128 bytes) for an expert-parallel group."""
    buf = (ctypes.c_uint8 * 128)()
    rc = dev.L.e4b_nccl_unique_id(ctypes.cast(buf, ctypes.c_void_p))
    if rc != 0:
        raise RuntimeError(f"e4b_nccl_unique_id failed ({rc})")
    return bytes(buf)


def argmax_parts(rows: int) -> int:
    """Stage-0 partials per row of e4b_argmax_rows: about 4096 CTAs in all, so
    a batch's rows give each CTA a few thousand logits (at most ARGMAX_PARTS
    per row, the size of the partial buffers)."""
    return max(1, min(ARGMAX_PARTS, 4096 // max(1, rows)))


def to_xfo(x: np.ndarray) -> np.ndarray:
    """Rows of x (last axis) permuted into fragment order."""
    out = np.empty_like(x)
    out[..., xfo_perm(x.shape[-1])] = x
    return out


def from_xfo(x: np.ndarray) -> np.ndarray:
    return x[..., xfo_perm(x.shape[-1])]


class BatchEngine(Engine):
    def __init__(self, src, nseq: int, device=0, *, chunk: int = 64, ep=None, zipf: float | None = None,
                 tok0: int = 0, route_seed: int = 1234, ep_overlap: bool = True, ep_transport: str = "nccl",
                 overlap_route: bool = True):
        """nseq sequences decoded in lockstep on this GPU.  ep = (nranks, rank,
        nccl_id): expert parallelism -- this rank decodes its nseq sequences and
        owns experts [rank*E/nranks, (rank+1)*E/nranks); every rank of the
        communicator must build its engine with the same nccl_id (from
        e4b_nccl_unique_id on one rank).  zipf = s: benchmark routing -- each
        layer's experts are drawn from a seeded Zipf(s) popularity instead of
        the router's top-K (benchmark config 5); tok0 = this rank's first global
        sequence, so any rank count routes identically.  ep_transport: "nccl"
        (grouped send/recv of the slabs) or "p2p" (rows and results stored
        straight into the peers' slabs through CUDA IPC mappings, device-side
        epoch flags; 2 or more ranks, one process per GPU).  overlap_route (one
        GPU): each layer's routing chain (router, Zipf draw, expert sort) runs
        on a side stream concurrently with the dense FFN."""
        if ep_transport not in ("nccl", "p2p"):
            raise ValueError(f"ep_transport {ep_transport!r}: 'nccl' or 'p2p'")
        self.ep_transport = ep_transport
        self._ipc_open = []
        self.nseq = int(nseq)
        self.zipf, self.tok0, self.route_seed = zipf, int(tok0), int(route_seed)
        self.ep_overlap = bool(ep_overlap)     # row exchange on a side stream beside the dense FFN
        self.overlap_route = bool(overlap_route)   # routing chain on a side stream beside the dense FFN
        self.ep = None
        if ep is not None:
            nranks, rank, nid = ep
            self.ep = (int(nranks), int(rank), bytes(nid))
        super().__init__(src, device, chunk=chunk, record=False, fused=False)
        if not self.cfg.moe:
            raise ValueError("BatchEngine drives the MoE (A4B) graph")
        if self.chunk > 64:
            raise ValueError("BatchEngine's attention partials are sized for 64-slot chunks (chunk <= 64)")
        H, IN = self.cfg.hidden, self.cfg.hidden
        for n, what in ((H, "hidden"), (self.cfg.q_dim, "q_dim"), (self.cfg.ff, "ff"), (self.cfg.expert_ff, "expert ff")):
            if n % 64:
                raise ValueError(f"{what} {n} must be a multiple of 64 for the batched GEMMs")

    def _alloc_activations(self):
        c, d, B = self.cfg, self.dev, self.nseq
        H, FF, QD, E, K, EF = c.hidden, c.ff, c.q_dim, c.experts, c.topk, c.expert_ff
        maxrows = max(c.qkv_rows(l) for l in range(c.layers))
        maxch = max(L.max_chunks for L in self.layers)
        A = type("Acts", (), {})()
        A.params = d.alloc(32, "params")
        A.tok = d.alloc(B * 4, "tok")
        A.hidden = d.alloc(B * H * 4, "hidden")
        A.hidden_b = d.alloc(B * H * 4, "hiddenB")
        A.normed = d.alloc(B * H * 2, "normed")
        # the dense q|k|v and o GEMMs split K over CTA groups when the batch is
        # large enough to share each weight decode (partials summed by the consumer)
        def kparts(n_in, rows):
            # as many K-parts as keep (K-part x 8-tile group) items within one wave of CTAs
            if not (8 <= B <= 64 and n_in % 256 == 0):
                return 1
            groups = -(-rows // 256)
            return max(1, min(n_in // 256, d.sm_count // groups))
        self.kp_qkv = kparts(H, maxrows)
        self.kp_o = kparts(c.q_dim, H)
        A.qkv = d.alloc(self.kp_qkv * B * maxrows * 4, "qkv")
        A.oparts = d.alloc(self.kp_o * B * H * 4, "oParts")
        A.q = d.alloc(B * QD * 4, "qPrep")
        A.attn = d.alloc(B * QD * 2, "attnOut")
        A.part_o = d.alloc(B * c.q_heads * maxch * c.head_dim * 4, "partO")
        A.part_ml = d.alloc(B * c.q_heads * maxch * 2 * 4, "partML")
        A.tmp = d.alloc(B * H * 4, "tmp")
        A.geglu = d.alloc(B * FF * 2, "geglu")
        A.router_in = d.alloc(B * H * 4, "routerIn")
        A.moe_in = d.alloc(B * H * 2, "moeIn")
        A.topk_idx = d.alloc(B * K * 4, "topkIdx")
        A.topk_w = d.alloc(B * K * 4, "topkW")
        A.offsets = d.alloc((E + 1) * 4, "expOffsets")
        A.entries = d.alloc(B * K * 4, "expEntries")
        A.inv = d.alloc(B * K * 4, "expInv")
        # a second expert grouping: under benchmark routing the next layer's
        # grouping is formed on the side stream while this layer uses the other
        A.offsets1 = d.alloc((E + 1) * 4, "expOffsets1")
        A.entries1 = d.alloc(B * K * 4, "expEntries1")
        A.inv1 = d.alloc(B * K * 4, "expInv1")
        A.gl = d.alloc(B * K * EF * 2, "expGeglu")
        A.yo = d.alloc(B * K * H * 4, "expOut")
        A.moe_out = d.alloc(B * H * 4, "moeOut")
        A.xf = d.alloc(B * H * 4, "xfinal")
        A.xsplit = d.alloc(2 * max(64, (B + 7) // 8 * 8) * H * 2, "xSplit")
        A.logits = d.alloc(B * c.vocab * 4, "logits")
        A.amax_part = d.alloc(B * ARGMAX_PARTS * 8, "amaxPart")
        A.amax = d.alloc(B * 8, "amax")
        A.ring = d.alloc(B * RING_CAP * 4, "tokRing")
        # the LM head streams a tile-packed copy of the (tied) q6_K embedding: one
        # contiguous TMA copy per 128 rows x superblock (e4b_q6k_lmhead_tiles)
        self.emb_tiles = self._pack_lm_head(self.emb, c.vocab) if B <= 64 else None
        # tile-packed copies of the experts' gate|up weights, the largest weight
        # stream of a step (e4b_q40gugrp_tiles reads them with aligned 16-byte loads)
        self.gu_tiles = H % 256 == 0 and (2 * EF) % 16 == 0
        if self.gu_tiles:
            for L in self.layers:
                L.gu_exps_t = d.alloc(E * 2 * EF * (H // 32) * 18, "guExpsTiles")
                d.call("e4b_q40_pack_tiles", L.gu_exps, L.gu_exps_t, E * 2 * EF, H)
        self.emb_shard_tiles = None
        self.zipf_all = bool(self.zipf)
        if self.zipf_all:
            # benchmark routing of every layer drawn in one launch per step from a
            # popularity table built once
            A.zipf_table = d.alloc(2 * E * 4, "zipfTable")
            d.call("e4b_zipf_table", A.zipf_table, E, ctypes.c_float(self.zipf), ctypes.c_uint32(self.route_seed))
            A.ztop_idx = d.alloc(c.layers * B * K * 4, "zipfTopkAll")
            A.ztop_w = d.alloc(c.layers * B * K * 4, "zipfWAll")
        if self.ep is not None:
            self._alloc_ep(A)
        self.A = A
        ws = int(d.L.e4b_workspace_bytes())
        A.ws = d.alloc(ws, "workspace")
        d.call("e4b_set_workspace", A.ws.ptr, ctypes.c_size_t(ws))
        p = ctypes.c_void_p()
        d.call("e4b_host_alloc", ctypes.c_size_t(32), ctypes.byref(p))
        self.host_params = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_uint32)), shape=(8,))
        self._host_params_ptr = p.value

    def _alloc_ep(self, A):
        c, d, B = self.cfg, self.dev, self.nseq
        N, rank, nid = self.ep
        H, E, K, EF = c.hidden, c.experts, c.topk, c.expert_ff
        if E % N:
            raise ValueError(f"{E} experts do not split over {N} ranks")
        self.e_loc = E // N
        self.cap = B * K                       # every entry of this rank could go to one peer
        rows = N * self.cap
        if self.ep_transport == "nccl":          # the peer-memory transport stores rows and results directly
            A.ep_sx = d.alloc(rows * H * 2, "epSendX")
            A.ep_sy = d.alloc(rows * H * 4, "epSendY")
        A.ep_rx = d.alloc(rows * H * 2, "epRecvX")
        A.ep_sid = d.alloc(rows * 4, "epSendIds")
        A.ep_rid = d.alloc(rows * 4, "epRecvIds")
        A.ep_slot = d.alloc(B * K * 4, "epSlot")
        A.ep_off = d.alloc((self.e_loc + 1) * 4, "epOffsets")
        A.ep_ent = d.alloc(rows * 4, "epEntries")
        A.ep_inv = d.alloc(rows * 4, "epInv")
        A.ep_gl = d.alloc(rows * EF * 2, "epGeglu")
        A.ep_y = d.alloc(rows * H * 4, "epY")
        A.ep_ry = d.alloc(rows * H * 4, "epRecvY")
        idbuf = (ctypes.c_uint8 * 128).from_buffer_copy(nid)
        d.call("e4b_nccl_init", N, rank, ctypes.cast(idbuf, ctypes.c_void_p))
        if self.ep_transport == "p2p":
            self._map_peers(A, N, rank)
        # this rank's experts inside the full expert tensors
        per_gu = 2 * EF * (H // 32) * 18
        per_dn = H * (EF // 32) * 18
        for L in self.layers:
            L.gu_loc = ctypes.c_void_p((L.gu_exps_t if self.gu_tiles else L.gu_exps).ptr + rank * self.e_loc * per_gu)
            L.dn_loc = ctypes.c_void_p(L.down_exps.ptr + rank * self.e_loc * per_dn)
        # vocabulary-sharded LM head: this rank's V/N rows for every rank's tokens
        V = c.vocab
        self.v_shard = V % N == 0 and (V // N) % 8 == 0
        if self.v_shard:
            Bt, Vs = N * B, V // N
            self.vs = Vs
            A.xf_all = d.alloc(Bt * H * 4, "xfAll")
            A.xsplit_all = d.alloc(2 * max(64, (Bt + 7) // 8 * 8) * H * 2, "xSplitAll")
            A.logits_s = d.alloc(Bt * Vs * 4, "logitsShard")
            A.amax_part_s = d.alloc(Bt * ARGMAX_PARTS * 8, "amaxPartShard")
            A.amax_s = d.alloc(Bt * 8, "amaxShard")
            A.amax_all = d.alloc(N * Bt * 8, "amaxAll")
            self.emb_shard = ctypes.c_void_p(self.emb.ptr + rank * Vs * (H // 256) * 210)
            if Bt <= 64:
                self.emb_shard_tiles = self._pack_lm_head(self.emb_shard, Vs)

    def _gugrp(self, L, offsets, entries):
        """The experts' gate|up + GeGLU over this layer's expert grouping."""
        c, A = self.cfg, self.A
        if self.gu_tiles:
            self.dev.call("e4b_q40gugrp_tiles", A.moe_in, L.gu_exps_t, offsets, entries, A.gl, c.hidden, c.expert_ff,
                          c.experts, c.topk)
        else:
            self.dev.call("e4b_q40gugrp", A.moe_in, L.gu_exps, offsets, entries, A.gl, c.hidden, c.expert_ff,
                          c.experts, c.topk)

    def _pack_lm_head(self, w, rows):
        d, H = self.dev, self.cfg.hidden
        buf = d.alloc(int(d.L.e4b_q6k_packed_bytes(H, rows)), "lmHeadTiles")
        d.call("e4b_q6k_pack_tiles", w, buf, H, rows)
        return buf

    def _lm_head(self, w, wt, x, xsplit, logits, rows, n):
        """softcap(W x) for n rows of x: the tile-packed copy when there is one."""
        c, d = self.cfg, self.dev
        if wt is not None and n <= 64:
            d.call("e4b_q6k_lmhead_tiles", wt, x, xsplit, logits, c.hidden, rows, ctypes.c_float(c.softcap), n)
        else:
            d.call("e4b_q6k_lmhead_rows", w, x, xsplit, logits, c.hidden, rows, ctypes.c_float(c.softcap), n)

    def _map_peers(self, A, N: int, rank: int):
        """Peer-memory transport: export this rank's receive slabs and flag
        arrays, gather every rank's handles (NCCL), map the peers' buffers and
        upload the address tables (rows, ids, results, dispatch flags, return
        flags: nranks addresses each)."""
        if N < 2:
            raise ValueError("the peer-memory transport needs 2 or more ranks")
        d = self.dev
        self._bar = (d.alloc(4, "epBarrier"), d.alloc(4 * N, "epBarrierAll"))
        A.ep_flag_d = d.alloc(N * 4, "epFlagDispatch")
        A.ep_flag_r = d.alloc(N * 4, "epFlagReturn")
        A.ep_ctr = d.alloc(16, "epCounters")         # [dispatch epoch, arrivals, return epoch, arrivals]
        mine = [A.ep_rx, A.ep_rid, A.ep_ry, A.ep_flag_d, A.ep_flag_r]
        hs = np.zeros((len(mine), 64), np.uint8)
        for k, b in enumerate(mine):
            d.call("e4b_ipc_handle", b.ptr, hs[k].ctypes.data_as(ctypes.c_void_p))
        sbuf, rbuf = d.upload(hs.reshape(-1), "ipcHandles"), d.alloc(N * hs.size, "ipcHandlesAll")
        d.call("e4b_ep_allgather", sbuf, rbuf, ctypes.c_size_t(hs.size))
        d.sync()
        allh = np.ascontiguousarray(d.read(rbuf, np.uint8, N * hs.size).reshape(N, len(mine), 64))
        table = np.zeros((len(mine), N), np.uint64)
        for r in range(N):
            for k, b in enumerate(mine):
                if r == rank:
                    table[k, r] = b.ptr
                    continue
                p = ctypes.c_void_p()
                d.call("e4b_ipc_open", allh[r, k].ctypes.data_as(ctypes.c_void_p), ctypes.byref(p))
                self._ipc_open.append(p.value)
                table[k, r] = p.value
        A.ep_tab = [d.upload(table[k], f"epPeers{k}") for k in range(len(mine))]

    def run_token(self, count: int = 1):
        """As Engine.run_token; with the peer-memory transport every rank first
        meets the others on the device (an NCCL all-gather queued before the
        tokens), so no rank's bounded flag waits start while a peer's host is
        still preparing its run."""
        self.build_plan()
        if self._ipc_open:
            self.dev.call("e4b_ep_allgather", self._bar[0], self._bar[1], ctypes.c_size_t(4))
        super().run_token(count)

    def close(self):
        if self._ipc_open:
            # every rank has finished its stores into peer memory before a mapping goes away
            d = self.dev
            d.sync()
            d.call("e4b_ep_allgather", self._bar[0], self._bar[1], ctypes.c_size_t(4))
            d.sync()
            for p in self._ipc_open:
                d.call("e4b_ipc_close", ctypes.c_void_p(p))
            self._ipc_open = []
        super().close()

    def _timed(self, what, *args):
        """Queue a call; inside exchange_time() bracket it with events."""
        d, xev = self.dev, getattr(self, "_xev", None)
        timed = xev is not None and len(xev) < 29
        if timed:
            a = 4 + 2 * len(xev)
            d.call("e4b_event_record", a)
        d.call(what, *args)
        if timed:
            d.call("e4b_event_record", a + 1)
            xev.append((a, a + 1))

    def _moe_ep_send(self, topk_idx):
        """Dispatch this layer's entries (experts topk_idx) and start the exchange
        of rows + expert ids (one NCCL group on the side stream)."""
        c, d, A, B = self.cfg, self.dev, self.A, self.nseq
        N, rank = self.ep[0], self.ep[1]
        H, E, K = c.hidden, c.experts, c.topk
        if self.ep_transport == "p2p":
            d.call("e4b_ep_dispatch", topk_idx, B, K, E, N, self.cap, A.moe_in, H, None, A.ep_sid, A.ep_slot)
            d.call("e4b_ep_push", A.ep_slot, B, K, A.moe_in, H, A.ep_sid, N, rank, self.cap, A.ep_tab[0], A.ep_tab[1],
                   A.ep_tab[3], A.ep_ctr)
            return
        d.call("e4b_ep_dispatch", topk_idx, B, K, E, N, self.cap, A.moe_in, H, A.ep_sx, A.ep_sid, A.ep_slot)
        d.call("e4b_ep_exchange2_async", A.ep_sx, A.ep_rx, ctypes.c_size_t(self.cap * H * 2), A.ep_sid, A.ep_rid,
               ctypes.c_size_t(self.cap * 4))

    def _moe_ep_finish(self, L):
        """Wait for the rows, run this rank's experts on them, send each result
        back to its slab slot; returns (result rows, entry -> row map)."""
        c, d, A = self.cfg, self.dev, self.A
        N, rank = self.ep[0], self.ep[1]
        H, EF = c.hidden, c.expert_ff
        rows = N * self.cap
        p2p = self.ep_transport == "p2p"
        if p2p:
            self._timed("e4b_ep_wait", A.ep_flag_d, A.ep_ctr, N)
        else:
            self._timed("e4b_ep_join")
        d.call("e4b_expgroup", A.ep_rid, rows, 1, self.e_loc, A.ep_off, A.ep_ent, A.ep_inv)
        d.call("e4b_q40gugrp_tiles" if self.gu_tiles else "e4b_q40gugrp", A.ep_rx, L.gu_loc, A.ep_off, A.ep_ent,
               A.ep_gl, H, EF, self.e_loc, 1)
        d.call("e4b_q40downgrp", A.ep_gl, L.dn_loc, A.ep_off, A.ep_ent, A.ep_y, EF, H, self.e_loc)
        if p2p:
            d.call("e4b_ep_push_back", A.ep_rid, A.ep_inv, A.ep_y, H, N, rank, self.cap, A.ep_tab[2], A.ep_tab[4],
                   A.ep_ctr.at(8))
            self._timed("e4b_ep_wait", A.ep_flag_r, A.ep_ctr.at(8), N)
            return A.ep_ry, A.ep_slot
        d.call("e4b_ep_return", A.ep_rid, A.ep_inv, A.ep_y, rows, H, A.ep_sy)
        self._timed("e4b_ep_exchange", A.ep_sy, A.ep_ry, ctypes.c_size_t(self.cap * H * 4))
        return A.ep_ry, A.ep_slot

    def exchange_time(self, pos: int) -> float:
        """Exposed exchange time (us) of one step: what the main stream waits at
        each join for the overlapped row exchange, plus the result exchange (as
        the stream sees them, waits for peers included); one eager step with
        events around them for the first layers, scaled to all layers."""
        d = self.dev
        toks = d.read(self.A.tok, np.uint32, self.nseq)
        self.set_step(toks, pos)
        self._xev = []
        try:
            self.encode_forward()
            d.sync()
            ms = ctypes.c_float()
            tot = 0.0
            for a, b in self._xev:
                d.call("e4b_event_elapsed", a, b, ctypes.byref(ms))
                tot += ms.value
            n = len(self._xev)
        finally:
            self._xev = None
        return 1000.0 * tot * (2 * self.cfg.layers) / max(n, 1)

    # ------------------------------------------------------------ one step (B tokens)
    def _tail(self, L, y_rows, y_map, topk_w, nxt):
        c, A = self.cfg, self.A
        self.dev.call("e4b_a4btail_wacc", A.tmp, L.post_ffw1, y_rows, y_map, topk_w, c.topk, L.post_ffw2, L.post_ffw,
                      A.hidden_b, nxt if nxt is not None else L.attn_norm, A.normed, A.hidden, c.hidden,
                      ctypes.c_float(c.eps), ctypes.c_float(L.scale), int(nxt is not None), self.nseq, 1)

    def _moe_zipf(self, L, topk_idx, topk_w, nxt):
        """The MoE half of a layer under benchmark routing: the step's Zipf draw
        (topk_idx / topk_w, drawn for every layer at the start of the step)
        replaces the router's choice, so nothing waits for the router; it still
        scores the tokens (the model's work), on the side stream, and joins at
        the end of the layer (its input buffer is rewritten by the next layer)."""
        c, d, A, B = self.cfg, self.dev, self.A, self.nseq
        H, E, K, EF, FF = c.hidden, c.experts, c.topk, c.expert_ff, c.ff
        side = self.overlap_route
        grp = [(A.offsets, A.entries, A.inv), (A.offsets1, A.entries1, A.inv1)]
        # expert grouping of this layer (groupings alternate by layer parity): the
        # first layer's on the main stream, later ones were formed on the previous
        # layer's side stream, whose join precedes this layer
        early = side and self.ep is None
        offs, ents, inv = grp[L.i % 2]
        if self.ep is None and (L.i == 0 or not early):
            d.call("e4b_expgroup", topk_idx, B, K, E, offs, ents, inv)
        if side:
            d.call("e4b_side_begin")
        d.call("e4b_routertop", A.router_in, L.wr, L.pes, A.topk_idx, A.topk_w, H, E, K, B)
        if early and L.i + 1 < c.layers:
            # the next layer's Zipf routes are known: group them now, into the
            # grouping the previous layer used (its kernels precede the fork)
            nidx = ctypes.c_void_p(A.ztop_idx.ptr + (L.i + 1) * B * K * 4)
            d.call("e4b_expgroup", nidx, B, K, E, *grp[(L.i + 1) % 2])
        if side:
            d.call("e4b_side_end")
        if self.ep is not None:
            if self.ep_overlap:
                self._moe_ep_send(topk_idx)       # the rows travel while the dense FFN runs
        d.call("e4b_q40gumm", A.normed, L.gu, A.geglu, H, FF, B)
        d.call("e4b_q40mm", A.geglu, L.down, A.tmp, FF, H, B)
        if self.ep is None:
            self._gugrp(L, offs, ents)
            d.call("e4b_q40downgrp", A.gl, L.down_exps, offs, ents, A.yo, EF, H, E)
            y_rows, y_map = A.yo, inv
        else:
            if not self.ep_overlap:
                self._moe_ep_send(topk_idx)
            y_rows, y_map = self._moe_ep_finish(L)
        self._tail(L, y_rows, y_map, topk_w, nxt)
        if side:
            d.call("e4b_join")

    def encode_forward(self):
        c, d, A, B = self.cfg, self.dev, self.A, self.nseq
        H, V, E, K, EF, FF = c.hidden, c.vocab, c.experts, c.topk, c.expert_ff, c.ff
        d.call("e4b_q6k_embed", self.emb, A.params, A.tok, A.hidden, H, V, ctypes.c_float(F32(math.sqrt(H))), 1, B)
        d.call("e4b_rmsnorm", A.hidden, self.layers[0].attn_norm, None, None, A.normed, H, B, ctypes.c_float(c.eps),
               1, 0, 2)
        if self.zipf_all:
            d.call("e4b_route_zipf_layers", A.params, A.zipf_table, A.ztop_idx, A.ztop_w, B, c.layers, K, E,
                   ctypes.c_uint32(self.route_seed), 0, self.tok0)
        for L in self.layers:
            nxt = self.layers[L.i + 1].attn_norm if L.i + 1 < c.layers else None
            topk_idx, topk_w = A.topk_idx, A.topk_w
            if self.zipf_all:
                topk_idx = ctypes.c_void_p(A.ztop_idx.ptr + L.i * B * K * 4)
                topk_w = ctypes.c_void_p(A.ztop_w.ptr + L.i * B * K * 4)
            if self.kp_qkv > 1:
                d.call("e4b_q40mm_kparts", A.normed, L.qkv, A.qkv, H, L.qkv_rows, B, self.kp_qkv)
            else:
                d.call("e4b_q40mm", A.normed, L.qkv, A.qkv, H, L.qkv_rows, B)
            d.call("e4b_headprep_seq", A.qkv, L.q_norm, L.k_norm, A.params, L.kc, L.vc, A.q, c.q_heads, c.kv_heads,
                   c.head_dim, L.angles, ctypes.c_float(L.theta), ctypes.c_float(c.eps), int(L.keqv), L.cachemode,
                   L.ring, L.slots, B, self.kp_qkv)
            d.call("e4b_attdec_seq", A.q, L.kc, L.vc, A.params, A.part_o, A.part_ml, A.attn, c.q_heads, c.kv_heads,
                   c.head_dim, c.window if L.sliding else 0, L.cachemode, L.ring, L.max_chunks, ctypes.c_float(1.0),
                   L.slots, B, 1)
            if self.kp_o > 1:
                d.call("e4b_q40mm_kparts", A.attn, L.o, A.oparts, c.q_dim, H, B, self.kp_o)
            else:
                d.call("e4b_q40mm", A.attn, L.o, A.oparts, c.q_dim, H, B)
            d.call("e4b_rmsacc3", A.oparts, L.post_attn, L.ffn_norm, L.router_s, L.pre_ffw2, A.hidden, A.normed,
                   A.router_in, A.moe_in, A.hidden_b, H, ctypes.c_float(c.eps), B, 1, self.kp_o)
            if self.zipf_all:
                self._moe_zipf(L, topk_idx, topk_w, nxt)
                continue
            side = self.ep is None and self.overlap_route
            if side:
                # the routing chain (router, Zipf draw, expert sort) on the side stream,
                # concurrent with the dense FFN on the main stream
                d.call("e4b_side_begin")
            d.call("e4b_routertop", A.router_in, L.wr, L.pes, A.topk_idx, A.topk_w, H, E, K, B)
            if self.zipf:
                d.call("e4b_route_zipf", A.params, A.topk_idx, A.topk_w, B, K, E, ctypes.c_float(self.zipf),
                       ctypes.c_uint32(self.route_seed), L.i, self.tok0)
            if self.ep is not None and self.ep_overlap:
                self._moe_ep_send(A.topk_idx)     # the rows travel while the dense FFN runs
            if side:
                d.call("e4b_expgroup", A.topk_idx, B, K, E, A.offsets, A.entries, A.inv)
                d.call("e4b_side_end")
            d.call("e4b_q40gumm", A.normed, L.gu, A.geglu, H, FF, B)
            d.call("e4b_q40mm", A.geglu, L.down, A.tmp, FF, H, B)
            if self.ep is None:
                if side:
                    d.call("e4b_join")
                else:
                    d.call("e4b_expgroup", A.topk_idx, B, K, E, A.offsets, A.entries, A.inv)
                self._gugrp(L, A.offsets, A.entries)
                d.call("e4b_q40downgrp", A.gl, L.down_exps, A.offsets, A.entries, A.yo, EF, H, E)
                y_rows, y_map = A.yo, A.inv
            else:
                if not self.ep_overlap:
                    self._moe_ep_send(A.topk_idx)
                y_rows, y_map = self._moe_ep_finish(L)
            self._tail(L, y_rows, y_map, A.topk_w, nxt)
        d.call("e4b_rmsnorm", A.hidden, self.out_norm, A.xf, None, None, H, B, ctypes.c_float(c.eps), 1, 0, 0)
        if self.ep is not None and self.v_shard:
            # every rank: its V/N LM-head rows for all ranks' tokens, then the argmax merge
            N, rank = self.ep[0], self.ep[1]
            Bt = N * B
            d.call("e4b_ep_allgather", A.xf, A.xf_all, ctypes.c_size_t(B * H * 4))
            self._lm_head(self.emb_shard, self.emb_shard_tiles, A.xf_all, A.xsplit_all, A.logits_s, self.vs, Bt)
            d.call("e4b_argmax_rows", A.logits_s, A.amax_part_s, A.amax_s, self.vs, argmax_parts(Bt), Bt)
            d.call("e4b_ep_allgather", A.amax_s, A.amax_all, ctypes.c_size_t(Bt * 8))
            d.call("e4b_argmax_merge", A.amax_all, N, Bt, self.vs, rank * B, B, A.amax)
        else:
            self._lm_head(self.emb, self.emb_tiles, A.xf, A.xsplit, A.logits, V, B)
            d.call("e4b_argmax_rows", A.logits, A.amax_part, A.amax, V, argmax_parts(B), B)
        d.call("e4b_feedtok_rows", A.amax, A.params, A.ring, RING_CAP, A.tok, B)

    # ------------------------------------------------------------ host API
    def set_step(self, tokens, pos: int):
        """Tokens of all B sequences at position `pos`."""
        t = np.ascontiguousarray(np.asarray(tokens, np.uint32).reshape(self.nseq))
        self.dev.write(self.A.tok, t)
        self.host_params[:] = (pos, pos + 1, int(t[0]), 0, pos, pos + 1, pos, 0)
        self.dev.write(self.A.params, self.host_params)

    def step(self, tokens, pos: int):
        self.set_step(tokens, pos)
        self.run_token(1)

    def prefill(self, prompts, chunk: int | None = None):
        """Fill the KV caches for prompts [B][P] and leave the last position's
        greedy tokens on the device, ready for decode_chunk at position P
        (src/engine-a4b.js:549-585).  One GPU: chunked batched prefill (B x C
        token rows per step, tensor-core GEMMs); expert parallel, or chunk=0:
        token by token (src/engine-a4b.js:828)."""
        prompts = np.asarray(prompts)
        P = prompts.shape[1]
        if self.ep is None and chunk != 0:
            return self.prefill_chunked(prompts, chunk)
        for pos in range(P):
            self.step(prompts[:, pos], pos)
            if (pos + 1) % STATUS_EVERY == 0 or pos + 1 == P:
                self.check_status(f"prefill (position {pos})")

    def prefill_chunk_len(self) -> int:
        """Positions per prefill chunk: about 4096 token rows, at most 512
        positions (the sliding rings hold window + 512 slots, so a chunk never
        overwrites a slot one of its own queries still needs)."""
        c = self.cfg
        lim = 512
        if any(L.sliding for L in self.layers):
            lim = min(lim, min(L.ring for L in self.layers if L.sliding) - c.window + 1)
        return max(1, min(lim, 4096 // self.nseq))

    def _alloc_prefill(self, R: int):
        c, d, B = self.cfg, self.dev, self.nseq
        H, QD, FF, E, K, EF = c.hidden, c.q_dim, c.ff, c.experts, c.topk, c.expert_ff
        if getattr(self, "PA", None) is not None and self.PA.R >= R:
            return self.PA
        if getattr(self, "PA", None) is not None:
            for b in self.PA.bufs:
                d.free(b)
        PA = type("PrefillActs", (), {})()
        PA.R = R
        maxrows = max(L.qkv_rows for L in self.layers)
        sizes = dict(tok=R * 4, hidden=R * H * 4, hidden_b=R * H * 4, normed=R * H * 2, qkv=R * maxrows * 4,
                     q=R * QD * 4, attn=R * QD * 2, o=R * H * 4, router_in=R * H * 4, moe_in=R * H * 2,
                     topk_idx=R * K * 4, topk_w=R * K * 4, geglu=R * FF * 2, tmp=R * H * 4,
                     offsets=(E + 1) * 4, entries=R * K * 4, inv=R * K * 4, xs=R * K * H * 2,
                     gl=R * K * EF * 2, yo=R * K * H * 4, params=32)
        PA.bufs = []
        for name, n in sizes.items():
            b = d.alloc(n, f"pre_{name}", zero=False)
            setattr(PA, name, b)
            PA.bufs.append(b)
        self.PA = PA
        return PA

    def prefill_chunked(self, prompts, chunk: int | None = None):
        """Batched prefill (src/engine-a4b.js:467-585): chunks of C positions of
        all B sequences as B x C position-major token rows (row = p * B + b).
        Per layer: q|k|v, o, dense gate|up + GeGLU and down as tcgen05 GEMMs over
        all rows (e4b_q40gemm); head prep writes every row's K/V into its
        sequence's cache (e4b_headprep_rows); causal attention of the chunk
        (e4b_attn_prefill); router per row; the rows' B x C x K expert entries
        sorted by expert, their activation rows gathered contiguously, and the
        grouped expert GEMMs; the combine fused into the layer tail.  After the
        last chunk, the last position's rows go through the final norm, LM head,
        argmax and token feedback, so decoding continues at position P."""
        c, d, B = self.cfg, self.dev, self.nseq
        H, QD, FF, E, K, EF, V = c.hidden, c.q_dim, c.ff, c.experts, c.topk, c.expert_ff, c.vocab
        prompts = np.asarray(prompts, np.uint32)
        assert prompts.shape[0] == B
        P = prompts.shape[1]
        C = min(chunk or self.prefill_chunk_len(), P)
        PA = self._alloc_prefill(B * C)
        eps = ctypes.c_float(c.eps)
        hp = np.zeros(8, np.uint32)
        for p0 in range(0, P, C):
            n = min(C, P - p0)
            R = B * n
            d.write(PA.tok, np.ascontiguousarray(prompts[:, p0:p0 + n].T).reshape(-1))
            hp[:] = (p0, p0 + 1, 0, 0, p0, p0 + 1, 0, 0)
            d.write(PA.params, hp)
            d.call("e4b_q6k_embed", self.emb, PA.params, PA.tok, PA.hidden, H, V, ctypes.c_float(F32(math.sqrt(H))),
                   1, R)
            d.call("e4b_rmsnorm", PA.hidden, self.layers[0].attn_norm, None, None, PA.normed, H, R, eps, 1, 0, 1)
            for L in self.layers:
                nxt = self.layers[L.i + 1].attn_norm if L.i + 1 < c.layers else None
                d.call("e4b_q40gemm", PA.normed, L.qkv, PA.qkv, None, None, H, L.qkv_rows, R, 1, 0)
                d.call("e4b_headprep_rows", PA.qkv, L.q_norm, L.k_norm, PA.params, L.kc, L.vc, PA.q, c.q_heads,
                       c.kv_heads, c.head_dim, L.angles, ctypes.c_float(L.theta), eps, int(L.keqv), L.cachemode,
                       L.ring, L.slots, B, n)
                d.call("e4b_attn_prefill", PA.q, L.kc, L.vc, PA.params, PA.attn, c.q_heads, c.kv_heads, c.head_dim,
                       c.window if L.sliding else 0, L.cachemode, L.ring, ctypes.c_float(1.0), L.slots, B, n)
                d.call("e4b_q40gemm", PA.attn, L.o, PA.o, None, None, QD, H, R, 1, 0)
                d.call("e4b_rmsacc3", PA.o, L.post_attn, L.ffn_norm, L.router_s, L.pre_ffw2, PA.hidden, PA.normed,
                       PA.router_in, PA.moe_in, PA.hidden_b, H, eps, R, 0, 1)
                d.call("e4b_routertop", PA.router_in, L.wr, L.pes, PA.topk_idx, PA.topk_w, H, E, K, R)
                if self.zipf:
                    d.call("e4b_route_zipf_rows", PA.params, PA.topk_idx, PA.topk_w, B, n, K, E,
                           ctypes.c_float(self.zipf), ctypes.c_uint32(self.route_seed), L.i, self.tok0)
                d.call("e4b_q40gemm", PA.normed, L.gu, None, PA.geglu, None, H, FF, R, 1, 1)
                d.call("e4b_q40gemm", PA.geglu, L.down, PA.tmp, None, None, FF, H, R, 1, 0)
                d.call("e4b_expgroup", PA.topk_idx, R, K, E, PA.offsets, PA.entries, PA.inv)
                d.call("e4b_gather_rows", PA.moe_in, PA.entries, K, PA.xs, H, R * K, R)
                d.call("e4b_q40gemm", PA.xs, L.gu_exps, None, PA.gl, PA.offsets, H, EF, R * K, E, 1)
                d.call("e4b_q40gemm", PA.gl, L.down_exps, PA.yo, None, PA.offsets, EF, H, R * K, E, 0)
                d.call("e4b_a4btail_wacc", PA.tmp, L.post_ffw1, PA.yo, PA.inv, PA.topk_w, K, L.post_ffw2, L.post_ffw,
                       PA.hidden_b, nxt if nxt is not None else L.attn_norm, PA.normed, PA.hidden, H, eps,
                       ctypes.c_float(L.scale), int(nxt is not None), R, 0)
            self.check_status(f"prefill chunk at position {p0}")
        # the last position's B rows: final norm, LM head, argmax, token feedback
        A = self.A
        last = ctypes.c_void_p(PA.hidden.ptr + (n - 1) * B * H * 4)
        self.host_params[:] = (P - 1, P, 0, 0, P - 1, P, P - 1, 0)
        d.write(A.params, self.host_params)
        d.call("e4b_rmsnorm", last, self.out_norm, A.xf, None, None, H, B, eps, 1, 0, 0)
        self._lm_head(self.emb, self.emb_tiles, A.xf, A.xsplit, A.logits, V, B)
        d.call("e4b_argmax_rows", A.logits, A.amax_part, A.amax, V, argmax_parts(B), B)
        d.call("e4b_feedtok_rows", A.amax, A.params, A.ring, RING_CAP, A.tok, B)
        self.check_status("prefill (last position)")

    def generate(self, prompts, n_new: int, chunk: int | None = None):
        """prompts [B][P] (same length) -> [B][n_new] greedy ids; chunk as prefill's."""
        prompts = np.asarray(prompts)
        P = prompts.shape[1]
        assert P + n_new <= RING_CAP
        self.prefill(prompts, chunk=chunk)
        if n_new > 1:
            self.decode_chunk(n_new - 1)
        self.dev.sync()
        ring = self.dev.read(self.A.ring, np.uint32, self.nseq * RING_CAP).reshape(self.nseq, RING_CAP)
        return ring[:, P - 1:P - 1 + n_new].astype(np.int64)

    def read_hidden(self) -> np.ndarray:
        return self.dev.read(self.A.hidden, F32, self.nseq * self.cfg.hidden).reshape(self.nseq, -1)

    def read_logits(self) -> np.ndarray:
        """Logits of the last step, [nseq][vocab] (one GPU; an expert-parallel
        rank holds only its vocabulary slice for every rank's tokens)."""
        if self.ep is not None and getattr(self, "v_shard", False):
            raise RuntimeError("expert-parallel ranks keep vocabulary slices, not full logit rows")
        return self.dev.read(self.A.logits, F32, self.nseq * self.cfg.vocab).reshape(self.nseq, -1)

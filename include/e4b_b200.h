/*
 * e4b_b200.h -- C ABI of the B200 (sm_100a) per-token decode path.
 *
 * Drop-in boundary for the reference's WebGPU operator API: where the reference
 * compiles kernels/<op>.wgsl with ${NAME} substitution and dispatches it with an
 * ordered list of storage buffers (src/gpu.js:67-84 `Kernels.pipeline`,
 * src/gpu.js:95-108 / src/engine-a4b.js:401-420 `run`), this library exports one
 * C function per operator.  Device buffers are passed as plain pointers in the
 * reference's binding order; the former ${} compile-time parameters become int /
 * float arguments.  Weights are the GGUF q4_0 (18 B / 32 weights) and q6_K
 * (210 B / 256 weights) blocks exactly as stored in the file.
 *
 * Conventions
 *   - Every function returns E4B_OK (0) or a negative E4B_E* code; the message
 *     of the last failure on a context is e4b_last_error(ctx).
 *   - Kernels are enqueued on the context's stream and never allocate; the
 *     caller owns all device memory (e4b_alloc / e4b_free).  Scratch buffers an
 *     operator needs (split-KV partials, argmax partials) are caller-provided.
 *   - A context is bound to one device and is not thread-safe.
 *   - f16 buffers are IEEE binary16 stored as uint16_t.
 *   - `params` is the reference's per-token parameter block (8 x u32,
 *     src/engine-a4b.js:697-698): [0]=pos [1]=pos+1 [2]=token [3]=0
 *     [4]=kvCount (global-layer slot) [5]=kvCount+1 [6]=token-ring index [7]=0.
 */
#ifndef E4B_B200_H
#define E4B_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define E4B_API __attribute__((visibility("default")))
#else
#define E4B_API
#endif

enum {
  E4B_OK = 0,
  E4B_EINVAL = -1,    /* bad argument (null pointer, size not a block multiple, ...) */
  E4B_ECUDA = -2,     /* CUDA runtime error */
  E4B_ETIMEOUT = -3,  /* a bounded device-side wait gave up (device status word) */
  E4B_ENCCL = -4,     /* NCCL error */
  E4B_ENOMEM = -5,    /* allocation failed */
  E4B_EDEVICE = -6    /* device-side check failed (index out of range, ...) */
};

typedef struct e4b_ctx e4b_ctx;

/* ------------------------------------------------------------------ runtime */
/* Replaces initDevice (src/gpu.js:4-24). */
E4B_API int e4b_create(int device, e4b_ctx** out);
E4B_API int e4b_destroy(e4b_ctx* ctx);
E4B_API const char* e4b_last_error(const e4b_ctx* ctx);
E4B_API int e4b_device_info(e4b_ctx* ctx, int* sm_count, int* cc_major, int* cc_minor, size_t* total_mem);
/* Buffers: replaces alloc / upload / readback (src/gpu.js:26-50). */
E4B_API int e4b_alloc(e4b_ctx* ctx, size_t bytes, void** out);
E4B_API int e4b_free(e4b_ctx* ctx, void* ptr);
E4B_API int e4b_host_alloc(e4b_ctx* ctx, size_t bytes, void** out); /* pinned host memory */
E4B_API int e4b_host_free(e4b_ctx* ctx, void* ptr);
E4B_API int e4b_upload(e4b_ctx* ctx, void* dst, const void* src, size_t bytes);   /* synchronous */
E4B_API int e4b_download(e4b_ctx* ctx, void* dst, const void* src, size_t bytes); /* synchronous */
E4B_API int e4b_upload_async(e4b_ctx* ctx, void* dst, const void* src, size_t bytes);
E4B_API int e4b_download_async(e4b_ctx* ctx, void* dst, const void* src, size_t bytes);
E4B_API int e4b_memset(e4b_ctx* ctx, void* dst, int value, size_t bytes);           /* stream-ordered */
E4B_API int e4b_copy(e4b_ctx* ctx, void* dst, const void* src, size_t bytes);        /* device to device, stream-ordered */
E4B_API int e4b_sync(e4b_ctx* ctx);
/* Timing: events recorded on the context stream (slots 0..63). */
E4B_API int e4b_event_record(e4b_ctx* ctx, int slot);
E4B_API int e4b_event_elapsed(e4b_ctx* ctx, int slot_a, int slot_b, float* ms);
/* Programmatic dependent launch between consecutive kernels (default on). */
E4B_API int e4b_set_pdl(e4b_ctx* ctx, int enable);
/* Workspace for the streaming GEMVs (split-K partials and arrival counters).
 * Caller-owned device memory of at least e4b_workspace_bytes(); it is zeroed
 * here and must not be shared by two contexts.  Ops that need it fail with
 * E4B_EINVAL until one is set. */
E4B_API int e4b_set_workspace(e4b_ctx* ctx, void* ws, size_t bytes); /* ws = NULL, bytes = 0 detaches */
E4B_API size_t e4b_workspace_bytes(void);
/* Tuning knobs of the streaming kernels: "stream_ctas_per_sm" (1..2, default 1),
 * "stream_stages" (2..4, default 4), "stream_variant" (GEMV warps per CTA x
 * blocks per staged piece: 0 = 8 x 32, 1 = 16 x 16, 2 = 16 x 8).
 * "attn_grid_cap" (>= 0, default 0 = one CTA per SM): at most this many CTAs for
 * e4b_attdec_seq, so each CTA runs more items (the stage ring's wrap-around).
 * "lmhead_tc_min" (1..65, default 1): e4b_q6k_lmhead_rows uses its tcgen05
 * kernel for n >= this many rows (65: never).
 * "lmhead_tiles_tc" (0..2, default 0): how e4b_q6k_lmhead_tiles runs 2..64
 * rows: 0 = the warp-MMA kernel up to 32 rows, the tcgen05 one above; 1 = always
 * tcgen05; 2 = always warp-MMA.
 * "wait_limit_us" (1000..10000000, default 1000000): the bound of the batched
 * attention's and e4b_ep_wait's device waits, after which the call records
 * E4B_ST_TIMEOUT in the status word and returns. */
E4B_API int e4b_set_option(e4b_ctx* ctx, const char* name, int value);
/* Device status word: nonzero after a device-side check or bounded wait failed;
 * reading it resets it to zero. */
E4B_API int e4b_device_status(e4b_ctx* ctx, uint32_t* status);

/* Plan = one recorded per-token dispatch sequence, replayed as a CUDA graph.
 * Replaces the token-plan record/replay of src/engine-a4b.js:800-818. */
E4B_API int e4b_plan_begin(e4b_ctx* ctx);
E4B_API int e4b_plan_end(e4b_ctx* ctx, int* plan);
E4B_API int e4b_plan_launch(e4b_ctx* ctx, int plan, int count);
E4B_API int e4b_plan_destroy(e4b_ctx* ctx, int plan);
/* Two concurrent chains on one context: after e4b_side_begin the launches go
 * to a second stream that starts after the work queued so far; e4b_side_end
 * sends later launches to the main stream again (which does not wait for the
 * side chain); e4b_join makes the main stream's later work wait for the side
 * chain.  So "side_begin, A, side_end, B, join, C" runs A and B concurrently
 * and C after both.  Plans (graph capture) may contain such pairs; they do
 * not nest.  No counterpart in the reference, whose WebGPU queue runs its
 * dispatches in submission order. */
E4B_API int e4b_side_begin(e4b_ctx* ctx);
E4B_API int e4b_side_end(e4b_ctx* ctx);
E4B_API int e4b_join(e4b_ctx* ctx);

/* ----------------------------------------------------------- dequantisation */
/* Bit-exact block decoders (for parity checks of the in-kernel decode).
 * q4_0: scripts/ternarize_a4b.py:80-87; q6_K: kernels/q6k.wgsl:44-68. */
E4B_API int e4b_dequant_q40(e4b_ctx* ctx, const uint8_t* w, float* out, int64_t nblocks);
E4B_API int e4b_dequant_q6k(e4b_ctx* ctx, const uint8_t* w, float* out, int64_t nblocks);

/* --------------------------------------------------------- q6_K embed / head */
/* kernels/q6k.wgsl MODE 0 (:37-73): y[b*N+i] = ((d*sc)*(q-32))*mult of row
 * tok[b] (batch > 0), else of row tok[0] (toksrc=1) or params[2] (toksrc=0).
 * A row >= rows sets the device status word and writes zeros. */
E4B_API int e4b_q6k_embed(e4b_ctx* ctx, const uint8_t* w, const uint32_t* params, const uint32_t* tok,
                          float* y, int N, int rows, float mult, int toksrc, int batch);
/* kernels/q6k.wgsl MODE 1 (:75-131): y[o] = softcap(sum d*sc*(q-32)*x), OUT rows
 * of N; softcap = 0 disables.  batch rows of x / y (stride N / OUT). */
E4B_API int e4b_q6k_lmhead(e4b_ctx* ctx, const uint8_t* w, const float* x, float* y, int N, int OUT,
                           float softcap, int batch);

/* ------------------------------------------------------------ norms / tails */
/* Fragment order ("xfo"): the f16 activation rows that feed the multi-token
 * q4_0 GEMMs below are stored permuted inside each 32-element block so one
 * 16-byte load gives an MMA lane its 8 values: element j of a block sits at
 * half 8t + slot with, for odd blocks, t = (j%16)/4; for even blocks
 * t = ((j%16)-2)/4 for j%16 in [2,14) and t = 3 for j%16 in {0,1,14,15};
 * slots [j0, j2, j1, j3] of t's four indices, +4 for j >= 16.  The python host
 * gives the permutation as batch.xfo_perm(n). */

/* kernels/rmsnorm.wgsl:13-51.  rows x dim; y (f32) or yh (f16) per f16out
 * (2: f16 in fragment order); sums[row] = sum(y) if sumout. */
E4B_API int e4b_rmsnorm(e4b_ctx* ctx, const float* x, const float* w, float* y, float* sums, uint16_t* yh,
                        int dim, int rows, float eps, int with_scale, int sumout, int f16out);
/* kernels/rmsacc.wgsl:10-26: hidden = (hidden + rms(x)*w) * mul. */
E4B_API int e4b_rmsacc(e4b_ctx* ctx, const float* x, const float* w, float* hidden, int dim, float eps,
                       float mul);
/* kernels/rmsaccsrq.wgsl:30-76 without its int8 activation quantisation:
 * hidden = (hidden + rms(t)*w1) * mul; yh = f16(rms(hidden)*w2) (norm2=1) or
 * f16(hidden) (norm2=0). */
E4B_API int e4b_rmsaccn(e4b_ctx* ctx, const float* t, const float* w1, float* hidden, const float* w2,
                        uint16_t* yh, int dim, float eps, float mul, int norm2);
/* kernels/rmsacc3.wgsl:27-53 (rows = batch); xfo=1: y1, y3 in fragment order;
 * nparts > 1: t is the sum of nparts [rows][dim] partials (e4b_q40mm_kparts), in order. */
E4B_API int e4b_rmsacc3(e4b_ctx* ctx, const float* t, const float* w_acc, const float* w1, const float* w2,
                        const float* w3, const float* h_in, uint16_t* y1, float* y2, uint16_t* y3,
                        float* h_out, int dim, float eps, int rows, int xfo, int nparts);
/* kernels/a4btail.wgsl:26-71 (rows = batch); xfo=1: y_next in fragment order. */
E4B_API int e4b_a4btail(e4b_ctx* ctx, const float* t1, const float* w1, const float* m, const float* w2,
                        const float* wp, const float* h_in, const float* w_next, uint16_t* y_next,
                        float* h_out, int H, float eps, float mul, int next, int rows,
                        int xfo);
/* kernels/wacc.wgsl + a4btail.wgsl in one pass (batched MoE tail): the MoE
 * output row m[row] = sum_k topk_w[row][k] * y[inv[row*K+k]] (slot order) is
 * formed in place of reading m; an inv of 0xffffffff (an entry an expert-parallel
 * slab had no room for, flagged in the status word) contributes nothing.  K <= 32. */
E4B_API int e4b_a4btail_wacc(e4b_ctx* ctx, const float* t1, const float* w1, const float* y, const uint32_t* inv,
                             const float* topk_w, int K, const float* w2, const float* wp, const float* h_in,
                             const float* w_next, uint16_t* y_next, float* h_out, int H, float eps, float mul,
                             int next, int rows, int xfo);

/* ------------------------------------------------------------ q4_0 GEMVs */
/* kernels/q40mv.wgsl:56-89: y[z*OUT+o] = sum_b d_b sum_i (n_i-8) x_i.
 * x is f32 (x_f16=0) or f16 (x_f16=1).  expert=1: weights of expert topk[z]
 * (stride OUT*IN/32 blocks); xslot=1: x row z (stride IN); nz = slots (1 if
 * neither).  batch > 1: rows of x / y per token (stride IN / nz*OUT). */
E4B_API int e4b_q40mv(e4b_ctx* ctx, const void* x, const uint8_t* w, const uint32_t* topk, float* y,
                      int IN, int OUT, int expert, int xslot, int x_f16, int nz, int batch);
/* kernels/q40gu.wgsl:62-119 (EXPERT=2 merged grid): dense rows [gate FF2 | up FF2]
 * of w2 on x2 -> yh2 = f16(gelu(g)*u) [FF2]; expert slot k: rows of expert
 * topk[k] of w ([E][2*FF][IN]) on x -> yh[k*FF ..]; w2 == NULL skips the dense
 * part, K == 0 skips the experts.  batch rows (token stride IN in x/x2, FF2 in
 * yh2, K*FF in yh, K in topk). */
E4B_API int e4b_q40gu(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, const uint32_t* topk, uint16_t* yh,
                      const uint16_t* x2, const uint8_t* w2, uint16_t* yh2, int IN, int FF, int FF2, int K,
                      int batch);
/* kernels/q40moedown.wgsl:42-75: y[o] = sum_k tkw[k] * (W_topk[k] x_k)[o],
 * x f16 [K][IN], W [E][OUT][IN]. */
E4B_API int e4b_q40moedown(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, const uint32_t* topk,
                           const float* tkw, float* y, int IN, int OUT, int K, int batch);
/* ---- grouped MoE for batched decode (kernels/expgroup.wgsl, q40gugrp.wgsl,
 * q40downgrp.wgsl, wacc.wgsl).  Entries are (token, slot) pairs e = token*K + slot.
 * expgroup: sort the n_tok*K entries of topk[n_tok][K] by expert (stable):
 *   offsets[E+1], entries[pos] = e, inv[e] = pos; an id of 0xffffffff is an
 *   empty slot and is left out (its inv is not written).
 * q40gugrp: per entry at sorted position pos, yh[pos][FF] = f16(gelu(gate)*up)
 *   with expert rows [gate FF | up FF] of w[E][2FF][IN] and x = x[token][IN];
 *   IN % 256 == 0, FF % 32 == 0.
 * q40downgrp: y[pos][OUT] = W_e x[pos] (x rows by position; w[E][OUT][IN]);
 *   OUT % 16 == 0 when IN % 256 != 0.
 * wacc: out[t][o] = sum_k topk_w[t][k] * y[inv[t*K+k]][o], slots in order.
 * Every f16 x and yh of the multi-token GEMMs is in fragment order; IN % 64 == 0;
 * weights and x 16-byte aligned.  An expert's tokens are processed 16 at a time. */
E4B_API int e4b_expgroup(e4b_ctx* ctx, const uint32_t* topk, int n_tok, int K, int E, uint32_t* offsets,
                         uint32_t* entries, uint32_t* inv);
E4B_API int e4b_q40gugrp(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
                         const uint32_t* entries, uint16_t* yh, int IN, int FF, int E, int K);
E4B_API int e4b_q40downgrp(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, const uint32_t* offsets,
                           const uint32_t* entries, float* y, int IN, int OUT, int E);
/* Tile-packed copy of a q4_0 matrix (rows % 16 == 0, IN % 256 == 0; the same
 * number of bytes as the GGUF blocks, wt 16-byte aligned): per 16-row group r
 * and 256-k quantum q one 2304-byte piece at (r * IN/256 + q) * 2304, the 16
 * rows' 8 f16 block scales ([row][block], 256 B) then the nibble bytes
 * regrouped into the 32-bit words the tensor-core A operand of each lane reads
 * ([block half][row][lane] x 4 words, 2048 B).  e4b_q40gugrp_tiles is
 * e4b_q40gugrp on that copy of w[E][2FF][IN] (rows = E * 2FF): one 16-byte load
 * per row for 8 scales and per 4 blocks for the nibbles, no unaligned block
 * reads; its outputs are bit-identical to e4b_q40gugrp's. */
E4B_API int e4b_q40_pack_tiles(e4b_ctx* ctx, const uint8_t* w, uint8_t* wt, int rows, int IN);
E4B_API int e4b_q40gugrp_tiles(e4b_ctx* ctx, const uint16_t* x, const uint8_t* wt, const uint32_t* offsets,
                               const uint32_t* entries, uint16_t* yh, int IN, int FF, int E, int K);
/* dst[i] = src[idx[i] / div] for n f16 rows of H (a zero row where idx[i] is
 * 0xffffffff or out of range): the expert-sorted activation rows of a prefill
 * chunk (entries from e4b_expgroup, div = K), contiguous per expert as the
 * grouped GEMM reads them (the row gather of kernels/q40grpsg32.wgsl:51-58,
 * done once per layer instead of per tile). */
E4B_API int e4b_gather_rows(e4b_ctx* ctx, const uint16_t* src, const uint32_t* idx, int div, uint16_t* dst, int H,
                            int n, int n_src);
/* Ternary experts (kernels/t2gu.wgsl, kernels/t2moedown.wgsl; format of
 * scripts/ternarize_a4b.py): w = 2-bit planes, 16 values of t + 1 per u32 in the
 * shift-group layout (element 4g + j at bits 2g + 8j), rows of IN/16 words;
 * scale = one f16 per row.  t2gu: expert slots of the fused gate|up + GeGLU,
 * rows [e][gate FF | up FF] -> yh[k][FF] (f16); t2moedown: y[o] = sum_k topk_w[k] *
 * scale[e_k][o] * t[e_k][o] . x[k] (slot-combined).  Expert ids >= E set the
 * BADINDEX status. */
E4B_API int e4b_t2gu(e4b_ctx* ctx, const uint16_t* x, const uint32_t* w, const uint16_t* scale, const uint32_t* topk,
                     uint16_t* yh, int IN, int FF, int K, int E);
E4B_API int e4b_t2moedown(e4b_ctx* ctx, const uint16_t* x, const uint32_t* w, const uint16_t* scale,
                          const uint32_t* topk, const float* topk_w, float* y, int IN, int OUT, int K, int E);
/* Batched-prefill q4_0 GEMM on the tcgen05 tensor cores: kernels/q40sg.wgsl:30-124
 * (TPREC=f32) and, grouped, kernels/q40grpsg32.wgsl:31-129.  x: f16 [M][IN]
 * row-major (plain order), IN a multiple of 64, 16-byte aligned.  w: q4_0
 * [groups][rows][IN] with rows = OUT (epi 0) or 2*OUT ([gate OUT | up OUT],
 * epi 1).  groups == 1: one matrix over rows [0, M) (offsets may be NULL);
 * groups > 1 (<= 256): rows [offsets[g], offsets[g+1]) of x use matrix g
 * (offsets: device u32 [groups+1], e.g. from e4b_expgroup).  epi 0: y f32
 * [M][OUT] = W x; epi 1: yh f16 [M][OUT] = f16(gelu(gate) * up).  Weights are
 * dequantised exactly (f16 hi + lo), products summed in f32. */
E4B_API int e4b_q40gemm(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, float* y, uint16_t* yh,
                        const uint32_t* offsets, int IN, int OUT, int M, int groups, int epi);
/* Dense batched GEMMs on the same tensor-core path (n token rows, f16 x in
 * fragment order):
 * q40mm: y[n][OUT] = W x[n] (f32); q40gumm: yh[n][FF] = f16(gelu(gate)*up) with
 * rows [gate FF | up FF] (kernels/q40gu.wgsl dense part, per token; yh in fragment order). */
E4B_API int e4b_q40mm(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, float* y, int IN, int OUT, int n);
/* q40mm with K split over kparts CTA groups, all n <= 64 tokens per weight
 * decode: y_parts[kp][n][OUT] = the kp-th K-range's share (quanta of 256 k,
 * split evenly); the consumer sums the parts in order.  IN % 256 == 0. */
E4B_API int e4b_q40mm_kparts(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, float* y_parts, int IN, int OUT,
                             int n, int kparts);
E4B_API int e4b_q40gumm(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, uint16_t* yh, int IN, int FF, int n);
E4B_API int e4b_wacc(e4b_ctx* ctx, const float* y, const uint32_t* inv, const float* topk_w, float* out, int n_tok,
                     int K, int OUT);
/* kernels/moecomb.wgsl:6-15: y[i] = sum_k topkW[k] * slots[k*H+i]. */
E4B_API int e4b_moecomb(e4b_ctx* ctx, const float* slots, const float* topk_w, float* y, int H, int K);

/* ------------------------------------------------------- expert parallelism
 * Experts in contiguous blocks of E/nranks per rank; every rank decodes its own
 * sequences.  nccl_unique_id on one rank, shared by the caller (any transport),
 * then nccl_init on every rank (one communicator per context).
 * ep_dispatch: entry i = t*K+k of topk[n_tok][K] goes to rank e/(E/nranks):
 *   send_x[rank][pos] = x[t] (H halves), send_ids[rank][pos] = e - rank*E/nranks,
 *   slot[i] = rank*cap + pos, pos in entry order; unused rows get id 0xffffffff.
 *   cap entries per peer (n_tok*K is always enough); overflow sets the status word.
 * ep_exchange: grouped ncclSend/ncclRecv of bytes_per_peer with every rank
 *   (recv block p = what rank p sent here).
 * ep_return: send_y[i] = y[inv[i]] for the rows i < rows whose id is not
 *   0xffffffff (y rows of H floats, inv from expgroup over the received ids).
 * After the results come back, e4b_a4btail_wacc(y = received rows, inv = slot)
 * combines in slot order. */
E4B_API int e4b_nccl_unique_id(uint8_t* out128);
E4B_API int e4b_nccl_init(e4b_ctx* ctx, int nranks, int rank, const uint8_t* id128);
E4B_API int e4b_nccl_destroy(e4b_ctx* ctx);
E4B_API int e4b_ep_dispatch(e4b_ctx* ctx, const uint32_t* topk, int n_tok, int K, int E, int nranks, int cap,
                            const uint16_t* x, int H, uint16_t* send_x, uint32_t* send_ids, uint32_t* slot);
E4B_API int e4b_ep_exchange(e4b_ctx* ctx, const void* send, void* recv, size_t bytes_per_peer);
/* Two exchanges in one NCCL group on the communicator's side stream, after the
 * work queued so far; e4b_ep_join makes later work wait for them (work queued
 * in between overlaps the transfer). */
E4B_API int e4b_ep_exchange2_async(e4b_ctx* ctx, const void* send_a, void* recv_a, size_t bytes_a,
                                   const void* send_b, void* recv_b, size_t bytes_b);
E4B_API int e4b_ep_join(e4b_ctx* ctx);
E4B_API int e4b_ep_return(e4b_ctx* ctx, const uint32_t* recv_ids, const uint32_t* inv, const float* y, int rows,
                          int H, float* send_y);
/* Vocabulary-sharded LM head for N > 1: ep_allgather = ncclAllGather of
 * bytes_per_rank (rank-major); argmax_merge: all[r][t] = (index within rank r's
 * slice of `slice` rows, f32 value bits) from e4b_argmax_rows -> out[b] for
 * tokens row0 + b = the best over ranks with global index r*slice + index, ties
 * to the lowest global index. */
E4B_API int e4b_ep_allgather(e4b_ctx* ctx, const void* send, void* recv, size_t bytes_per_rank);
E4B_API int e4b_argmax_merge(e4b_ctx* ctx, const uint32_t* all, int nranks, int ntok, int slice, int row0,
                             int nrows, uint32_t* out);
/* Peer-memory transport (N >= 2 ranks, one process per GPU, in place of
 * ep_exchange*): each rank exports its receive slabs (rows, ids, results) and
 * two flag arrays of nranks u32 with ipc_handle (64 bytes each), the handles
 * travel by any means (ep_allgather), and every rank opens its peers' with
 * ipc_open; *_ptrs are device arrays of nranks addresses (this rank's own
 * buffer at index rank).
 * ep_dispatch with send_x = NULL fills only send_ids / slot; ep_push then
 *   stores x[t] of every entry straight into rx_ptrs[d] row rank*cap + pos and
 *   this rank's ids into rid_ptrs[d] rows rank*cap.., and publishes epoch
 *   ctr[0] + 1 into flag_ptrs[d][rank] of every rank (ctr: 2 u32 of this rank,
 *   zero-initialised, one pair per direction).
 * ep_wait: the stream waits (device side, ~1 s bound, then the TIMEOUT status)
 *   until flag[p] has reached ctr[0] for every p.
 * ep_push_back: received row i = p*cap + pos holding an entry -> ry_ptrs[p] row
 *   rank*cap + pos = y[inv[i]], then the same publication.
 * Slabs keep the NCCL path's layout, so expgroup / a4btail_wacc read them
 * unchanged. */
E4B_API int e4b_ipc_handle(e4b_ctx* ctx, const void* ptr, uint8_t* out64);
E4B_API int e4b_ipc_open(e4b_ctx* ctx, const uint8_t* handle64, void** out);
E4B_API int e4b_ipc_close(e4b_ctx* ctx, void* ptr);
E4B_API int e4b_ep_push(e4b_ctx* ctx, const uint32_t* slot, int n_tok, int K, const uint16_t* x, int H,
                        const uint32_t* send_ids, int nranks, int rank, int cap, const uint64_t* rx_ptrs,
                        const uint64_t* rid_ptrs, const uint64_t* flag_ptrs, uint32_t* ctr);
E4B_API int e4b_ep_push_back(e4b_ctx* ctx, const uint32_t* recv_ids, const uint32_t* inv, const float* y, int H,
                             int nranks, int rank, int cap, const uint64_t* ry_ptrs, const uint64_t* flag_ptrs,
                             uint32_t* ctr);
E4B_API int e4b_ep_wait(e4b_ctx* ctx, const uint32_t* flag, const uint32_t* ctr, int nranks);

/* ------------------------------------------------------------ router */
/* kernels/routertop.wgsl:19-71: scores = Wr[E][H] . x (f32), softmax, K-way
 * iterative argmax (ties -> lowest index), renormalise, x pes[e].  One token
 * per row of x (batch rows).  With a workspace attached the scores are a
 * split-K f32 GEMM into the workspace, then a per-token top-K pass (two
 * launches). */
E4B_API int e4b_routertop(e4b_ctx* ctx, const float* x, const float* wr, const float* pes, uint32_t* topk_idx,
                          float* topk_w, int H, int E, int K, int batch);
/* Benchmark routing (benchmark config 5, not a reference kernel): replaces the
 * router's choice for n_tok tokens with K distinct experts drawn from a seeded
 * Zipf(s) popularity over the E experts (weights 1/K); a pure function of
 * (seed, salt, position params[0], token tok0 + i). */
E4B_API int e4b_route_zipf(e4b_ctx* ctx, const uint32_t* params, uint32_t* topk_idx, float* topk_w, int n_tok,
                           int K, int E, float s, uint32_t seed, int salt, int tok0);
/* e4b_route_zipf for nseq x npos position-major rows (a batched-prefill chunk):
 * row i is token tok0 + i % nseq at position params[0] + i / nseq, routed as the
 * token-by-token calls route it. */
E4B_API int e4b_route_zipf_rows(e4b_ctx* ctx, const uint32_t* params, uint32_t* topk_idx, float* topk_w, int nseq,
                                int npos, int K, int E, float s, uint32_t seed, int salt, int tok0);
/* The Zipf(s) popularity table e4b_route_zipf builds per CTA, once into device
 * memory: table[0..E) cumulative popularity by rank, table[E..2E) the seeded
 * rank -> expert permutation (as u32 bits).  It depends on (s, seed, E) only. */
E4B_API int e4b_zipf_table(e4b_ctx* ctx, float* table, int E, float s, uint32_t seed);
/* e4b_route_zipf for every layer of one decode step in one launch: rows
 * (layer l, token i), layer salt salt0 + l, sequence tok0 + i at position
 * params[0]; topk_idx / topk_w [n_layers][n_tok][K]; same draws as
 * e4b_route_zipf with salt = salt0 + l. */
E4B_API int e4b_route_zipf_layers(e4b_ctx* ctx, const uint32_t* params, const float* table, uint32_t* topk_idx,
                                  float* topk_w, int n_tok, int n_layers, int K, int E, uint32_t seed, int salt0,
                                  int tok0);
/* kernels/router.wgsl:16-63: scale-less RMS of h, x scale x H^-0.5, then as routertop. */
E4B_API int e4b_router(e4b_ctx* ctx, const float* h, const float* scale, const float* wr, const float* pes,
                       uint32_t* topk_idx, float* topk_w, int H, int E, int K, float eps);
/* kernels/top8.wgsl:8-30 on precomputed scores. */
E4B_API int e4b_top8(e4b_ctx* ctx, const float* scores, const float* pes, uint32_t* topk_idx, float* topk_w,
                     int E, int K);

/* ------------------------------------------------------------ attention */
/* kernels/headprep.wgsl:19-87: q/k per-head RMSNorm (q_norm/k_norm) + RoPE on
 * pairs (p, p+hd/2) for p < rope_angles; v scale-less RMSNorm (v = k slice when
 * keqv); K/V f16 written at slot pos % ring (cachemode 1) or params[4]+b
 * (cachemode 2); cache layout [cache_slots][KVH][HD].  batch tokens at pos
 * params[0]+b.  A slot >= cache_slots sets the device status word, no write. */
E4B_API int e4b_headprep(e4b_ctx* ctx, const float* qkv, const float* qw, const float* kw, const uint32_t* params,
                         uint16_t* kcache, uint16_t* vcache, float* q_out, int QH, int KVH, int HD,
                         int rope_angles, float theta, float eps, int keqv, int cachemode, int ring,
                         int cache_slots, int batch);
/* kernels/rope.wgsl:8-27 (in place, pos = params[0]). */
E4B_API int e4b_rope(e4b_ctx* ctx, float* x, const uint32_t* params, int heads, int HD, int rope_angles,
                     float theta);
/* The SCORE=1 mass pass of kernels/attnos.wgsl:82-97 for a counted (linear)
 * cache: score[h][t] += exp(scale * q_h . k_t - lse[h]) for t < params[5]; lse
 * from e4b_attcomb.  score: [QH][scap] f32, accumulated over decode steps and
 * read by the host's budget compaction (src/engine-a4b.js:589-617). */
E4B_API int e4b_attn_score(e4b_ctx* ctx, const float* q, const uint16_t* kcache, const float* lse,
                           const uint32_t* params, float* score, int QH, int KVH, int HD, float scale, int scap);
/* kernels/kvgather.wgsl:9-18: dst slot i <- src slot keep[i] (K and V rows of
 * KVH*HD f16) for i < n; keep entries >= src_slots are skipped. */
E4B_API int e4b_kvgather(e4b_ctx* ctx, const uint32_t* keep, int n, const uint16_t* src_k, const uint16_t* src_v,
                         uint16_t* dst_k, uint16_t* dst_v, int KVH, int HD, int src_slots);
/* kernels/kvwrite.wgsl:5-10: dst[params[0]*N + i] = src[i] (f32). */
E4B_API int e4b_kvwrite(e4b_ctx* ctx, const float* src, const uint32_t* params, float* dst, int N);
/* kernels/attsplit.wgsl:16-76 (flash-decode phase A) over the f16 cache.
 * Chunk c of `chunk` positions of head h -> part_o[(h*max_chunks+c)*HD] (unnormalised)
 * and part_ml[2*(h*max_chunks+c)] = (m, l); empty chunks write (-inf, 0).
 * cachemode 1: sliding ring (ring slots, window), query pos params[0];
 * cachemode 2: linear slots [0, params[5]); cachemode 0: linear [0, params[1]),
 * window applied if > 0.  scale multiplies q.k (the Gemma path uses 1.0). */
E4B_API int e4b_attsplit(e4b_ctx* ctx, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                         const uint32_t* params, float* part_o, float* part_ml, int QH, int KVH, int HD,
                         int window, int cachemode, int ring, int chunk, int max_chunks, float scale);
/* kernels/attcomb.wgsl:10-36 (phase B): LSE-merge of the chunk partials ->
 * out_h (f16, may be NULL), out_f (f32, may be NULL), lse (f32, may be NULL). */
E4B_API int e4b_attcomb(e4b_ctx* ctx, const float* part_o, const float* part_ml, uint16_t* out_h, float* out_f,
                        float* lse, int QH, int HD, int max_chunks);

/* ------------------------------------------------------------ GeGLU */
/* kernels/geglumul.wgsl:5-11: y = gelu_tanh(a) * b (f32). */
E4B_API int e4b_geglumul(e4b_ctx* ctx, const float* a, const float* b, float* y, int N);
/* kernels/geglusl.wgsl:5-13: out[k*FF+i] = gelu(gu[k*2FF+i]) * gu[k*2FF+FF+i] (f32). */
E4B_API int e4b_geglusl(e4b_ctx* ctx, const float* gu, float* out, int FF, int K);
/* kernels/geglub.wgsl:9-19: yh[r*N+j] = f16(gelu(gu[r*2N+j]) * gu[r*2N+N+j]), rows r. */
E4B_API int e4b_geglub(e4b_ctx* ctx, const float* gu, uint16_t* yh, int N, int rows);

/* ------------------------------------------------------------ PLE */
/* kernels/pleprep.wgsl:15-46 with a q6_K table: for layer block b,
 * pleIn[b*PD+i] = (rms(proj_b*proj_scale)[i]*normW[i] + row_b[i]*mult) * sqrt(1/2),
 * row = q6_K row tok[0] (toksrc=1) or params[2] of the [LAYERS*PD]-wide table. */
/* LM head for n token rows (batched decode): y[n][OUT] = softcap(W x[n][N]) on the
 * tensor cores, x used as f16 hi + lo; scratch: 2*N*max(64, ceil8(n)) u16, 16-byte
 * aligned (the split activations).  For n <= 64 (and n >= the "lmhead_tc_min"
 * option) and OUT % 8 == 0 the tcgen05 kernel runs, else the mma.sync ones.
 * kernels/q6k.wgsl:75-127 per row. */
E4B_API int e4b_q6k_lmhead_rows(e4b_ctx* ctx, const uint8_t* w, const float* x, uint16_t* scratch, float* y, int N,
                                int OUT, float softcap, int n);
/* Tile-packed copy of a row-major q6_K matrix for e4b_q6k_lmhead_tiles: for
 * tile t = row / 128, superblock sb, row m = row % 128 the 210-byte superblock
 * sits at ((t * N/256 + sb) * 128 + m) * 212, followed by 2 zero bytes (so
 * every entry is 4-byte aligned); rows past OUT are zero.  Size:
 * e4b_q6k_packed_bytes(N, OUT) = ceil(OUT/128) * N/256 * 27136.  Same bytes as
 * the reference's q6_K table (kernels/q6k.wgsl), reordered so that each
 * (tile, superblock) is one contiguous TMA bulk copy. */
E4B_API size_t e4b_q6k_packed_bytes(int N, int OUT);
E4B_API int e4b_q6k_pack_tiles(e4b_ctx* ctx, const uint8_t* w, uint8_t* wt, int N, int OUT);
/* e4b_q6k_lmhead_rows on the tile-packed copy (1 <= n <= 64), weights streamed
 * by bulk copies: n = 1 the warp-MMA GEMV (scratch unused, may be null); n >= 2
 * the warp-MMA kernel over activation slabs built in scratch, or the tcgen05
 * kernel (above 32 rows; option "lmhead_tiles_tc"); scratch: 2*N*64 u16,
 * 16-byte aligned; x 16-byte aligned. */
E4B_API int e4b_q6k_lmhead_tiles(e4b_ctx* ctx, const uint8_t* wt, const float* x, uint16_t* scratch, float* y, int N,
                                 int OUT, float softcap, int n);
E4B_API int e4b_pleprep(e4b_ctx* ctx, const uint8_t* table, const uint32_t* params, const uint32_t* tok,
                        const float* proj, const float* norm_w, float* ple_in, int PD, int LAYERS, int rows,
                        float mult, float proj_scale, float eps, int toksrc);
/* kernels/plegatemv.wgsl:20-60 with q4_0 weights and f16 activations (no int8
 * activation quantisation): y[o] = f16(gelu_tanh(W x)[o] * ple[off+o]). */
E4B_API int e4b_plegatemv(e4b_ctx* ctx, const uint16_t* x, const uint8_t* w, const float* ple, uint16_t* y,
                          int IN, int OUT, int off);
/* kernels/plemul.wgsl:6-12: y[i] = gelu_tanh(a[i]) * ple[off+i]. */
E4B_API int e4b_plemul(e4b_ctx* ctx, const float* a, const float* ple, float* y, int N, int off);

/* ---- batched decode of nseq sequences at one common position (params[0],
 * kvCount params[4]); sequence b's KV cache starts at cache + b * slots*KVH*HD,
 * its q / qkv / partial / output rows are row b of the per-sequence layouts.
 * attcomb_seq xfo=1: out_h rows (QH*HD) in fragment order.  headprep_seq
 * nparts > 1: qkv is the sum of nparts [nseq][rows] partials (e4b_q40mm_kparts). */
E4B_API int e4b_headprep_seq(e4b_ctx* ctx, const float* qkv, const float* qw, const float* kw, const uint32_t* params,
                             uint16_t* kcache, uint16_t* vcache, float* q_out, int QH, int KVH, int HD,
                             int rope_angles, float theta, float eps, int keqv, int cachemode, int ring,
                             int cache_slots, int nseq, int nparts);
/* e4b_headprep_seq for a batched-prefill chunk: nseq x npos position-major
 * rows (row r = sequence r % nseq at position params[0] + r / nseq, linear
 * cache slot params[4] + r / nseq); K/V of every row land in its sequence's
 * cache (kernels/headprep.wgsl:19-87 per row, as encodeLayerPre runs it,
 * src/engine-a4b.js:476-477). */
E4B_API int e4b_headprep_rows(e4b_ctx* ctx, const float* qkv, const float* qw, const float* kw,
                              const uint32_t* params, uint16_t* kcache, uint16_t* vcache, float* q_out, int QH,
                              int KVH, int HD, int rope_angles, float theta, float eps, int keqv, int cachemode,
                              int ring, int cache_slots, int nseq, int npos);
/* Causal attention of a batched-prefill chunk (the reference's per-token
 * attention over a prompt chunk, src/engine-a4b.js:478-479 with attnos.wgsl /
 * attnf32.wgsl semantics): q f32 [npos*nseq][QH][HD] position-major rows (row =
 * p * nseq + b), whose K/V rows are already in the caches; params = the chunk's
 * first position (src/engine-a4b.js:697 layout); query p attends with position
 * params[0] + p and length params[1] + p (params[5] + p for cachemode 2).
 * out f16 [npos*nseq][QH*HD].  QH/KVH must divide 64; for a ring, npos + window
 * <= ring + 1 (no slot a query still needs is overwritten within the chunk). */
E4B_API int e4b_attn_prefill(e4b_ctx* ctx, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                             const uint32_t* params, uint16_t* out, int QH, int KVH, int HD, int window,
                             int cachemode, int ring, float scale, int cache_slots, int nseq, int npos);
E4B_API int e4b_attsplit_seq(e4b_ctx* ctx, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                             const uint32_t* params, float* part_o, float* part_ml, int QH, int KVH, int HD,
                             int window, int cachemode, int ring, int chunk, int max_chunks, float scale,
                             int cache_slots, int nseq);
E4B_API int e4b_attcomb_seq(e4b_ctx* ctx, const float* part_o, const float* part_ml, uint16_t* out_h, float* out_f,
                            float* lse, int QH, int HD, int max_chunks, int nseq, int xfo);
/* attsplit_seq + attcomb_seq in one call for the batched decode, on the tensor
 * cores: work items are (sequence, KV head, 64-slot chunk) over the live chunks
 * only, each KV row is read once for its QH/KVH (<= 8) query heads, and
 * kcache == vcache (keqv layers) loads the shared rows once.  Writes out_h
 * (f16; fragment order when xfo) via part_o / part_ml [nseq][QH][max_chunks]
 * (max_chunks * 64 >= the scanned slots).  HD % 64 == 0, HD <= 256; two launches. */
E4B_API int e4b_attdec_seq(e4b_ctx* ctx, const float* q, const uint16_t* kcache, const uint16_t* vcache,
                           const uint32_t* params, float* part_o, float* part_ml, uint16_t* out_h, int QH, int KVH,
                           int HD, int window, int cachemode, int ring, int max_chunks, float scale, int cache_slots,
                           int nseq, int xfo);

/* ------------------------------------------------------------ argmax / feed */
/* kernels/argmax2.wgsl:8-48 (both stages): out[0] = index of the largest x (ties
 * -> lowest index), out[1] = its f32 bits.  part: scratch of 2*parts u32. */
E4B_API int e4b_argmax(e4b_ctx* ctx, const float* x, uint32_t* part, uint32_t* out, int N, int parts);
/* e4b_argmax without caller scratch (no counterpart in the reference): the
 * partials live in a fixed device array of the library, so the call allocates
 * nothing.  parts must be 1..4096.  The first call on a device looks the array's
 * address up (make it before any stream capture); all such calls on one device
 * share the array, so overlapping calls race. */
E4B_API int e4b_argmax_static(e4b_ctx* ctx, const float* x, uint32_t* out, int N, int parts);
/* kernels/feedtok.wgsl:5-6 plus the token-ring copy (src/engine-a4b.js:820) and
 * the per-token parameter advance (src/engine-a4b.js:793-795), on the device:
 * ring[params[6] % ring_cap] = amax[0]; params[2] = amax[0]; pos/len/kvCount/index += 1. */
E4B_API int e4b_feedtok(e4b_ctx* ctx, const uint32_t* amax, uint32_t* params, uint32_t* ring, int ring_cap);
/* argmax of each of `rows` rows of x[rows][N] -> out[rows][2]; part: 2*parts*rows u32. */
E4B_API int e4b_argmax_rows(e4b_ctx* ctx, const float* x, uint32_t* part, uint32_t* out, int N, int parts, int rows);
/* feedtok for `rows` sequences in lockstep: tok[b] = amax[2b], ring[b][params[6] % ring_cap]
 * = tok[b] (ring may be NULL), params[2] = tok[0]; the shared positions advance once. */
E4B_API int e4b_feedtok_rows(e4b_ctx* ctx, const uint32_t* amax, uint32_t* params, uint32_t* ring, int ring_cap,
                             uint32_t* tok, int rows);

/* ------------------------------------------------------------ fused token plan */
/* One dense (E4B-graph) decoder layer: q4_0 weights as stored in the GGUF
 * (qkv = q|k|v rows back to back, gu = gate|up rows back to back), f32 norm
 * weights, f16 KV cache [slots][KVH][HD]. */
typedef struct {
  const uint8_t* qkv;
  const uint8_t* o;
  const uint8_t* gu;
  const uint8_t* down;
  const uint8_t* ple_gate; /* may be NULL when the model has no per-layer embeddings */
  const uint8_t* ple_proj;
  const float* attn_norm;
  const float* q_norm;
  const float* k_norm;
  const float* post_attn;
  const float* ffn_norm;
  const float* post_ffw;
  const float* post_norm; /* post-PLE norm */
  float scale;            /* layer output scale */
  float theta;
  uint16_t* kcache;
  uint16_t* vcache;
  int sliding, ring, slots, rope_angles, keqv, qkv_rows;
} e4b_dense_layer;

/* The dense model: weights as uploaded from the GGUF, the per-token parameter
 * block, and the outputs the fused plan writes (caller-owned device memory).
 * The plan allocates its own intermediate activations at creation. */
typedef struct {
  int layers, hidden, q_heads, kv_heads, head_dim, ff, vocab, ple_dim, window;
  float eps;
  const uint8_t* token_embd;    /* q6_K [vocab][hidden] */
  const uint8_t* ple_table;     /* q6_K [vocab][layers*ple_dim] (ple_dim > 0) */
  const uint8_t* ple_proj_w;    /* q4_0 [layers*ple_dim][hidden] */
  const float* ple_norm;        /* [ple_dim] */
  const float* out_norm;        /* [hidden] */
  const e4b_dense_layer* layer; /* host array of `layers` entries */
  const uint32_t* params;       /* [8] per-token parameter block (token = params[2]) */
  float* hidden_out;            /* [hidden] residual stream after the last layer */
  float* xf;                    /* [hidden] final-norm output (LM-head input) */
  float* dump;                  /* [layers][hidden] per-layer residual, or NULL */
} e4b_dense_model;

/* Fused token plan.  It has no single counterpart in the reference: one run
 * performs the reference's per-token operator sequence of the dense graph up
 * to the final norm (src/engine.js:282-331; embedding, PLE prep, per layer
 * qkvMv/headprep/attsplit/attcomb/oMv/rmsacc/q40gu/downMv/plegate/proj/rmsacc,
 * final rmsnorm) as one persistent cooperative kernel, one CTA per SM, with
 * grid barriers between dependent steps.  Creation checks the shapes (hidden,
 * q_heads*head_dim, ff and ple_dim multiples of 256; head_dim a multiple of
 * 64), encodes the TMA descriptors and allocates the plan's activations; run
 * enqueues one token on the context stream, reading params[] on the device. */
E4B_API int e4b_dense_plan_create(e4b_ctx* ctx, const e4b_dense_model* model, int* handle);
E4B_API int e4b_dense_plan_run(e4b_ctx* ctx, int handle);
/* Phase timing: with buf non-NULL every later run writes globaltimer stamps
 * (ns) for each phase p into buf[8p .. 8p+7]: CTA 0's start, after its residual
 * step, after its input build, after its GEMV, after its epilogue, the latest
 * "work done" time over all CTAs (atomic max: zero buf before the run), and
 * CTA 0 past the phase's grid barrier, and the time CTA 0's warp 0 spent
 * waiting for weight copies in the phase (attention phases: slots 2-4 are the
 * ends of CTA 0's first item's head prep, scores + softmax, and p.V).  NULL
 * turns it off.
 * e4b_dense_plan_phases returns the number of phases and their kinds: 0 PLE
 * projection, 1 q|k|v, 2 attention, 3 o, 4 gate|up, 5 down, 6 PLE gate, 7 PLE
 * layer projection, 8 final norm. */
E4B_API int e4b_dense_plan_trace(e4b_ctx* ctx, int handle, unsigned long long* buf);
E4B_API int e4b_dense_plan_phases(e4b_ctx* ctx, int handle, int* kinds, int max);
E4B_API int e4b_dense_plan_destroy(e4b_ctx* ctx, int handle);

#ifdef __cplusplus
}
#endif
#endif /* E4B_B200_H */

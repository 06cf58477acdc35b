// Internal interface of the streaming q4_0 GEMV (q40_stream.cu).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace e4b {

// Workspace layout shared by the streaming kernels: a counter area that is
// zero between launches (each split row tile's last CTA resets its counter),
// followed by split-K partials.
constexpr size_t kWsMaxTiles = 16384;                       // u32 counters + u64 start masks
constexpr size_t kWsCounterBytes = kWsMaxTiles * (4 + 8);

// rows: output rows (OUT, or FF for the fused gate|up).
bool q40_stream_supported(const void* w, const void* x, int IN, int rows);
// epi 0: y = W x (f32); 1: gate|up rows [0,ff) and [ff,2ff) -> yh = f16(gelu(g)*u);
// 2: yh = f16(gelu(W x) * ple[off + o]).
int q40_stream(e4b_ctx* c, const uint8_t* w, const void* x, int x_f32, float* y, uint16_t* yh, const float* ple,
               int IN, int OUT, int epi, int ff, int off);

// cuTensorMapEncodeTiled through the runtime's driver entry point (null if absent).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Streaming q6_K LM head (q6k_stream.cu): batch 1, hidden a multiple of 2048.
bool lmhead_stream_supported(const uint8_t* w, const float* x, int N);
int lmhead_stream(e4b_ctx* c, const uint8_t* w, const float* x, float* y, int N, int OUT, float softcap);

// Batched q6_K LM head on tcgen05 (q6tc.cu): n <= 64 token rows; scratch holds
// 2 * 64 * N halves.
bool q6tc_supported(const uint8_t* w, const void* scratch, int N, int OUT, int n);
int q6tc_lmhead(e4b_ctx* c, const uint8_t* w, bool packed, const float* x, uint16_t* scratch, float* y, int N,
                int OUT, float softcap, int n);

}  // namespace e4b

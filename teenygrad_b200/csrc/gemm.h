// Internal linear-layer launch interface shared with the decoder executor.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "tb_internal.h"

namespace tb {

struct Epi {
    void* out;             // y
    int64_t ldo;           // row stride of y (elements)
    const float* bias;     // [N] or null
    const void* resid;     // [M, N] same dtype as y, or null
    int64_t ldr;
    const float* scale;    // int8 per-output-channel scale, or null
    int out_f32;           // y is f32
    int swiglu;            // gate/up interleaved in 128-row blocks
};

// Split-K workspace the decode GEMV needs for (M tokens, N rows, K): bytes of
// f32 partials and the number of tile counters (zero-initialised, left at zero).
void gemv_ws_need(tb_ctx* ctx, int M, int N, int K, size_t* bytes, size_t* counters);

// y = epilogue(x[M,K] w[N,K]^T).  int8 = 1: w is int8 with ep.scale (M <= 64).
// ws / counters: caller-owned split-K scratch (see gemv_ws_need).
int linear_launch(tb_ctx* ctx, int int8, const void* x, const void* w, const Epi& ep, int M, int N, int K,
                  float* ws, size_t ws_bytes, unsigned* counters, size_t n_counters);

}  // namespace tb

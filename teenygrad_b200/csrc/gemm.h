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
    int64_t x_ld;          // row stride of x in elements (0: dense, = K)
    // Optional RMSNorm of x fused into the decode GEMV (tokens <= 64): the
    // GEMV consumes bf16(x * rsqrt(mean(x^2) + eps) * norm_w) instead of x.
    const void* norm_w;    // bf16 [K] or null
    float norm_eps;
    const void* norm_x;    // (set by the launcher) the raw rows x
};

// y = epilogue(x[M,K] w[N,K]^T).  int8 = 1: w is int8 with ep.scale (M <= 64).
// Needs no global scratch: the decode GEMV reduces its K splits in shared
// memory across a thread-block cluster.
int linear_launch(tb_ctx* ctx, int int8, const void* x, const void* w, const Epi& ep, int M, int N, int K);

}  // namespace tb

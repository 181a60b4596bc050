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

// y = epilogue(x[M,K] w[N,K]^T).  int8 = 1: w is int8 with ep.scale (M <= 64).
// Needs no global scratch: the decode GEMV reduces its K splits in shared
// memory across a thread-block cluster.
int linear_launch(tb_ctx* ctx, int int8, const void* x, const void* w, const Epi& ep, int M, int N, int K);

}  // namespace tb

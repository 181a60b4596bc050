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
    // QKV projection with weight rows permuted per 256-row tile so that the
    // row pair (p, p + 128) holds dims (i, i + hd/2) of one head (qkv_perm).
    // perm_hd (gemm_tc): output columns are written back in the natural
    // [heads][hd] order.  rope_tab (decode GEMV): RoPE is applied in the
    // epilogue; q rows go to out in natural order, k and v to the KV cache.
    int perm_hd;
    const float2* rope_tab;   // [max_seq][hd / 2] (cos, sin)
    int rope_hq, rope_hkv;    // query / kv heads
    int rope_s_new;           // tokens per sequence in this call: token m = (m / s_new, m % s_new)
    const int* pos_ptr;       // position of token s = *pos_ptr + s (or pos_host + s if null)
    int pos_host;
    void* kcache;             // bf16 [B][Hkv][max_seq][hd]
    void* vcache;
    int max_seq;
};

// Row permutation of a QKV weight matrix with head_dim hd (256 % hd == 0,
// rows % 256 == 0): natural row r -> stored row.
__host__ __device__ __forceinline__ int64_t qkv_perm_row(int64_t r, int hd) {
    const int64_t t = r / 256, w = r % 256, hh = hd / 2;
    const int64_t j = w / hd, d = w % hd;
    return t * 256 + (d / hh) * 128 + j * hh + (d % hh);
}

// Inverse: stored row (column of the GEMM output) -> natural row.
__host__ __device__ __forceinline__ int64_t qkv_unperm_row(int64_t n, int hd) {
    const int64_t t = n / 256, h = (n % 256) / 128, p = n % 128, hh = hd / 2;
    return t * 256 + (p / hh) * hd + h * hh + (p % hh);
}

// y = epilogue(x[M,K] w[N,K]^T).  int8 = 1: w is int8 with ep.scale (M <= 64).
// Needs no global scratch: the decode GEMV reduces its K splits in shared
// memory across a thread-block cluster.
int linear_launch(tb_ctx* ctx, int int8, const void* x, const void* w, const Epi& ep, int M, int N, int K);

}  // namespace tb

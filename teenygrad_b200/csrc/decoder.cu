// Decoder executor: parameters, KV cache, activation buffers, prefill and
// CUDA-graph decode steps, built from the library's kernels.
#include <math.h>
#include <stdlib.h>

#include <algorithm>
#include <vector>

#include "attention.h"
#include "common.cuh"
#include "decode_chain.h"
#include "gemm.h"

namespace tb {

// ------------------------------------------------------------------ kernels --
// src row i -> dst row (row_off + (i / block) * block_stride + i % block),
// then (perm_hd != 0) through the QKV row permutation of head_dim perm_hd.
__global__ void convert_rows_kernel(const void* __restrict__ src, int src_f32, __nv_bfloat16* __restrict__ dst,
                                    int64_t rows, int64_t cols, int64_t row_off, int64_t block,
                                    int64_t block_stride, int perm_hd) {
    int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / cols, c = i % cols;
        int64_t dr = row_off + (r / block) * block_stride + (r % block);
        if (perm_hd) dr = qkv_perm_row(dr, perm_hd);
        float v = src_f32 ? reinterpret_cast<const float*>(src)[i]
                          : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[i]);
        dst[dr * cols + c] = __float2bfloat16_rn(v);
    }
}

// int8 rows (and their per-row f32 scales) into the decoder's layout, with the
// same row mapping as convert_rows_kernel; scale_dst / scale_src may be null.
__global__ void copy_rows_i8_kernel(const int8_t* __restrict__ src, const float* __restrict__ scale_src,
                                    int8_t* __restrict__ dst, float* __restrict__ scale_dst, int64_t rows, int64_t cols,
                                    int64_t row_off, int64_t block, int64_t block_stride, int perm_hd) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i % cols;
        int64_t dr = row_off + (r / block) * block_stride + (r % block);
        if (perm_hd) dr = qkv_perm_row(dr, perm_hd);
        dst[dr * cols + c] = src[i];
        if (c == 0 && scale_dst) scale_dst[dr] = scale_src[r];
    }
}

// dequantize_affine (teeny-quant quant/affine.rs:151-159) into bf16: int8
// embeddings of a quantised checkpoint become the bf16 gather table.
__global__ void dequant_rows_bf16_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                         __nv_bfloat16* __restrict__ dst, int64_t rows, int64_t cols) {
    const int64_t total = rows * cols;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn((float)q[i] * scale[i / cols]);
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

// Counter-based N(0, std): Box-Muller on two splitmix64 draws of (seed, i).
__global__ void init_normal_kernel(__nv_bfloat16* __restrict__ dst, int64_t n, uint64_t seed, float std) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        uint64_t h1 = splitmix64(seed ^ ((uint64_t)i * 0xD1B54A32D192ED03ull));
        uint64_t h2 = splitmix64(h1 ^ 0x8CB92BA72F3D8DD7ull);
        float u1 = ((float)(h1 >> 40) + 0.5f) * (1.0f / 16777216.0f);
        float u2 = (float)(h2 >> 40) * (1.0f / 16777216.0f);
        dst[i] = __float2bfloat16_rn(std * sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    }
}

// N(0, 1) keys / values for positions [0, len) of `blocks` cache rows blocks
// of max_seq * hd elements each (decode-only workloads).
__global__ void fill_cache_normal_kernel(__nv_bfloat16* __restrict__ base, int blocks, int len, int hd, int max_seq,
                                         uint64_t seed) {
    const int64_t per = (int64_t)len * hd, total = per * blocks;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i / per, off = i % per;
        uint64_t h1 = splitmix64(seed ^ ((uint64_t)i * 0xD1B54A32D192ED03ull));
        uint64_t h2 = splitmix64(h1 ^ 0x8CB92BA72F3D8DD7ull);
        float u1 = ((float)(h1 >> 40) + 0.5f) * (1.0f / 16777216.0f);
        float u2 = (float)(h2 >> 40) * (1.0f / 16777216.0f);
        base[blk * (int64_t)max_seq * hd + off] = __float2bfloat16_rn(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2));
    }
}

__global__ void fill_bf16_kernel(__nv_bfloat16* dst, int64_t n, float v) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __float2bfloat16_rn(v);
}

// Same cos/sin as tb_rope_fwd: inv_freq_i = theta^(-2i/hd), angle = pos * inv_freq_i.
__global__ void rope_table_kernel(float2* tab, int max_seq, int hd, float theta) {
    int half = hd / 2;
    int64_t total = (int64_t)max_seq * half;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += (int64_t)gridDim.x * blockDim.x) {
        int i = (int)(idx % half);
        int pos = (int)(idx / half);
        float inv = powf(theta, -2.0f * (float)i / (float)hd);
        float s, c;
        sincosf((float)pos * inv, &s, &c);
        tab[idx] = make_float2(c, s);
    }
}

// One thread per (token, head slot, 8-element chunk c of the first half):
// it rotates the 16-byte chunks c of both halves (rotate-half pairing).
// Head slots: [0, Hq) query heads (in place in the qkv row), [Hq, Hq+Hkv) key
// heads (written to the K cache), [Hq+Hkv, Hq+2Hkv) value heads (copied to the
// V cache).  Position of token s = base + s, base from device memory when
// pos_dev != 0.
__global__ void rope_kv_kernel(__nv_bfloat16* __restrict__ qkv, int qkv_n, int B, int S_new, int Hq, int Hkv,
                               int hd, const float2* __restrict__ tab, const int* __restrict__ pos_dev,
                               int pos_host, __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc,
                               int max_seq, int* err) {
    pdl_trigger();
    pdl_wait();
    const int nh = Hq + 2 * Hkv;
    const int half = hd / 2, cph = half / 8;        // chunks per half
    const int64_t total = (int64_t)B * S_new * nh * cph;
    const int base = pos_dev ? *pos_dev : pos_host;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(idx % cph);
        const int64_t th = idx / cph;
        const int hh = (int)(th % nh);
        const int64_t t = th / nh;
        const int b = (int)(t / S_new), s = (int)(t % S_new);
        const int pos = base + s;
        if (pos < 0 || pos >= max_seq) {
            atomicOr(err, 1 << 5);
            continue;
        }
        __nv_bfloat16* src = qkv + t * qkv_n + (int64_t)hh * hd;
        uint4* lo = reinterpret_cast<uint4*>(src + 8 * c);
        uint4* hi = reinterpret_cast<uint4*>(src + half + 8 * c);
        if (hh >= Hq + Hkv) {
            __nv_bfloat16* dst = vc + (((int64_t)b * Hkv + (hh - Hq - Hkv)) * max_seq + pos) * hd;
            reinterpret_cast<uint4*>(dst + 8 * c)[0] = *lo;
            reinterpret_cast<uint4*>(dst + half + 8 * c)[0] = *hi;
            continue;
        }
        uint4 va = *lo, vb = *hi;
        uint32_t xa[4] = {va.x, va.y, va.z, va.w}, xb[4] = {vb.x, vb.y, vb.z, vb.w}, oa[4], ob[4];
        const float4* tp = reinterpret_cast<const float4*>(tab + (int64_t)pos * half + 8 * c);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float4 cs = tp[j];   // (cos, sin) of elements 2j, 2j+1
            float a0 = bf16_lo(xa[j]), a1 = bf16_hi(xa[j]), b0 = bf16_lo(xb[j]), b1 = bf16_hi(xb[j]);
            oa[j] = pack_bf16x2(a0 * cs.x - b0 * cs.y, a1 * cs.z - b1 * cs.w);
            ob[j] = pack_bf16x2(b0 * cs.x + a0 * cs.y, b1 * cs.z + a1 * cs.w);
        }
        uint4* dlo = lo;
        uint4* dhi = hi;
        if (hh >= Hq) {
            __nv_bfloat16* dst = kc + (((int64_t)b * Hkv + (hh - Hq)) * max_seq + pos) * hd;
            dlo = reinterpret_cast<uint4*>(dst + 8 * c);
            dhi = reinterpret_cast<uint4*>(dst + half + 8 * c);
        }
        *dlo = make_uint4(oa[0], oa[1], oa[2], oa[3]);
        *dhi = make_uint4(ob[0], ob[1], ob[2], ob[3]);
    }
}

// RMSNorm with an input row stride (last-token gather for the LM head).  One
// warp per row; the row (N <= 4096 bf16) stays in registers: every load is
// issued before the reduction, and the second pass reads no memory.
// MAXC: 16-byte chunks per lane (rows up to 256 * MAXC elements); the smallest that
// fits keeps the registers low enough for more rows in flight per SM.
template <int MAXC>
__global__ void rmsnorm_ld_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ w,
                                  __nv_bfloat16* __restrict__ y, int M, int N, float eps) {
    pdl_trigger();
    const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    uint4 g[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; i++) {
        const int c = (lane + 32 * i) * 8;
        if (c < N) g[i] = __ldg(reinterpret_cast<const uint4*>(w + c));   // weights: before the wait
    }
    pdl_wait();
    if (row >= M) return;
    const __nv_bfloat16* xr = x + (int64_t)row * ldx;
    uint4 v[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; i++) {
        const int c = (lane + 32 * i) * 8;
        if (c < N) v[i] = *reinterpret_cast<const uint4*>(xr + c);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; i++) {
        const int c = (lane + 32 * i) * 8;
        if (c < N) {
            const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float a = bf16_lo(u[j]), b = bf16_hi(u[j]);
                ss += a * a + b * b;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss * (1.0f / (float)N) + eps);
#pragma unroll
    for (int i = 0; i < MAXC; i++) {
        const int c = (lane + 32 * i) * 8;
        if (c < N) {
            const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w}, gw[4] = {g[i].x, g[i].y, g[i].z, g[i].w};
            uint32_t o[4];
#pragma unroll
            for (int j = 0; j < 4; j++)
                o[j] = pack_bf16x2(bf16_lo(u[j]) * r * bf16_lo(gw[j]), bf16_hi(u[j]) * r * bf16_hi(gw[j]));
            *reinterpret_cast<uint4*>(y + (int64_t)row * N + c) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    }
}

__device__ __forceinline__ void amax_merge2(float& v, int& i, float v2, int i2) {
    if (i2 < 0) return;
    if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

// Greedy token per row, lowest index on ties, NaN skipped: one 1024-thread CTA
// per row, every thread with all of its 128-bit loads in flight at once (one
// round for a 32000-entry vocabulary), then a warp and a block reduction, and
// thread 0 writes cur_ids[b] and out_ids[b * max_gen + state[1]].  (A grid of
// row chunks merged through atomics and a last-CTA election took ~7 us after
// the LM head in the decode step, a chain of dependent global round trips; one
// CTA per row takes ~2.)  The (value, index) selection is order-independent, so
// -0.0 and +0.0 tie and the lower index wins, as in the oracle.
constexpr int kArgmaxThreads = 1024, kArgmaxU = 8;
__global__ void __launch_bounds__(kArgmaxThreads)
argmax_step_kernel(const float* __restrict__ logits, int V, int32_t* __restrict__ cur_ids,
                   int32_t* __restrict__ out_ids, int max_gen, const int* __restrict__ state) {
    pdl_trigger();
    pdl_wait();
    const int row = blockIdx.x;
    const float* xr = logits + (int64_t)row * V;
    float bv = -INFINITY;
    int bi = -1;
    if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        const int n4 = V >> 2;
        for (int c0 = threadIdx.x; c0 < n4; c0 += kArgmaxU * kArgmaxThreads) {
            float4 v[kArgmaxU];
#pragma unroll
            for (int u = 0; u < kArgmaxU; u++) {
                const int i4 = c0 + u * kArgmaxThreads;
                v[u] = i4 < n4 ? x4[i4] : make_float4(NAN, NAN, NAN, NAN);
            }
#pragma unroll
            for (int u = 0; u < kArgmaxU; u++) {
                const int c = 4 * (c0 + u * kArgmaxThreads);
                const float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int j = 0; j < 4; j++)
                    if (e[j] == e[j]) amax_merge2(bv, bi, e[j], c + j);
            }
        }
    } else {
        for (int c = threadIdx.x; c < V; c += kArgmaxThreads) {
            const float v = xr[c];
            if (v == v) amax_merge2(bv, bi, v, c);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        amax_merge2(bv, bi, v2, i2);
    }
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kArgmaxThreads / 32; w++) amax_merge2(bv, bi, sv[w], si[w]);
        const int id = bi >= 0 ? bi : 0;
        cur_ids[row] = id;
        const int step = state[1];
        if (step < max_gen) out_ids[(int64_t)row * max_gen + step] = id;
    }
}

__global__ void advance_kernel(int* state, int dpos, int dstep) {
    pdl_trigger();
    pdl_wait();
    state[0] += dpos;
    state[1] += dstep;
}

__global__ void set_state_kernel(int* state, int pos, int step) {
    pdl_trigger();
    pdl_wait();
    state[0] = pos;
    state[1] = step;
}

static int grid_for(tb_ctx* ctx, int64_t n) {
    int64_t b = (n + 255) / 256;
    int64_t cap = (int64_t)ctx->num_sms * 8;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace tb

using namespace tb;
using bf16 = __nv_bfloat16;

struct tb_decoder {
    tb_ctx* ctx = nullptr;
    tb_decoder_config cfg{};
    int q_dim = 0, kv_dim = 0, qkv_n = 0;
    // qkv_n % 256 == 0: the QKV weight rows are stored permuted (qkv_perm_row)
    // so that decode applies RoPE and fills the KV cache in the GEMV epilogue.
    bool qkv_perm = false;
    int64_t max_tokens = 0;
    struct Layer {
        bf16 *attn_norm, *mlp_norm, *wqkv, *wo, *wgu, *wdown;
        int8_t *qqkv = nullptr, *qo = nullptr, *qgu = nullptr, *qdown = nullptr;
        float *sqkv = nullptr, *so = nullptr, *sgu = nullptr, *sdown = nullptr;
        unsigned i8_loaded = 0;   // bit (1 << kind): set from int8 checkpoint tensors, not quantised here
    };
    std::vector<Layer> layers;
    bf16 *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr;
    int8_t* qlm = nullptr;
    float* slm = nullptr;
    bool lm_i8_loaded = false;
    bf16 *kcache = nullptr, *vcache = nullptr;
    int64_t cache_layer_elems = 0;
    float2* rope_tab = nullptr;
    bf16 *x = nullptr, *h = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr;
    float* logits = nullptr;
    int32_t *ids_in = nullptr, *cur_ids = nullptr, *out_ids = nullptr;
    int* state = nullptr;   // [0] tokens in cache, [1] tokens generated
    cudaStream_t cap_stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    // generate(): kGenGraphSteps decode steps captured back to back in one graph,
    // so consecutive steps are chained by programmatic dependent launch instead
    // of paying a graph launch each (~6 us of idle GPU between replays)
    cudaGraphExec_t graph_multi = nullptr;
    int graph_multi_B = 0;
    int graph_B = 0;
    int B = 0;       // batch of the current sequences
    int S0 = 0;      // prompt length
    int host_len = 0, host_step = 0;
    bool quantized = false;
    // Persistent decode chain (bf16 decode): O, gate/up, down and the next
    // layer's QKV projection of each layer run as one launch.
    bool use_chain = false;
    ChainScratch chain;
    std::vector<void*> allocs;

    template <typename T>
    int alloc(T** p, size_t n) {
        void* v = nullptr;
        if (cudaMalloc(&v, n * sizeof(T) + 16) != cudaSuccess) {
            cudaGetLastError();
            return set_error(ctx, TB_ERR_OOM, "decoder: cudaMalloc of %zu bytes failed", n * sizeof(T));
        }
        allocs.push_back(v);
        *p = reinterpret_cast<T*>(v);
        return TB_OK;
    }
};

namespace {

// Enables programmatic dependent launch for the decoder's kernel chain.
struct PdlScope {
    tb_ctx* ctx;
    bool saved;
    explicit PdlScope(tb_ctx* c) : ctx(c), saved(c->pdl) { c->pdl = true; }
    ~PdlScope() { ctx->pdl = saved; }
};

#define TB_TRY(x)          \
    do {                   \
        int rc_ = (x);     \
        if (rc_) return rc_; \
    } while (0)

int lin(tb_decoder* d, const void* x, const void* w, const int8_t* wq, const float* wscale, void* y, int M, int N,
        int K, const void* resid, bool swiglu, bool out_f32, int perm_hd = 0) {
    Epi ep{};
    ep.perm_hd = perm_hd;
    ep.out = y;
    ep.ldo = swiglu ? N / 2 : N;
    ep.resid = resid;
    ep.ldr = N;
    ep.out_f32 = out_f32 ? 1 : 0;
    ep.swiglu = swiglu ? 1 : 0;
    const bool int8 = d->cfg.weights_int8 && wq;
    if (int8) ep.scale = wscale;
    return linear_launch(d->ctx, int8 ? 1 : 0, x, int8 ? (const void*)wq : w, ep, M, N, K);
}

int rms(tb_decoder* d, const bf16* x, int64_t ldx, const bf16* w, bf16* y, int M) {
    const int N = d->cfg.d_model;
    if (N <= 256 * 8)
        return launch(d->ctx, "rmsnorm", rmsnorm_ld_kernel<8>, dim3((M + 7) / 8), dim3(256), 0, x, ldx, w, y, M, N,
                      d->cfg.norm_eps);
    return launch(d->ctx, "rmsnorm", rmsnorm_ld_kernel<16>, dim3((M + 7) / 8), dim3(256), 0, x, ldx, w, y, M, N,
                  d->cfg.norm_eps);
}

// y = rmsnorm(x) W^T.  Up to 64 tokens the norm runs inside the GEMV (its
// otherwise idle warps rescale each activation tile in shared memory), so the
// normalised rows never reach HBM; larger token counts normalise into d->h and
// run the tensor-core GEMM.
int norm_lin(tb_decoder* d, const bf16* x, int64_t ldx, const bf16* norm_w, const void* w, const int8_t* wq,
             const float* wscale, void* y, int M, int N, bool swiglu, bool out_f32, const Epi* qkv = nullptr) {
    const int K = d->cfg.d_model;
    if (M > 64) {
        TB_TRY(rms(d, x, ldx, norm_w, d->h, M));
        if (qkv && qkv->rope_tab) {
            // the QKV GEMM with RoPE and the KV-cache write in its epilogue
            Epi ep = *qkv;
            ep.out = y;
            ep.ldo = N;
            ep.ldr = N;
            const bool int8 = d->cfg.weights_int8 && wq;
            if (int8) ep.scale = wscale;
            return linear_launch(d->ctx, int8 ? 1 : 0, d->h, int8 ? (const void*)wq : w, ep, M, N, K);
        }
        return lin(d, d->h, w, wq, wscale, y, M, N, K, nullptr, swiglu, out_f32, qkv ? qkv->perm_hd : 0);
    }
    Epi ep = qkv ? *qkv : Epi{};
    ep.out = y;
    ep.ldo = swiglu ? N / 2 : N;
    ep.ldr = N;
    ep.out_f32 = out_f32 ? 1 : 0;
    ep.swiglu = swiglu ? 1 : 0;
    ep.x_ld = ldx;
    ep.norm_w = norm_w;
    ep.norm_eps = d->cfg.norm_eps;
    const bool int8 = d->cfg.weights_int8 && wq;
    if (int8) ep.scale = wscale;
    return linear_launch(d->ctx, int8 ? 1 : 0, x, int8 ? (const void*)wq : w, ep, M, N, K);
}

// Decode attention of layer l: one new token per sequence against the cache.
int decode_attention(tb_decoder* d, int l, int B) {
    const tb_decoder_config& c = d->cfg;
    const int hd = c.head_dim;
    const float scale = 1.0f / sqrtf((float)hd);
    bf16* kc = d->kcache + (int64_t)l * d->cache_layer_elems;
    bf16* vc = d->vcache + (int64_t)l * d->cache_layer_elems;
    DecodeArgs a{};
    a.q = d->qkv;
    a.q_sb = d->qkv_n;
    a.q_sh = hd;
    a.k = kc;
    a.v = vc;
    a.kv_sb = (int64_t)c.n_kv_heads * c.max_seq * hd;
    a.kv_sh = (int64_t)c.max_seq * hd;
    a.kv_ss = hd;
    a.kv_rows = c.max_seq;
    a.o = d->attn;
    a.o_sb = d->q_dim;
    a.o_sh = hd;
    a.lse = nullptr;
    a.Hq = c.n_heads;
    a.Hkv = c.n_kv_heads;
    a.len = 1;         // keys = tokens already cached + this one
    a.len_ptr = d->state;
    a.scale_log2 = scale * 1.4426950408889634f;
    return attn_decode_launch(d->ctx, a, B, hd, c.max_seq);
}

// One transformer layer over T = B * S_new tokens.  decode: S_new == 1 and
// positions come from d->state[0].
int layer_forward(tb_decoder* d, int l, int B, int S_new, bool decode) {
    const tb_decoder_config& c = d->cfg;
    tb_ctx* ctx = d->ctx;
    tb_decoder::Layer& L = d->layers[l];
    const int T = B * S_new;
    const int dm = c.d_model, hd = c.head_dim;
    bf16* kc = d->kcache + (int64_t)l * d->cache_layer_elems;
    bf16* vc = d->vcache + (int64_t)l * d->cache_layer_elems;

    // QKV projection.  With permuted QKV weights RoPE and the KV-cache writes
    // happen in the epilogue (the decode GEMV and the prefill GEMM alike);
    // otherwise the projection is written in natural order and rope_kv follows.
    const bool fused_rope = d->qkv_perm;
    Epi qe{};
    if (d->qkv_perm) qe.perm_hd = hd;
    if (fused_rope) {
        qe.rope_tab = d->rope_tab;
        qe.rope_hq = c.n_heads;
        qe.rope_hkv = c.n_kv_heads;
        qe.rope_s_new = S_new;
        qe.pos_ptr = decode ? d->state : nullptr;
        qe.pos_host = 0;
        qe.kcache = kc;
        qe.vcache = vc;
        qe.max_seq = c.max_seq;
    }
    TB_TRY(norm_lin(d, d->x, dm, L.attn_norm, L.wqkv, L.qqkv, L.sqkv, d->qkv, T, d->qkv_n, false, false, &qe));
    if (!fused_rope) {
        const int64_t work = (int64_t)T * (c.n_heads + 2 * c.n_kv_heads) * (hd / 16);
        TB_TRY(launch(ctx, "rope_kv", rope_kv_kernel, dim3(grid_for(ctx, work)), dim3(256), 0, d->qkv, d->qkv_n, B,
                      S_new, c.n_heads, c.n_kv_heads, hd, (const float2*)d->rope_tab,
                      decode ? (const int*)d->state : (const int*)nullptr, 0, kc, vc, c.max_seq, ctx->d_err));
    }
    const float scale = 1.0f / sqrtf((float)hd);
    if (!decode) {
        AttnTensors t{};
        t.q = d->qkv;
        t.q_sh = hd;
        t.q_ss = d->qkv_n;
        t.q_sb = (int64_t)S_new * d->qkv_n;
        t.k = kc;
        t.v = vc;
        t.kv_sh = (int64_t)c.max_seq * hd;
        t.kv_ss = hd;
        t.kv_sb = (int64_t)c.n_kv_heads * c.max_seq * hd;
        t.kv_len_alloc = c.max_seq;
        t.o = d->attn;
        t.o_sh = hd;
        t.o_ss = d->q_dim;
        t.o_sb = (int64_t)S_new * d->q_dim;
        t.lse = nullptr;
        TB_TRY(attn_tc_launch(ctx, t, B, c.n_heads, c.n_kv_heads, S_new, S_new, hd, scale, 1));
    } else {
        TB_TRY(decode_attention(d, l, B));
    }
    TB_TRY(lin(d, d->attn, L.wo, L.qo, L.so, d->x, T, dm, d->q_dim, d->x, false, false));
    TB_TRY(norm_lin(d, d->x, dm, L.mlp_norm, L.wgu, L.qgu, L.sgu, d->act, T, 2 * c.ffn_hidden, true, false));
    TB_TRY(lin(d, d->act, L.wdown, L.qdown, L.sdown, d->x, T, dm, c.ffn_hidden, d->x, false, false));
    return TB_OK;
}

// Final norm on each sequence's last token, LM head, greedy argmax.
int head_forward(tb_decoder* d, int B, int64_t last_row_stride, int64_t last_row_off) {
    const tb_decoder_config& c = d->cfg;
    TB_TRY(norm_lin(d, d->x + last_row_off, last_row_stride, d->final_norm, d->lm_head, d->qlm, d->slm, d->logits, B,
                    c.vocab, false, true));
    return launch(d->ctx, "argmax_step", argmax_step_kernel, dim3(B), dim3(kArgmaxThreads), 0, (const float*)d->logits,
                  c.vocab, d->cur_ids, d->out_ids, c.max_seq, (const int*)d->state);
}

// The decode chain's GEMVs of layer l (one token per sequence, B sequences).
ChainStep chain_qkv(tb_decoder* d, int l) {
    const tb_decoder_config& c = d->cfg;
    const tb_decoder::Layer& L = d->layers[l];
    ChainStep s{};
    s.x = d->x;
    s.x_ld = c.d_model;
    s.w = L.wqkv;
    s.Nw = d->qkv_n;
    s.K = c.d_model;
    Epi& e = s.ep;
    e.out = d->qkv;
    e.ldo = d->qkv_n;
    e.ldr = d->qkv_n;
    e.norm_w = L.attn_norm;
    e.norm_eps = c.norm_eps;
    e.perm_hd = c.head_dim;
    e.rope_tab = d->rope_tab;
    e.rope_hq = c.n_heads;
    e.rope_hkv = c.n_kv_heads;
    e.rope_s_new = 1;
    e.pos_ptr = d->state;
    e.kcache = d->kcache + (int64_t)l * d->cache_layer_elems;
    e.vcache = d->vcache + (int64_t)l * d->cache_layer_elems;
    e.max_seq = c.max_seq;
    return s;
}

ChainStep chain_o(tb_decoder* d, int l) {
    ChainStep s{};
    s.x = d->attn;
    s.x_ld = d->q_dim;
    s.w = d->layers[l].wo;
    s.Nw = d->cfg.d_model;
    s.K = d->q_dim;
    s.ep.out = d->x;
    s.ep.ldo = d->cfg.d_model;
    s.ep.resid = d->x;
    s.ep.ldr = d->cfg.d_model;
    return s;
}

ChainStep chain_gate_up(tb_decoder* d, int l) {
    const tb_decoder_config& c = d->cfg;
    ChainStep s{};
    s.x = d->x;
    s.x_ld = c.d_model;
    s.w = d->layers[l].wgu;
    s.Nw = 2 * c.ffn_hidden;
    s.K = c.d_model;
    s.ep.out = d->act;
    s.ep.ldo = c.ffn_hidden;
    s.ep.ldr = 2 * c.ffn_hidden;
    s.ep.swiglu = 1;
    s.ep.norm_w = d->layers[l].mlp_norm;
    s.ep.norm_eps = c.norm_eps;
    return s;
}

ChainStep chain_down(tb_decoder* d, int l) {
    const tb_decoder_config& c = d->cfg;
    ChainStep s{};
    s.x = d->act;
    s.x_ld = c.ffn_hidden;
    s.w = d->layers[l].wdown;
    s.Nw = c.d_model;
    s.K = c.ffn_hidden;
    s.ep.out = d->x;
    s.ep.ldo = c.d_model;
    s.ep.resid = d->x;
    s.ep.ldr = c.d_model;
    return s;
}

// Whether this decode step runs on the chain: bf16 weights, permuted QKV rows
// and every GEMV's shape within the chain's limits.
bool chain_fits(tb_decoder* d, int B) {
    if (!d->use_chain || B > 64) return false;
    return chain_step_ok(chain_qkv(d, 0), B) && chain_step_ok(chain_o(d, 0), B) &&
           chain_step_ok(chain_gate_up(d, 0), B) && chain_step_ok(chain_down(d, 0), B);
}

int decode_step_body(tb_decoder* d) {
    const int B = d->B;
    const int nl = d->cfg.n_layers;
    TB_TRY(tb_embedding_fwd(d->ctx, TB_BF16, d->embed, d->cur_ids, d->x, B, d->cfg.d_model, d->cfg.vocab));
    if (chain_fits(d, B)) {
        // QKV of layer 0, then per layer: attention, and one chain launch for
        // O, gate/up, down and the next layer's QKV
        ChainStep st[kChainMaxPhases];
        st[0] = chain_qkv(d, 0);
        TB_TRY(chain_launch(d->ctx, st, 1, B, d->chain));
        for (int l = 0; l < nl; l++) {
            TB_TRY(decode_attention(d, l, B));
            st[0] = chain_o(d, l);
            st[1] = chain_gate_up(d, l);
            st[2] = chain_down(d, l);
            int n = 3;
            if (l + 1 < nl) st[n++] = chain_qkv(d, l + 1);
            TB_TRY(chain_launch(d->ctx, st, n, B, d->chain));
        }
    } else {
        for (int l = 0; l < nl; l++) TB_TRY(layer_forward(d, l, B, 1, true));
    }
    TB_TRY(head_forward(d, B, d->cfg.d_model, 0));
    return launch(d->ctx, "advance", advance_kernel, dim3(1), dim3(1), 0, d->state, 1, 1);
}

constexpr int kGenGraphSteps = 8;

// Capture `steps` decode steps into *exec (rebuilt when the batch changes).
int capture_steps(tb_decoder* d, int steps, cudaGraphExec_t* exec, int* exec_B) {
    if (*exec && *exec_B == d->B) return TB_OK;
    if (*exec) {
        cudaGraphExecDestroy(*exec);
        *exec = nullptr;
    }
    tb_ctx* ctx = d->ctx;
    cudaStream_t saved = ctx->stream;
    // order capture after everything already queued on the caller's stream
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(saved));
    ctx->stream = d->cap_stream;
    PdlScope pdl(ctx);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(d->cap_stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) {
        ctx->stream = saved;
        return set_error(ctx, TB_ERR_CUDA, "decode graph: begin capture: %s", cudaGetErrorString(e));
    }
    int rc = TB_OK;
    for (int i = 0; i < steps && !rc; i++) rc = decode_step_body(d);
    e = cudaStreamEndCapture(d->cap_stream, &g);
    ctx->stream = saved;
    if (rc) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "decode graph: end capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "decode graph: instantiate: %s", cudaGetErrorString(e));
    *exec_B = d->B;
    return TB_OK;
}

int ensure_graph(tb_decoder* d) { return capture_steps(d, 1, &d->graph, &d->graph_B); }

}  // namespace

extern "C" {

int tb_decoder_create(tb_ctx* ctx, const tb_decoder_config* cfg, tb_decoder** out) {
    if (!ctx || !cfg || !out) return TB_ERR_ARG;
    *out = nullptr;
    const tb_decoder_config c = *cfg;
    TB_REQUIRE(ctx, c.n_layers > 0 && c.d_model > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.vocab > 0,
               TB_ERR_SHAPE, "decoder: bad config");
    TB_REQUIRE(ctx, c.head_dim == 64 || c.head_dim == 128, TB_ERR_SHAPE, "decoder: head_dim must be 64 or 128");
    TB_REQUIRE(ctx, c.n_heads % c.n_kv_heads == 0 && c.n_heads / c.n_kv_heads <= 8, TB_ERR_SHAPE,
               "decoder: n_heads must be a multiple of n_kv_heads, group <= 8");
    TB_REQUIRE(ctx, c.d_model % 64 == 0 && c.d_model <= 4096 && c.ffn_hidden % 128 == 0 && c.vocab % 8 == 0,
               TB_ERR_SHAPE, "decoder: d_model %% 64 (<= 4096), ffn_hidden %% 128, vocab %% 8 must be 0");
    TB_REQUIRE(ctx, c.max_batch > 0 && c.max_seq > 0, TB_ERR_SHAPE, "decoder: max_batch / max_seq");
    TB_REQUIRE(ctx, !c.weights_int8 || c.max_batch <= 64, TB_ERR_SHAPE, "decoder int8: max_batch <= 64");
    tb_decoder* d = new tb_decoder();
    d->ctx = ctx;
    d->cfg = c;
    d->q_dim = c.n_heads * c.head_dim;
    d->kv_dim = c.n_kv_heads * c.head_dim;
    d->qkv_n = d->q_dim + 2 * d->kv_dim;
    d->qkv_perm = d->qkv_n % 256 == 0;
    d->max_tokens = c.max_prefill_tokens > 0 ? c.max_prefill_tokens : (int64_t)c.max_batch * c.max_seq;
    if (d->max_tokens < c.max_batch) d->max_tokens = c.max_batch;
    const int64_t dm = c.d_model, F = c.ffn_hidden, V = c.vocab;
    int rc = TB_OK;
    auto A = [&](auto** p, size_t n) {
        if (!rc) rc = d->alloc(p, n);
    };
    d->layers.resize(c.n_layers);
    for (auto& L : d->layers) {
        A(&L.attn_norm, dm);
        A(&L.mlp_norm, dm);
        A(&L.wqkv, (size_t)d->qkv_n * dm);
        A(&L.wo, (size_t)dm * d->q_dim);
        A(&L.wgu, (size_t)2 * F * dm);
        A(&L.wdown, (size_t)dm * F);
        if (c.weights_int8) {
            A(&L.qqkv, (size_t)d->qkv_n * dm);
            A(&L.qo, (size_t)dm * d->q_dim);
            A(&L.qgu, (size_t)2 * F * dm);
            A(&L.qdown, (size_t)dm * F);
            A(&L.sqkv, d->qkv_n);
            A(&L.so, dm);
            A(&L.sgu, 2 * F);
            A(&L.sdown, dm);
        }
    }
    A(&d->embed, (size_t)V * dm);
    A(&d->lm_head, (size_t)V * dm);
    A(&d->final_norm, dm);
    if (c.weights_int8) {
        A(&d->qlm, (size_t)V * dm);
        A(&d->slm, V);
    }
    d->cache_layer_elems = (int64_t)c.max_batch * c.n_kv_heads * c.max_seq * c.head_dim;
    A(&d->kcache, (size_t)d->cache_layer_elems * c.n_layers);
    A(&d->vcache, (size_t)d->cache_layer_elems * c.n_layers);
    A(&d->rope_tab, (size_t)c.max_seq * (c.head_dim / 2));
    const int64_t T = d->max_tokens;
    A(&d->x, (size_t)T * dm);
    A(&d->h, (size_t)T * dm);
    A(&d->qkv, (size_t)T * d->qkv_n);
    A(&d->attn, (size_t)T * d->q_dim);
    A(&d->act, (size_t)T * F);
    A(&d->logits, (size_t)c.max_batch * V);
    A(&d->ids_in, (size_t)T);
    A(&d->cur_ids, (size_t)c.max_batch);
    A(&d->out_ids, (size_t)c.max_batch * c.max_seq);
    A(&d->state, 4);
    if (rc) {
        tb_decoder_destroy(d);
        return rc;
    }
    {
        // the decode chain (opt-in, TB_DECODE_CHAIN=1): bf16 weights with permuted
        // QKV rows.  Measured slower than one cluster-reduced GEMV launch per
        // matrix on C4 (its split-K exchange goes through L2 under the weight
        // stream), so the per-GEMV path is the default.
        const char* env = getenv("TB_DECODE_CHAIN");
        if (!c.weights_int8 && d->qkv_perm && c.max_batch <= 64 && env && env[0] == '1') {
            const int cols = (int)std::max<int64_t>(std::max<int64_t>(dm, F), d->qkv_n);
            d->chain.ll_words = chain_ll_words(c.max_batch, cols);
            A(&d->chain.sync, (size_t)kChainSyncWords);
            A(&d->chain.ll, d->chain.ll_words);
            if (rc) {
                tb_decoder_destroy(d);
                return rc;
            }
            cudaMemset(d->chain.sync, 0, kChainSyncWords * sizeof(unsigned));
            cudaMemset(d->chain.ll, 0, d->chain.ll_words * sizeof(uint64_t));
            d->use_chain = true;
        }
    }
    cudaMemset(d->state, 0, 4 * sizeof(int));
    cudaMemset(d->kcache, 0, (size_t)d->cache_layer_elems * c.n_layers * sizeof(bf16));
    cudaMemset(d->vcache, 0, (size_t)d->cache_layer_elems * c.n_layers * sizeof(bf16));
    rope_table_kernel<<<grid_for(ctx, (int64_t)c.max_seq * c.head_dim / 2), 256, 0, ctx->stream>>>(
        d->rope_tab, c.max_seq, c.head_dim, c.rope_theta);
    if (cudaStreamCreateWithFlags(&d->cap_stream, cudaStreamNonBlocking) != cudaSuccess) {
        tb_decoder_destroy(d);
        return set_error(ctx, TB_ERR_CUDA, "decoder: stream create failed");
    }
    rc = check_launch(ctx, "decoder init");
    if (rc) {
        tb_decoder_destroy(d);
        return rc;
    }
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    *out = d;
    return TB_OK;
}

int tb_decoder_destroy(tb_decoder* d) {
    if (!d) return TB_OK;
    cudaSetDevice(d->ctx->device);
    if (d->graph) cudaGraphExecDestroy(d->graph);
    if (d->graph_multi) cudaGraphExecDestroy(d->graph_multi);
    if (d->cap_stream) cudaStreamDestroy(d->cap_stream);
    for (void* p : d->allocs) cudaFree(p);
    delete d;
    return TB_OK;
}

int tb_decoder_set_param(tb_decoder* d, int layer, int kind, const void* src, int src_dtype, int src_on_host) {
    if (!d || !src) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    TB_REQUIRE(ctx, src_dtype == TB_F32 || src_dtype == TB_BF16, TB_ERR_UNSUPPORTED, "set_param: dtype");
    const bool per_layer = kind >= TB_P_ATTN_NORM && kind <= TB_P_W_DOWN;
    TB_REQUIRE(ctx, !per_layer || (layer >= 0 && layer < c.n_layers), TB_ERR_ARG, "set_param: layer %d", layer);
    const int64_t dm = c.d_model, F = c.ffn_hidden;
    bf16* dst = nullptr;
    int64_t rows = 0, cols = dm, row_off = 0, block = 1ll << 40, bstride = 0;
    tb_decoder::Layer* L = per_layer ? &d->layers[layer] : nullptr;
    switch (kind) {
        case TB_P_EMBED: dst = d->embed; rows = c.vocab; break;
        case TB_P_LM_HEAD: dst = d->lm_head; rows = c.vocab; break;
        case TB_P_FINAL_NORM: dst = d->final_norm; rows = 1; break;
        case TB_P_ATTN_NORM: dst = L->attn_norm; rows = 1; break;
        case TB_P_MLP_NORM: dst = L->mlp_norm; rows = 1; break;
        case TB_P_WQ: dst = L->wqkv; rows = d->q_dim; break;
        case TB_P_WK: dst = L->wqkv; rows = d->kv_dim; row_off = d->q_dim; break;
        case TB_P_WV: dst = L->wqkv; rows = d->kv_dim; row_off = d->q_dim + d->kv_dim; break;
        case TB_P_WO: dst = L->wo; rows = dm; cols = d->q_dim; break;
        case TB_P_W_GATE: dst = L->wgu; rows = F; block = 128; bstride = 256; break;
        case TB_P_W_UP: dst = L->wgu; rows = F; row_off = 128; block = 128; bstride = 256; break;
        case TB_P_W_DOWN: dst = L->wdown; rows = dm; cols = F; break;
        default: return set_error(ctx, TB_ERR_ARG, "set_param: kind %d", kind);
    }
    const size_t bytes = (size_t)rows * cols * (src_dtype == TB_F32 ? 4 : 2);
    const void* dsrc = src;
    void* staging = nullptr;
    if (src_on_host) {
        TB_CUDA_TRY(ctx, cudaMalloc(&staging, bytes));
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(staging, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
        dsrc = staging;
    }
    const bool qkv = kind == TB_P_WQ || kind == TB_P_WK || kind == TB_P_WV;
    convert_rows_kernel<<<grid_for(ctx, rows * cols), 256, 0, ctx->stream>>>(dsrc, src_dtype == TB_F32, dst, rows, cols,
                                                                            row_off, block, bstride,
                                                                            qkv && d->qkv_perm ? c.head_dim : 0);
    int rc = check_launch(ctx, "set_param");
    if (staging) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(staging);
    }
    if (L) L->i8_loaded &= ~(1u << kind);
    if (kind == TB_P_LM_HEAD) d->lm_i8_loaded = false;
    d->quantized = false;
    return rc;
}

int tb_decoder_set_param_int8(tb_decoder* d, int layer, int kind, const int8_t* q, const float* scale,
                              int src_on_host) {
    if (!d || !q || !scale) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    const bool per_layer = kind >= TB_P_ATTN_NORM && kind <= TB_P_W_DOWN;
    TB_REQUIRE(ctx, !per_layer || (layer >= 0 && layer < c.n_layers), TB_ERR_ARG, "set_param_int8: layer %d", layer);
    tb_decoder::Layer* L = per_layer ? &d->layers[layer] : nullptr;
    const int64_t dm = c.d_model, F = c.ffn_hidden;
    int8_t* dst = nullptr;
    float* sdst = nullptr;
    bf16* deq = nullptr;   // int8 tensors that the decoder keeps in bf16 (the embedding table)
    int64_t rows = 0, cols = dm, row_off = 0, block = 1ll << 40, bstride = 0;
    switch (kind) {
        case TB_P_EMBED: deq = d->embed; rows = c.vocab; break;
        case TB_P_LM_HEAD: dst = d->qlm; sdst = d->slm; rows = c.vocab; break;
        case TB_P_WQ: dst = L->qqkv; sdst = L->sqkv; rows = d->q_dim; break;
        case TB_P_WK: dst = L->qqkv; sdst = L->sqkv; rows = d->kv_dim; row_off = d->q_dim; break;
        case TB_P_WV: dst = L->qqkv; sdst = L->sqkv; rows = d->kv_dim; row_off = d->q_dim + d->kv_dim; break;
        case TB_P_WO: dst = L->qo; sdst = L->so; rows = dm; cols = d->q_dim; break;
        case TB_P_W_GATE: dst = L->qgu; sdst = L->sgu; rows = F; block = 128; bstride = 256; break;
        case TB_P_W_UP: dst = L->qgu; sdst = L->sgu; rows = F; row_off = 128; block = 128; bstride = 256; break;
        case TB_P_W_DOWN: dst = L->qdown; sdst = L->sdown; rows = dm; cols = F; break;
        default: return set_error(ctx, TB_ERR_ARG, "set_param_int8: kind %d has no int8 form", kind);
    }
    TB_REQUIRE(ctx, deq || c.weights_int8, TB_ERR_UNSUPPORTED,
               "set_param_int8: int8 linear weights need a decoder created with weights_int8");
    const size_t qbytes = (size_t)rows * cols, sbytes = (size_t)rows * sizeof(float);
    const int8_t* dq = q;
    const float* ds = scale;
    void* staging = nullptr;
    if (src_on_host) {
        TB_CUDA_TRY(ctx, cudaMalloc(&staging, qbytes + sbytes + 256));
        uint8_t* sp = reinterpret_cast<uint8_t*>(staging);
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(sp, q, qbytes, cudaMemcpyHostToDevice, ctx->stream));
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(sp + (qbytes + 255) / 256 * 256, scale, sbytes, cudaMemcpyHostToDevice,
                                         ctx->stream));
        dq = reinterpret_cast<const int8_t*>(sp);
        ds = reinterpret_cast<const float*>(sp + (qbytes + 255) / 256 * 256);
    }
    if (deq) {
        dequant_rows_bf16_kernel<<<grid_for(ctx, rows * cols), 256, 0, ctx->stream>>>(dq, ds, deq, rows, cols);
    } else {
        const bool qkv = kind == TB_P_WQ || kind == TB_P_WK || kind == TB_P_WV;
        copy_rows_i8_kernel<<<grid_for(ctx, rows * cols), 256, 0, ctx->stream>>>(
            dq, ds, dst, sdst, rows, cols, row_off, block, bstride, qkv && d->qkv_perm ? c.head_dim : 0);
    }
    int rc = check_launch(ctx, "set_param_int8");
    if (staging) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(staging);
    }
    if (L) L->i8_loaded |= 1u << kind;
    if (kind == TB_P_LM_HEAD) d->lm_i8_loaded = true;
    d->quantized = false;
    return rc;
}

int tb_decoder_init_random(tb_decoder* d, uint64_t seed, float std) {
    if (!d) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    const int64_t dm = c.d_model, F = c.ffn_hidden;
    uint64_t stream_id = 0;
    auto normal = [&](bf16* p, int64_t n) {
        init_normal_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(p, n, seed * 0x100000001B3ull + (++stream_id), std);
    };
    auto ones = [&](bf16* p, int64_t n) { fill_bf16_kernel<<<grid_for(ctx, n), 256, 0, ctx->stream>>>(p, n, 1.0f); };
    for (auto& L : d->layers) {
        ones(L.attn_norm, dm);
        ones(L.mlp_norm, dm);
        normal(L.wqkv, (int64_t)d->qkv_n * dm);
        normal(L.wo, dm * d->q_dim);
        normal(L.wgu, 2 * F * dm);
        normal(L.wdown, dm * F);
    }
    normal(d->embed, (int64_t)c.vocab * dm);
    normal(d->lm_head, (int64_t)c.vocab * dm);
    ones(d->final_norm, dm);
    d->quantized = false;
    return check_launch(ctx, "init_random");
}

int tb_decoder_prepare(tb_decoder* d) {
    if (!d) return TB_ERR_ARG;
    if (!d->cfg.weights_int8 || d->quantized) return TB_OK;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    const int64_t dm = c.d_model, F = c.ffn_hidden;
    // a fused matrix is quantised here from its bf16 values unless all of its
    // parts came in as int8 (tb_decoder_set_param_int8); a mix is an error
    auto need = [&](const tb_decoder::Layer& L, unsigned kinds, const char* what, int l, bool* q) {
        const unsigned got = L.i8_loaded & kinds;
        if (got && got != kinds)
            return set_error(ctx, TB_ERR_ARG, "prepare: layer %d %s mixes int8 and float parts", l, what);
        *q = got == 0;
        return (int)TB_OK;
    };
    for (int l = 0; l < c.n_layers; l++) {
        tb_decoder::Layer& L = d->layers[l];
        bool q;
        TB_TRY(need(L, (1u << TB_P_WQ) | (1u << TB_P_WK) | (1u << TB_P_WV), "QKV", l, &q));
        if (q) TB_TRY(tb_quantize_int8_bf16(ctx, L.wqkv, L.qqkv, L.sqkv, d->qkv_n, dm));
        TB_TRY(need(L, 1u << TB_P_WO, "O", l, &q));
        if (q) TB_TRY(tb_quantize_int8_bf16(ctx, L.wo, L.qo, L.so, dm, d->q_dim));
        TB_TRY(need(L, (1u << TB_P_W_GATE) | (1u << TB_P_W_UP), "gate/up", l, &q));
        if (q) TB_TRY(tb_quantize_int8_bf16(ctx, L.wgu, L.qgu, L.sgu, 2 * F, dm));
        TB_TRY(need(L, 1u << TB_P_W_DOWN, "down", l, &q));
        if (q) TB_TRY(tb_quantize_int8_bf16(ctx, L.wdown, L.qdown, L.sdown, dm, F));
    }
    if (!d->lm_i8_loaded) TB_TRY(tb_quantize_int8_bf16(ctx, d->lm_head, d->qlm, d->slm, c.vocab, dm));
    d->quantized = true;
    return TB_OK;
}

int tb_decoder_prefill(tb_decoder* d, const int32_t* ids, int B, int S, float* logits, int32_t* next_ids) {
    if (!d || !ids) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    TB_REQUIRE(ctx, B > 0 && B <= c.max_batch && S > 0 && S < c.max_seq && (int64_t)B * S <= d->max_tokens,
               TB_ERR_SHAPE, "prefill: B=%d S=%d exceeds the decoder's capacity", B, S);
    TB_REQUIRE(ctx, !c.weights_int8 || (int64_t)B * S <= 64, TB_ERR_UNSUPPORTED,
               "prefill with int8 weights: at most 64 tokens per call");
    TB_REQUIRE(ctx, !c.weights_int8 || d->quantized, TB_ERR_ARG, "int8 decoder: call tb_decoder_prepare first");
    d->B = B;
    d->S0 = S;
    PdlScope pdl(ctx);
    TB_TRY(launch(ctx, "set_state", set_state_kernel, dim3(1), dim3(1), 0, d->state, 0, 0));
    TB_TRY(tb_embedding_fwd(ctx, TB_BF16, d->embed, ids, d->x, (int64_t)B * S, c.d_model, c.vocab));
    for (int l = 0; l < c.n_layers; l++) TB_TRY(layer_forward(d, l, B, S, false));
    TB_TRY(head_forward(d, B, (int64_t)S * c.d_model, (int64_t)(S - 1) * c.d_model));
    TB_TRY(launch(ctx, "advance", advance_kernel, dim3(1), dim3(1), 0, d->state, S, 1));
    d->host_len = S;
    d->host_step = 1;
    if (logits)
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(logits, d->logits, (size_t)B * c.vocab * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
    if (next_ids)
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(next_ids, d->cur_ids, (size_t)B * sizeof(int32_t), cudaMemcpyDeviceToDevice, ctx->stream));
    return TB_OK;
}

int tb_decoder_decode_step(tb_decoder* d, const int32_t* ids, float* logits, int32_t* next_ids) {
    if (!d) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    TB_REQUIRE(ctx, d->B > 0, TB_ERR_ARG, "decode_step: no sequences (call prefill or fill_kv_random)");
    TB_REQUIRE(ctx, d->host_len < c.max_seq, TB_ERR_SHAPE, "decode_step: KV cache full (%d)", c.max_seq);
    TB_REQUIRE(ctx, !c.weights_int8 || d->quantized, TB_ERR_ARG, "int8 decoder: call tb_decoder_prepare first");
    if (ids)
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(d->cur_ids, ids, (size_t)d->B * sizeof(int32_t), cudaMemcpyDeviceToDevice, ctx->stream));
    TB_TRY(ensure_graph(d));
    TB_CUDA_TRY(ctx, cudaGraphLaunch(d->graph, ctx->stream));
    d->host_len++;
    d->host_step++;
    if (logits)
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(logits, d->logits, (size_t)d->B * c.vocab * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream));
    if (next_ids)
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(next_ids, d->cur_ids, (size_t)d->B * sizeof(int32_t), cudaMemcpyDeviceToDevice, ctx->stream));
    return TB_OK;
}

int tb_decoder_generate(tb_decoder* d, const int32_t* prompt_ids, int B, int S, int n_new, int32_t* out_ids) {
    if (!d || !prompt_ids || !out_ids) return TB_ERR_ARG;
    TB_REQUIRE(d->ctx, n_new >= 1 && S + n_new <= d->cfg.max_seq, TB_ERR_SHAPE, "generate: S + n_new > max_seq");
    TB_TRY(tb_decoder_prefill(d, prompt_ids, B, S, nullptr, nullptr));
    int left = n_new - 1;
    if (left >= kGenGraphSteps) TB_TRY(capture_steps(d, kGenGraphSteps, &d->graph_multi, &d->graph_multi_B));
    for (; left >= kGenGraphSteps; left -= kGenGraphSteps) {
        TB_CUDA_TRY(d->ctx, cudaGraphLaunch(d->graph_multi, d->ctx->stream));
        d->host_len += kGenGraphSteps;
        d->host_step += kGenGraphSteps;
    }
    for (; left > 0; left--) TB_TRY(tb_decoder_decode_step(d, nullptr, nullptr, nullptr));
    TB_CUDA_TRY(d->ctx, cudaMemcpy2DAsync(out_ids, (size_t)n_new * sizeof(int32_t), d->out_ids,
                                          (size_t)d->cfg.max_seq * sizeof(int32_t), (size_t)n_new * sizeof(int32_t), B,
                                          cudaMemcpyDeviceToDevice, d->ctx->stream));
    return TB_OK;
}

int tb_decoder_fill_kv_random(tb_decoder* d, int B, int len, uint64_t seed, const int32_t* ids) {
    if (!d || !ids) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    TB_REQUIRE(ctx, B > 0 && B <= c.max_batch && len >= 0 && len < c.max_seq, TB_ERR_SHAPE, "fill_kv_random: B / len");
    // every (layer, b, kv head) row block of the cache: positions [0, len) get N(0,1)
    for (int l = 0; l < c.n_layers; l++) {
        for (int which = 0; which < 2; which++) {
            bf16* base = (which ? d->vcache : d->kcache) + (int64_t)l * d->cache_layer_elems;
            const int blocks = B * c.n_kv_heads;
            fill_cache_normal_kernel<<<grid_for(ctx, (int64_t)blocks * len * c.head_dim), 256, 0, ctx->stream>>>(
                base, blocks, len, c.head_dim, c.max_seq, seed * 0x100000001B3ull + ((uint64_t)l << 8) + which);
        }
    }
    TB_CUDA_TRY(ctx, cudaMemcpyAsync(d->cur_ids, ids, (size_t)B * sizeof(int32_t), cudaMemcpyDeviceToDevice, ctx->stream));
    set_state_kernel<<<1, 1, 0, ctx->stream>>>(d->state, len, 0);
    d->B = B;
    d->S0 = len;
    d->host_len = len;
    d->host_step = 0;
    return check_launch(ctx, "fill_kv_random");
}

int tb_decoder_load_safetensors(tb_decoder* d, tb_st* st) {
    if (!d || !st) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    // Llama checkpoint names (Hugging Face layout) -> parameter kinds
    struct Name {
        int kind;
        const char* fmt;
    };
    static const Name global_names[] = {{TB_P_EMBED, "model.embed_tokens.weight"},
                                        {TB_P_FINAL_NORM, "model.norm.weight"},
                                        {TB_P_LM_HEAD, "lm_head.weight"}};
    static const Name layer_names[] = {{TB_P_ATTN_NORM, "model.layers.%d.input_layernorm.weight"},
                                       {TB_P_WQ, "model.layers.%d.self_attn.q_proj.weight"},
                                       {TB_P_WK, "model.layers.%d.self_attn.k_proj.weight"},
                                       {TB_P_WV, "model.layers.%d.self_attn.v_proj.weight"},
                                       {TB_P_WO, "model.layers.%d.self_attn.o_proj.weight"},
                                       {TB_P_MLP_NORM, "model.layers.%d.post_attention_layernorm.weight"},
                                       {TB_P_W_GATE, "model.layers.%d.mlp.gate_proj.weight"},
                                       {TB_P_W_UP, "model.layers.%d.mlp.up_proj.weight"},
                                       {TB_P_W_DOWN, "model.layers.%d.mlp.down_proj.weight"}};
    const int64_t dm = c.d_model, F = c.ffn_hidden, V = c.vocab;
    auto expected = [&](int kind, int64_t* r, int64_t* k) {
        switch (kind) {
            case TB_P_EMBED: case TB_P_LM_HEAD: *r = V; *k = dm; return 2;
            case TB_P_FINAL_NORM: case TB_P_ATTN_NORM: case TB_P_MLP_NORM: *r = dm; *k = 1; return 1;
            case TB_P_WQ: *r = d->q_dim; *k = dm; return 2;
            case TB_P_WK: case TB_P_WV: *r = d->kv_dim; *k = dm; return 2;
            case TB_P_WO: *r = dm; *k = d->q_dim; return 2;
            case TB_P_W_GATE: case TB_P_W_UP: *r = F; *k = dm; return 2;
            default: *r = dm; *k = F; return 2;   // TB_P_W_DOWN
        }
    };
    auto load_one = [&](int layer, int kind, const char* name) -> int {
        int dt = -1, rank = 4;
        int64_t shape[4] = {0, 0, 0, 0};
        const void* data = nullptr;
        if (tb_st_tensor(st, name, &dt, shape, &rank, &data, nullptr) != TB_OK) {
            if (kind == TB_P_LM_HEAD) return 1;   // tied to the embedding (handled below)
            return set_error(ctx, TB_ERR_ARG, "checkpoint: tensor %s missing", name);
        }
        int64_t r, k;
        const int want = expected(kind, &r, &k);
        if (rank != want || shape[0] != r || (want == 2 && shape[1] != k))
            return set_error(ctx, TB_ERR_SHAPE, "checkpoint: %s has the wrong shape for this decoder", name);
        if (dt == TB_I8) {
            const std::string zname = std::string(name) + "_zero_point";
            if (tb_st_tensor(st, zname.c_str(), nullptr, nullptr, nullptr, nullptr, nullptr) == TB_OK)
                return set_error(ctx, TB_ERR_UNSUPPORTED, "checkpoint: %s is asymmetric int8 (has %s)", name,
                                 zname.c_str());
            const std::string sname = std::string(name) + "_scale";
            int sdt = -1, srank = 1;
            int64_t sshape[1] = {0};
            const void* sdata = nullptr;
            if (tb_st_tensor(st, sname.c_str(), &sdt, sshape, &srank, &sdata, nullptr) != TB_OK || sdt != TB_F32 ||
                srank != 1 || sshape[0] != r)
                return set_error(ctx, TB_ERR_SHAPE,
                                 "checkpoint: %s is I8 but %s is not an F32 scale per output channel (only "
                                 "symmetric per-channel int8 is supported)",
                                 name, sname.c_str());
            return tb_decoder_set_param_int8(d, layer, kind, reinterpret_cast<const int8_t*>(data),
                                             reinterpret_cast<const float*>(sdata), 1);
        }
        if (dt != TB_F32 && dt != TB_BF16)
            return set_error(ctx, TB_ERR_UNSUPPORTED, "checkpoint: %s: dtype not F32, BF16 or I8", name);
        return tb_decoder_set_param(d, layer, kind, data, dt, 1);
    };
    bool tied = false;
    for (const Name& n : global_names) {
        const int rc = load_one(0, n.kind, n.fmt);
        if (rc == 1) tied = true;
        else if (rc) return rc;
    }
    char buf[256];
    for (int l = 0; l < c.n_layers; l++)
        for (const Name& n : layer_names) {
            snprintf(buf, sizeof(buf), n.fmt, l);
            TB_TRY(load_one(l, n.kind, buf));
        }
    if (tied) {   // no lm_head.weight: the output projection shares the embedding table
        TB_CUDA_TRY(ctx, cudaMemcpyAsync(d->lm_head, d->embed, (size_t)V * dm * sizeof(bf16), cudaMemcpyDeviceToDevice,
                                         ctx->stream));
        d->lm_i8_loaded = false;
    }
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    return tb_decoder_prepare(d);
}

int tb_decoder_read_kv(tb_decoder* d, int layer, int B, int len, void* k_out, void* v_out) {
    if (!d || !k_out || !v_out) return TB_ERR_ARG;
    tb_ctx* ctx = d->ctx;
    const tb_decoder_config& c = d->cfg;
    TB_REQUIRE(ctx, layer >= 0 && layer < c.n_layers && B > 0 && B <= c.max_batch && len > 0 && len <= c.max_seq,
               TB_ERR_SHAPE, "read_kv: layer %d, B %d, len %d", layer, B, len);
    // cache rows [b][kv head][max_seq][hd] -> [b][kv head][len][hd]
    const size_t row = (size_t)len * c.head_dim * sizeof(bf16), pitch = (size_t)c.max_seq * c.head_dim * sizeof(bf16);
    const int64_t off = (int64_t)layer * d->cache_layer_elems;
    TB_CUDA_TRY(ctx, cudaMemcpy2DAsync(k_out, row, d->kcache + off, pitch, row, (size_t)B * c.n_kv_heads,
                                       cudaMemcpyDeviceToDevice, ctx->stream));
    TB_CUDA_TRY(ctx, cudaMemcpy2DAsync(v_out, row, d->vcache + off, pitch, row, (size_t)B * c.n_kv_heads,
                                       cudaMemcpyDeviceToDevice, ctx->stream));
    return TB_OK;
}

int tb_decoder_seq_len(tb_decoder* d, int* len) {
    if (!d || !len) return TB_ERR_ARG;
    *len = d->host_len;
    return TB_OK;
}

}  // extern "C"

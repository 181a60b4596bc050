// Bandwidth-bound kernels: RMSNorm, LayerNorm, activations, SwiGLU, residual
// add, int8 quantise/dequantise, embedding gather, argmax, RoPE.
//
// All of them move 16-byte vectors per thread (8 bf16 or 4 f32), reduce rows
// with warp shuffles, and compute in f32.
#include <float.h>
#include <math.h>

#include "common.cuh"

namespace tb {

template <typename T>
struct V16;
template <>
struct V16<float> {
    static constexpr int N = 4;
    __device__ static void load(const float* p, float* v) {
        float4 a = *reinterpret_cast<const float4*>(p);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    }
    __device__ static void store(float* p, const float* v) {
        *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    }
};
template <>
struct V16<__nv_bfloat16> {
    static constexpr int N = 8;
    __device__ static void load(const __nv_bfloat16* p, float* v) {
        uint4 a = *reinterpret_cast<const uint4*>(p);
        uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[2 * i] = bf16_lo(w[i]);
            v[2 * i + 1] = bf16_hi(w[i]);
        }
    }
    __device__ static void store(__nv_bfloat16* p, const float* v) {
        uint4 a;
        a.x = pack_bf16x2(v[0], v[1]);
        a.y = pack_bf16x2(v[2], v[3]);
        a.z = pack_bf16x2(v[4], v[5]);
        a.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(p) = a;
    }
};

__device__ __forceinline__ float to_f(float x) { return x; }
__device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x);
template <>
__device__ __forceinline__ float from_f<float>(float x) { return x; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ------------------------------------------------------------------ norms --
// One warp per row.  Pass 1 accumulates sum(x^2) (rmsnorm.rs:61-80), pass 2
// re-reads the row (from L1) and writes x * rrms * w (rmsnorm.rs:86-121).
template <typename T, bool VEC>
__global__ void rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y,
                               float* __restrict__ rrms, int64_t M, int64_t N, float eps) {
    constexpr int V = V16<T>::N;
    int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (row >= M) return;
    const T* xr = x + row * N;
    T* yr = y + row * N;
    float ss = 0.f;
    if (VEC) {
        for (int64_t c = (int64_t)lane * V; c < N; c += 32 * V) {
            float v[V];
            V16<T>::load(xr + c, v);
#pragma unroll
            for (int i = 0; i < V; i++) ss += v[i] * v[i];
        }
    } else {
        for (int64_t c = lane; c < N; c += 32) {
            float v = to_f(xr[c]);
            ss += v * v;
        }
    }
    ss = warp_sum(ss);
    float r = rsqrtf(ss * (1.0f / (float)N) + eps);
    if (rrms && lane == 0) rrms[row] = r;
    if (VEC) {
        for (int64_t c = (int64_t)lane * V; c < N; c += 32 * V) {
            float v[V], g[V];
            V16<T>::load(xr + c, v);
            V16<T>::load(w + c, g);
#pragma unroll
            for (int i = 0; i < V; i++) v[i] = v[i] * r * g[i];
            V16<T>::store(yr + c, v);
        }
    } else {
        for (int64_t c = lane; c < N; c += 32) yr[c] = from_f<T>(to_f(xr[c]) * r * to_f(w[c]));
    }
}

// One warp per row: mean, centred variance, affine (layernorm.rs:57-156).
template <typename T, bool VEC>
__global__ void layernorm_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                 const T* __restrict__ b, T* __restrict__ y, int64_t M, int64_t N,
                                 float eps) {
    constexpr int V = V16<T>::N;
    int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (row >= M) return;
    const T* xr = x + row * N;
    T* yr = y + row * N;
    float s = 0.f;
    if (VEC) {
        for (int64_t c = (int64_t)lane * V; c < N; c += 32 * V) {
            float v[V];
            V16<T>::load(xr + c, v);
#pragma unroll
            for (int i = 0; i < V; i++) s += v[i];
        }
    } else {
        for (int64_t c = lane; c < N; c += 32) s += to_f(xr[c]);
    }
    float mean = warp_sum(s) * (1.0f / (float)N);
    float vs = 0.f;
    if (VEC) {
        for (int64_t c = (int64_t)lane * V; c < N; c += 32 * V) {
            float v[V];
            V16<T>::load(xr + c, v);
#pragma unroll
            for (int i = 0; i < V; i++) {
                float d = v[i] - mean;
                vs += d * d;
            }
        }
    } else {
        for (int64_t c = lane; c < N; c += 32) {
            float d = to_f(xr[c]) - mean;
            vs += d * d;
        }
    }
    float rstd = rsqrtf(warp_sum(vs) * (1.0f / (float)N) + eps);
    if (VEC) {
        for (int64_t c = (int64_t)lane * V; c < N; c += 32 * V) {
            float v[V], g[V], bb[V];
            V16<T>::load(xr + c, v);
            V16<T>::load(w + c, g);
            V16<T>::load(b + c, bb);
#pragma unroll
            for (int i = 0; i < V; i++) v[i] = (v[i] - mean) * rstd * g[i] + bb[i];
            V16<T>::store(yr + c, v);
        }
    } else {
        for (int64_t c = lane; c < N; c += 32)
            yr[c] = from_f<T>((to_f(xr[c]) - mean) * rstd * to_f(w[c]) + to_f(b[c]));
    }
}

// ------------------------------------------------------------ elementwise --
__device__ __forceinline__ float act_f(int kind, float x) {
    switch (kind) {
        case TB_ACT_SILU: return x / (1.0f + expf(-x));
        case TB_ACT_GELU_TANH:
            return x / (1.0f + expf(-2.0f * 0.7978845608028654f * (x + 0.044715f * x * x * x)));
        case TB_ACT_RELU: return x > 0.f ? x : 0.f;
        case TB_ACT_SIGMOID: return 1.0f / (1.0f + expf(-x));
        default: return x;
    }
}

// op: 0 act(a), 1 silu(a) * b, 2 a + b
template <typename T, int OP>
__global__ void ew_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ y,
                          int64_t n, int kind) {
    constexpr int V = V16<T>::N;
    int64_t nv = n / V;
    int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += stride) {
        float va[V], vb[V];
        V16<T>::load(a + i * V, va);
        if (OP != 0) V16<T>::load(b + i * V, vb);
#pragma unroll
        for (int j = 0; j < V; j++) {
            if (OP == 0) va[j] = act_f(kind, va[j]);
            else if (OP == 1) va[j] = act_f(TB_ACT_SILU, va[j]) * vb[j];
            else va[j] = va[j] + vb[j];
        }
        V16<T>::store(y + i * V, va);
    }
    // scalar tail
    for (int64_t i = nv * V + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float va = to_f(a[i]);
        float r;
        if (OP == 0) r = act_f(kind, va);
        else if (OP == 1) r = act_f(TB_ACT_SILU, va) * to_f(b[i]);
        else r = va + to_f(b[i]);
        y[i] = from_f<T>(r);
    }
}

// ------------------------------------------------------------------- int8 --
// One CTA per output channel.  Pass 1: min / max (affine.rs:91-101); scale =
// amax == 0 ? 1 : amax / 127 in IEEE f32 (:103-112); pass 2: q = clamp(
// roundf(x / scale), -127, 127) (:135-143).  roundf rounds half away from zero
// like Rust's f32::round; `/` is IEEE division (no fast-math in this build).
// Rust's `as i32` saturates and sends NaN to 0, so NaN / scale (and Inf / Inf
// when a row holds +Inf) quantises to 0 and +-Inf / finite to +-127.
template <typename T>
__global__ void quantize_int8_kernel(const T* __restrict__ w, int8_t* __restrict__ q,
                                     float* __restrict__ scale, int64_t K) {
    int64_t n = blockIdx.x;
    const T* wr = w + n * K;
    float vmin = INFINITY, vmax = -INFINITY;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
        float v = to_f(wr[k]);
        vmin = fminf(vmin, v);
        vmax = fmaxf(vmax, v);
    }
    __shared__ float smin[32], smax[32];
    __shared__ float s_scale;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        vmin = fminf(vmin, __shfl_xor_sync(0xffffffffu, vmin, o));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, o));
    }
    int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    if (lane == 0) {
        smin[warp] = vmin;
        smax[warp] = vmax;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float mn = smin[0], mx = smax[0];
        for (int i = 1; i < (int)(blockDim.x / 32); i++) {
            mn = fminf(mn, smin[i]);
            mx = fmaxf(mx, smax[i]);
        }
        float lo = 0.f, hi = 0.f;
        if (isfinite(mn)) {
            lo = fminf(mn, 0.f);
            hi = fmaxf(mx, 0.f);
        }
        float amax = fmaxf(fabsf(lo), fabsf(hi));
        float s = (amax == 0.f) ? 1.0f : __fdiv_rn(amax, 127.0f);
        s_scale = s;
        scale[n] = s;
    }
    __syncthreads();
    float s = s_scale;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
        const float t = __fdiv_rn(to_f(wr[k]), s);
        const float r = t != t ? 0.f : fminf(fmaxf(roundf(t), -127.f), 127.f);
        q[n * K + k] = (int8_t)(int)r;
    }
}

__global__ void dequantize_int8_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                       float* __restrict__ w, int64_t N, int64_t K) {
    int64_t total = N * K;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x)
        w[i] = (float)q[i] * scale[i / K];
}

// -------------------------------------------------------------- embedding --
template <typename T>
__global__ void embedding_kernel(const T* __restrict__ table, const int32_t* __restrict__ ids,
                                 T* __restrict__ y, int64_t T_, int64_t D, int64_t vocab, int* err) {
    pdl_trigger();
    pdl_wait();
    int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (t >= T_) return;
    int64_t id = ids[t];
    bool ok = id >= 0 && id < vocab;
    if (!ok && lane == 0) atomicOr(err, 1 << 4);
    const uint4* src = reinterpret_cast<const uint4*>(table + (ok ? id : 0) * D);
    uint4* dst = reinterpret_cast<uint4*>(y + t * D);
    int64_t nv = D * (int64_t)sizeof(T) / 16;
    for (int64_t i = lane; i < nv; i += 32) dst[i] = ok ? src[i] : make_uint4(0, 0, 0, 0);
}

// ----------------------------------------------------------------- argmax --
// One CTA per row.  (value, index) pairs reduce with "greater value, or equal
// value and lower index"; NaN is skipped (the oracle's or_argmax).
__device__ __forceinline__ void amax_merge(float& v, int& i, float v2, int i2) {
    if (i2 < 0) return;
    if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
        v = v2;
        i = i2;
    }
}

template <typename T>
__global__ void argmax_kernel(const T* __restrict__ x, int32_t* __restrict__ out, int64_t N) {
    const T* xr = x + (int64_t)blockIdx.x * N;
    float bv = -INFINITY;
    int bi = -1;
    for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
        float v = to_f(xr[c]);
        if (v != v) continue;
        amax_merge(bv, bi, v, (int)c);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        amax_merge(bv, bi, v2, i2);
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x / 32); w++) amax_merge(bv, bi, sv[w], si[w]);
        out[blockIdx.x] = bi < 0 ? 0 : bi;
    }
}

// ------------------------------------------------------------------- rope --
// Rotate-half pairing (d, d + D/2); inv_freq_i = theta^(-2i/D).
template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, const int32_t* __restrict__ pos, T* __restrict__ y,
                            int64_t T_, int H, int D, float theta) {
    int half = D / 2;
    int64_t total = T_ * H * half;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        int i = (int)(idx % half);
        int64_t th = idx / half;
        int64_t t = th / H;
        float inv = powf(theta, -2.0f * (float)i / (float)D);
        float s, c;
        sincosf((float)pos[t] * inv, &s, &c);
        const T* xr = x + th * D;
        T* yr = y + th * D;
        float a = to_f(xr[i]), b = to_f(xr[i + half]);
        yr[i] = from_f<T>(a * c - b * s);
        yr[i + half] = from_f<T>(b * c + a * s);
    }
}

static int ew_grid(tb_ctx* ctx, int64_t work, int threads) {
    int64_t blocks = (work + threads - 1) / threads;
    int64_t cap = (int64_t)ctx->num_sms * 16;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

template <int OP>
int launch_ew(tb_ctx* ctx, int dtype, const void* a, const void* b, void* y, int64_t n, int kind) {
    if (n < 0) return set_error(ctx, TB_ERR_SHAPE, "elementwise: n < 0");
    if (n == 0) return TB_OK;
    bool al = aligned16(a) && aligned16(y) && (OP == 0 || aligned16(b));
    if (!al) return set_error(ctx, TB_ERR_ALIGN, "elementwise: pointers must be 16-byte aligned");
    int threads = 256;
    if (dtype == TB_F32) {
        ew_kernel<float, OP><<<ew_grid(ctx, n / 4 + 1, threads), threads, 0, ctx->stream>>>((const float*)a, (const float*)b, (float*)y, n, kind);
    } else if (dtype == TB_BF16) {
        using B = __nv_bfloat16;
        ew_kernel<B, OP><<<ew_grid(ctx, n / 8 + 1, threads), threads, 0, ctx->stream>>>((const B*)a, (const B*)b, (B*)y, n, kind);
    } else {
        return set_error(ctx, TB_ERR_UNSUPPORTED, "elementwise: dtype %d", dtype);
    }
    return check_launch(ctx, "elementwise");
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_rmsnorm_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, void* y, float* rrms,
                   int64_t M, int64_t N, float eps) {
    if (!ctx || !x || !w || !y) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0, TB_ERR_SHAPE, "rmsnorm: bad shape M=%lld N=%lld", (long long)M, (long long)N);
    if (M == 0) return TB_OK;
    int threads = 256;
    int blocks = (int)((M + 7) / 8);
    bool vec = aligned16(x) && aligned16(w) && aligned16(y);
    if (dtype == TB_F32) {
        vec = vec && N % 4 == 0;
        if (vec) rmsnorm_kernel<float, true><<<blocks, threads, 0, ctx->stream>>>((const float*)x, (const float*)w, (float*)y, rrms, M, N, eps);
        else rmsnorm_kernel<float, false><<<blocks, threads, 0, ctx->stream>>>((const float*)x, (const float*)w, (float*)y, rrms, M, N, eps);
    } else if (dtype == TB_BF16) {
        vec = vec && N % 8 == 0;
        using B = __nv_bfloat16;
        if (vec) rmsnorm_kernel<B, true><<<blocks, threads, 0, ctx->stream>>>((const B*)x, (const B*)w, (B*)y, rrms, M, N, eps);
        else rmsnorm_kernel<B, false><<<blocks, threads, 0, ctx->stream>>>((const B*)x, (const B*)w, (B*)y, rrms, M, N, eps);
    } else {
        return set_error(ctx, TB_ERR_UNSUPPORTED, "rmsnorm: dtype %d", dtype);
    }
    return check_launch(ctx, "rmsnorm");
}

int tb_layernorm_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const void* b, void* y,
                     int64_t M, int64_t N, float eps) {
    if (!ctx || !x || !w || !b || !y) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0, TB_ERR_SHAPE, "layernorm: bad shape");
    if (M == 0) return TB_OK;
    int threads = 256;
    int blocks = (int)((M + 7) / 8);
    bool vec = aligned16(x) && aligned16(w) && aligned16(b) && aligned16(y);
    if (dtype == TB_F32) {
        vec = vec && N % 4 == 0;
        if (vec) layernorm_kernel<float, true><<<blocks, threads, 0, ctx->stream>>>((const float*)x, (const float*)w, (const float*)b, (float*)y, M, N, eps);
        else layernorm_kernel<float, false><<<blocks, threads, 0, ctx->stream>>>((const float*)x, (const float*)w, (const float*)b, (float*)y, M, N, eps);
    } else if (dtype == TB_BF16) {
        vec = vec && N % 8 == 0;
        using B = __nv_bfloat16;
        if (vec) layernorm_kernel<B, true><<<blocks, threads, 0, ctx->stream>>>((const B*)x, (const B*)w, (const B*)b, (B*)y, M, N, eps);
        else layernorm_kernel<B, false><<<blocks, threads, 0, ctx->stream>>>((const B*)x, (const B*)w, (const B*)b, (B*)y, M, N, eps);
    } else {
        return set_error(ctx, TB_ERR_UNSUPPORTED, "layernorm: dtype %d", dtype);
    }
    return check_launch(ctx, "layernorm");
}

int tb_act_fwd(tb_ctx* ctx, int act, int dtype, const void* x, void* y, int64_t n) {
    if (!ctx || !x || !y) return TB_ERR_ARG;
    if (act < TB_ACT_SILU || act > TB_ACT_SIGMOID) return set_error(ctx, TB_ERR_ARG, "act: kind %d", act);
    return launch_ew<0>(ctx, dtype, x, nullptr, y, n, act);
}

int tb_swiglu_fwd(tb_ctx* ctx, int dtype, const void* gate, const void* up, void* y, int64_t n) {
    if (!ctx || !gate || !up || !y) return TB_ERR_ARG;
    return launch_ew<1>(ctx, dtype, gate, up, y, n, 0);
}

int tb_add_fwd(tb_ctx* ctx, int dtype, const void* a, const void* b, void* y, int64_t n) {
    if (!ctx || !a || !b || !y) return TB_ERR_ARG;
    return launch_ew<2>(ctx, dtype, a, b, y, n, 0);
}

int tb_quantize_int8(tb_ctx* ctx, const float* w, int8_t* q, float* scale, int64_t N, int64_t K) {
    if (!ctx || !w || !q || !scale) return TB_ERR_ARG;
    TB_REQUIRE(ctx, N >= 0 && K > 0 && N < (1ll << 31), TB_ERR_SHAPE, "quantize: bad shape");
    if (N == 0) return TB_OK;
    quantize_int8_kernel<float><<<(unsigned)N, 256, 0, ctx->stream>>>(w, q, scale, K);
    return check_launch(ctx, "quantize_int8");
}

int tb_quantize_int8_bf16(tb_ctx* ctx, const void* w, int8_t* q, float* scale, int64_t N, int64_t K) {
    if (!ctx || !w || !q || !scale) return TB_ERR_ARG;
    TB_REQUIRE(ctx, N >= 0 && K > 0 && N < (1ll << 31), TB_ERR_SHAPE, "quantize: bad shape");
    if (N == 0) return TB_OK;
    quantize_int8_kernel<__nv_bfloat16><<<(unsigned)N, 256, 0, ctx->stream>>>((const __nv_bfloat16*)w, q, scale, K);
    return check_launch(ctx, "quantize_int8_bf16");
}

int tb_dequantize_int8(tb_ctx* ctx, const int8_t* q, const float* scale, float* w, int64_t N, int64_t K) {
    if (!ctx || !w || !q || !scale) return TB_ERR_ARG;
    TB_REQUIRE(ctx, N >= 0 && K > 0, TB_ERR_SHAPE, "dequantize: bad shape");
    if (N == 0) return TB_OK;
    dequantize_int8_kernel<<<ew_grid(ctx, N * K, 256), 256, 0, ctx->stream>>>(q, scale, w, N, K);
    return check_launch(ctx, "dequantize_int8");
}

int tb_embedding_fwd(tb_ctx* ctx, int dtype, const void* table, const int32_t* ids, void* y,
                     int64_t T, int64_t D, int64_t vocab) {
    if (!ctx || !table || !ids || !y) return TB_ERR_ARG;
    int64_t eb = dtype == TB_F32 ? 4 : (dtype == TB_BF16 ? 2 : 0);
    if (!eb) return set_error(ctx, TB_ERR_UNSUPPORTED, "embedding: dtype %d", dtype);
    TB_REQUIRE(ctx, (D * eb) % 16 == 0 && aligned16(table) && aligned16(y), TB_ERR_ALIGN,
               "embedding: rows must be 16-byte multiples and aligned");
    if (T == 0) return TB_OK;
    int blocks = (int)((T + 7) / 8);
    if (dtype == TB_F32)
        return launch(ctx, "embedding", embedding_kernel<float>, dim3(blocks), dim3(256), 0, (const float*)table, ids,
                      (float*)y, T, D, vocab, ctx->d_err);
    return launch(ctx, "embedding", embedding_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0,
                  (const __nv_bfloat16*)table, ids, (__nv_bfloat16*)y, T, D, vocab, ctx->d_err);
}

int tb_argmax_fwd(tb_ctx* ctx, int dtype, const void* x, int32_t* out, int64_t M, int64_t N) {
    if (!ctx || !x || !out) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0 && N < (1ll << 31) && M < (1ll << 31), TB_ERR_SHAPE, "argmax: bad shape");
    if (M == 0) return TB_OK;
    if (dtype == TB_F32)
        argmax_kernel<float><<<(unsigned)M, 512, 0, ctx->stream>>>((const float*)x, out, N);
    else if (dtype == TB_BF16)
        argmax_kernel<__nv_bfloat16><<<(unsigned)M, 512, 0, ctx->stream>>>((const __nv_bfloat16*)x, out, N);
    else
        return set_error(ctx, TB_ERR_UNSUPPORTED, "argmax: dtype %d", dtype);
    return check_launch(ctx, "argmax");
}

int tb_rope_fwd(tb_ctx* ctx, int dtype, const void* x, const int32_t* pos, void* y, int64_t T, int H,
                int D, float theta) {
    if (!ctx || !x || !pos || !y) return TB_ERR_ARG;
    TB_REQUIRE(ctx, D > 0 && D % 2 == 0 && H > 0 && T >= 0, TB_ERR_SHAPE, "rope: bad shape");
    if (T == 0) return TB_OK;
    int64_t work = T * H * (D / 2);
    if (dtype == TB_F32)
        rope_kernel<float><<<ew_grid(ctx, work, 256), 256, 0, ctx->stream>>>((const float*)x, pos, (float*)y, T, H, D, theta);
    else if (dtype == TB_BF16)
        rope_kernel<__nv_bfloat16><<<ew_grid(ctx, work, 256), 256, 0, ctx->stream>>>((const __nv_bfloat16*)x, pos, (__nv_bfloat16*)y, T, H, D, theta);
    else
        return set_error(ctx, TB_ERR_UNSUPPORTED, "rope: dtype %d", dtype);
    return check_launch(ctx, "rope");
}

}  // extern "C"

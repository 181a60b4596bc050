// Backward kernels for the training executor: RMSNorm, linear, attention and
// conv2d gradients (the reference's rms_norm_backward, linear_backward,
// flash_attention2_backward_dq / _dkv and conv2d_backward).
//
//  * RMSNorm: one warp per row computes dx (the row stays in L1 for the second
//    pass); dw is a column reduction over the rows, split over CTAs into f32
//    partials (workspace) that a second launch adds in split order.
//  * linear: dx = dy w and dw = dy^T x run on the tensor-core GEMM (bf16) or
//    the exact f32 GEMM, dy^T written once into the workspace by a tiled
//    transpose; db is the same column reduction as RMSNorm's dw.
//  * attention: f32 math on CUDA cores.  delta_i = O_i . dO_i first (workspace);
//    dQ: one warp per query row, a lane per key for the scores, lanes over the
//    head dims for the accumulation; dK / dV: one warp per key row over every
//    query of the kv head's group (GQA), causal mask j <= i + Sk - Sq.
//  * conv2d: dx gathered per input element (no atomics); dw reduced per
//    (c_out, c_in) pair by one CTA over all output pixels, taps in registers.
// Every reduction is in a fixed order: results are deterministic.
#include <math.h>

#include "common.cuh"
#include "gemm.h"

namespace tb {

template <typename T>
__device__ __forceinline__ float ldf(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ldf<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ldf<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
    return __bfloat162float(p[i]);
}
__device__ __forceinline__ void stf(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

// ------------------------------------------------------------ RMSNorm ------
// dx[m,n] = rrms[m] * (w[n] dy[m,n] - x[m,n] rrms[m]^2 dot[m] / N),
// dot[m] = sum_n dy w x.  One warp per row.
template <typename T>
__global__ void __launch_bounds__(256) rmsnorm_bwd_dx_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                             const T* __restrict__ w, const float* __restrict__ rrms,
                                                             T* __restrict__ dx, int64_t M, int64_t N) {
    const int64_t row = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= M) return;
    const T* dr = dy + row * N;
    const T* xr = x + row * N;
    float dot = 0.f;
    for (int64_t n = lane; n < N; n += 32) dot += ldf(dr, n) * ldf(w, n) * ldf(xr, n);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    const float r = rrms[row];
    const float c = r * r * dot / (float)N;
    for (int64_t n = lane; n < N; n += 32) stf(dx + row * N, n, r * (ldf(w, n) * ldf(dr, n) - ldf(xr, n) * c));
}

// Column sums over rows [r0, r1) of a[m,n] (* b[m,n] * rs[m] when b is given):
// grid (ceil(N / 64), S); 256 threads = 4 row lanes x 64 columns; the 4 lanes
// combine in fixed order; partial[split][n] (f32).
template <typename T>
__global__ void __launch_bounds__(256) colsum_partial_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                             const float* __restrict__ rs, float* __restrict__ part,
                                                             int64_t M, int64_t N, int64_t rows_per_split) {
    __shared__ float red[4][64];
    const int c = threadIdx.x & 63, rl = threadIdx.x >> 6;
    const int64_t n = (int64_t)blockIdx.x * 64 + c;
    const int64_t r0 = (int64_t)blockIdx.y * rows_per_split;
    const int64_t r1 = r0 + rows_per_split < M ? r0 + rows_per_split : M;
    float acc = 0.f;
    if (n < N)
        for (int64_t m = r0 + rl; m < r1; m += 4) {
            float v = ldf(a, m * N + n);
            if (b) v *= ldf(b, m * N + n) * rs[m];
            acc += v;
        }
    red[rl][c] = acc;
    __syncthreads();
    if (rl == 0 && n < N) part[(int64_t)blockIdx.y * N + n] = ((red[0][c] + red[1][c]) + red[2][c]) + red[3][c];
}

// out[n] (+)= sum over splits of part[s][n], in split order.
__global__ void colsum_final_kernel(const float* __restrict__ part, float* __restrict__ out, int64_t N, int S,
                                    int accumulate) {
    const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    float acc = 0.f;
    for (int s = 0; s < S; s++) acc += part[(int64_t)s * N + n];
    out[n] = accumulate ? out[n] + acc : acc;
}

// Splits of the column reduction: about two CTAs per SM of a 148-SM part, at
// least 32 rows per split.  A function of the shape only, so the workspace
// query needs no device.
static int colsum_splits(int64_t M, int64_t N) {
    const int64_t tiles = (N + 63) / 64;
    int64_t s = (296 + tiles - 1) / tiles;
    const int64_t maxs = (M + 31) / 32;
    if (s > maxs) s = maxs;
    if (s > 64) s = 64;
    return (int)(s < 1 ? 1 : s);
}

template <typename T>
static int colsum(tb_ctx* ctx, const T* a, const T* b, const float* rs, float* out, int64_t M, int64_t N,
                  float* part, int accumulate) {
    const int S = colsum_splits(M, N);
    const int64_t rps = (M + S - 1) / S;
    int rc = launch(ctx, "colsum_partial", colsum_partial_kernel<T>, dim3((unsigned)((N + 63) / 64), (unsigned)S),
                    dim3(256), 0, a, b, rs, part, M, N, rps);
    if (rc) return rc;
    return launch(ctx, "colsum_final", colsum_final_kernel, dim3((unsigned)((N + 255) / 256)), dim3(256), 0,
                  (const float*)part, out, N, S, accumulate);
}

static size_t colsum_ws_bytes(int64_t M, int64_t N) { return (size_t)colsum_splits(M, N) * (size_t)N * 4; }

// ------------------------------------------------------------- linear -------
// 32 x 32 tiles through shared memory: out[c, r] = in[r, c], in [R, C].
template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T* __restrict__ in, T* __restrict__ out, int64_t R,
                                                        int64_t C) {
    __shared__ T t[32][33];
    const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8)
        if (r0 + i < R && c0 + tx < C) t[i][tx] = in[(r0 + i) * C + c0 + tx];
    __syncthreads();
    for (int i = ty; i < 32; i += 8)
        if (c0 + i < C && r0 + tx < R) out[(c0 + i) * R + r0 + tx] = t[tx][i];
}

static size_t round256(size_t b) { return (b + 255) / 256 * 256; }

static size_t linear_bwd_ws(int dtype, int64_t M, int64_t N) {
    const size_t esz = dtype == TB_F32 ? 4 : 2;
    return round256((size_t)M * N * esz) + colsum_ws_bytes(M, N);
}

// ---------------------------------------------------------- attention -------
template <typename T>
__global__ void __launch_bounds__(256) attn_delta_kernel(const T* __restrict__ o, const T* __restrict__ dout,
                                                         float* __restrict__ delta, int64_t rows, int D) {
    const int64_t row = (int64_t)blockIdx.x * 8 + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    float acc = 0.f;
    for (int d = lane; d < D; d += 32) acc += ldf(o, row * D + d) * ldf(dout, row * D + d);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) delta[row] = acc;
}

// dQ: one warp per query row (b, h, i).  Keys go 32 at a time, lane j taking
// key j's scores (q.k_j, dO.v_j from the row staged in shared memory); the
// accumulation dq[d] += dS_j k_j[d] spreads the dims over the lanes.
template <typename T>
__global__ void __launch_bounds__(256) attn_bwd_dq_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                          const T* __restrict__ v, const T* __restrict__ dout,
                                                          const float* __restrict__ lse, const float* __restrict__ delta,
                                                          T* __restrict__ dq, int B, int Hq, int Hkv, int Sq, int Sk,
                                                          int D, float scale, int causal) {
    __shared__ float sq[8][128], sdo[8][128];
    const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + w;
    const bool live = row < (int64_t)B * Hq * Sq;
    const int i = live ? (int)(row % Sq) : 0;
    const int h = live ? (int)((row / Sq) % Hq) : 0;
    const int b = live ? (int)(row / ((int64_t)Sq * Hq)) : 0;
    if (live)
        for (int d = lane; d < D; d += 32) {
            sq[w][d] = ldf(q, row * D + d);
            sdo[w][d] = ldf(dout, row * D + d);
        }
    __syncwarp();
    if (!live) return;
    const int hk = h / (Hq / Hkv);
    const T* kb = k + ((int64_t)b * Hkv + hk) * Sk * D;
    const T* vb = v + ((int64_t)b * Hkv + hk) * Sk * D;
    int jmax = causal ? i + (Sk - Sq) : Sk - 1;
    if (jmax > Sk - 1) jmax = Sk - 1;
    const float L = lse[row], Dl = delta[row];
    float acc[4] = {0.f, 0.f, 0.f, 0.f};   // dims lane + 32 t (D <= 128)
    for (int j0 = 0; j0 <= jmax; j0 += 32) {
        const int j = j0 + lane;
        float ds = 0.f;
        if (j <= jmax) {
            float s = 0.f, dp = 0.f;
            for (int d = 0; d < D; d++) {
                s += sq[w][d] * ldf(kb, (int64_t)j * D + d);
                dp += sdo[w][d] * ldf(vb, (int64_t)j * D + d);
            }
            const float p = expf(s * scale - L);
            ds = p * (dp - Dl);
        }
        const int nj = jmax - j0 + 1 < 32 ? jmax - j0 + 1 : 32;
        for (int t = 0; t < nj; t++) {
            const float dst = __shfl_sync(0xffffffffu, ds, t);
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int d = lane + 32 * u;
                if (d < D) acc[u] += dst * ldf(kb, (int64_t)(j0 + t) * D + d);
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int d = lane + 32 * u;
        if (d < D) stf(dq, row * D + d, acc[u] * scale);
    }
}

// dK, dV: one warp per key row (b, hk, j); over the G query heads of the
// group and their queries i >= j - (Sk - Sq) (causal), 32 at a time (lane per
// query for p and dS), dims over the lanes for the accumulations.
template <typename T>
__global__ void __launch_bounds__(256) attn_bwd_dkv_kernel(const T* __restrict__ q, const T* __restrict__ k,
                                                           const T* __restrict__ v, const T* __restrict__ dout,
                                                           const float* __restrict__ lse,
                                                           const float* __restrict__ delta, T* __restrict__ dk,
                                                           T* __restrict__ dv, int B, int Hq, int Hkv, int Sq, int Sk,
                                                           int D, float scale, int causal) {
    __shared__ float sk[8][128], sv[8][128];
    const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + w;   // (b, hk, j)
    const bool live = row < (int64_t)B * Hkv * Sk;
    const int j = live ? (int)(row % Sk) : 0;
    const int hk = live ? (int)((row / Sk) % Hkv) : 0;
    const int b = live ? (int)(row / ((int64_t)Sk * Hkv)) : 0;
    if (live)
        for (int d = lane; d < D; d += 32) {
            sk[w][d] = ldf(k, row * D + d);
            sv[w][d] = ldf(v, row * D + d);
        }
    __syncwarp();
    if (!live) return;
    const int G = Hq / Hkv;
    int i0 = causal ? j - (Sk - Sq) : 0;
    if (i0 < 0) i0 = 0;
    float ak[4] = {0.f, 0.f, 0.f, 0.f}, av[4] = {0.f, 0.f, 0.f, 0.f};
    for (int h = hk * G; h < (hk + 1) * G; h++) {
        const int64_t qrow0 = ((int64_t)b * Hq + h) * Sq;
        for (int ib = i0; ib < Sq; ib += 32) {
            const int i = ib + lane;
            float p = 0.f, ds = 0.f;
            if (i < Sq) {
                const T* qr = q + (qrow0 + i) * D;
                const T* dr = dout + (qrow0 + i) * D;
                float s = 0.f, dp = 0.f;
                for (int d = 0; d < D; d++) {
                    s += ldf(qr, d) * sk[w][d];
                    dp += ldf(dr, d) * sv[w][d];
                }
                p = expf(s * scale - lse[qrow0 + i]);
                ds = p * (dp - delta[qrow0 + i]);
            }
            const int ni = Sq - ib < 32 ? Sq - ib : 32;
            for (int t = 0; t < ni; t++) {
                const float pt = __shfl_sync(0xffffffffu, p, t), dst = __shfl_sync(0xffffffffu, ds, t);
                const int64_t r = (qrow0 + ib + t) * D;
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int d = lane + 32 * u;
                    if (d < D) {
                        av[u] += pt * ldf(dout, r + d);
                        ak[u] += dst * ldf(q, r + d);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int d = lane + 32 * u;
        if (d < D) {
            stf(dk, row * D + d, ak[u] * scale);
            stf(dv, row * D + d, av[u]);
        }
    }
}

// -------------------------------------------------------------- conv2d ------
// dx[b,ci,ih,iw] = sum_{co,kh,kw} dy[b,co,oh,ow] w[co,ci,kh,kw] over the taps
// with oh * stride + kh - pad == ih and ow * stride + kw - pad == iw.
template <typename T>
__global__ void __launch_bounds__(256) conv_bwd_dx_kernel(const T* __restrict__ dy, const T* __restrict__ w,
                                                          T* __restrict__ dx, int B, int Cin, int Cout, int H, int W,
                                                          int KH, int KW, int stride, int pad, int OH, int OW) {
    const int64_t total = (int64_t)B * Cin * H * W;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int iw = (int)(e % W), ih = (int)((e / W) % H);
        const int ci = (int)((e / ((int64_t)W * H)) % Cin), b = (int)(e / ((int64_t)W * H * Cin));
        float acc = 0.f;
        for (int kh = 0; kh < KH; kh++) {
            const int th = ih + pad - kh;
            if (th < 0 || th % stride) continue;
            const int oh = th / stride;
            if (oh >= OH) continue;
            for (int kw = 0; kw < KW; kw++) {
                const int tw = iw + pad - kw;
                if (tw < 0 || tw % stride) continue;
                const int ow = tw / stride;
                if (ow >= OW) continue;
                for (int co = 0; co < Cout; co++)
                    acc += ldf(dy, (((int64_t)b * Cout + co) * OH + oh) * OW + ow) *
                           ldf(w, (((int64_t)co * Cin + ci) * KH + kh) * KW + kw);
            }
        }
        stf(dx, e, acc);
    }
}

// dw[co,ci,:,:]: one CTA per (co, ci); each thread walks output pixels and
// keeps the KH*KW (<= 49) tap sums in registers; taps are reduced over the
// CTA in a fixed tree order.
template <typename T>
__global__ void __launch_bounds__(256) conv_bwd_dw_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                          T* __restrict__ dw, int B, int Cin, int Cout, int H, int W,
                                                          int KH, int KW, int stride, int pad, int OH, int OW) {
    constexpr int MAXT = 49;
    __shared__ float red[256];
    const int co = blockIdx.x / Cin, ci = blockIdx.x % Cin;
    const int taps = KH * KW;
    float acc[MAXT];
#pragma unroll
    for (int t = 0; t < MAXT; t++) acc[t] = 0.f;
    const int64_t pix = (int64_t)B * OH * OW;
    for (int64_t p = threadIdx.x; p < pix; p += blockDim.x) {
        const int ow = (int)(p % OW), oh = (int)((p / OW) % OH), b = (int)(p / ((int64_t)OW * OH));
        const float g = ldf(dy, (((int64_t)b * Cout + co) * OH + oh) * OW + ow);
        const T* xb = x + ((int64_t)b * Cin + ci) * H * W;
#pragma unroll
        for (int t = 0; t < MAXT; t++) {
            if (t < taps) {
                const int kh = t / KW, kw = t % KW;
                const int ih = oh * stride + kh - pad, iw = ow * stride + kw - pad;
                if (ih >= 0 && ih < H && iw >= 0 && iw < W) acc[t] += g * ldf(xb, (int64_t)ih * W + iw);
            }
        }
    }
    for (int t = 0; t < taps; t++) {
        float v = 0.f;
#pragma unroll
        for (int u = 0; u < MAXT; u++)
            if (u == t) v = acc[u];
        red[threadIdx.x] = v;
        __syncthreads();
        for (int s = 128; s > 0; s >>= 1) {
            if ((int)threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
            __syncthreads();
        }
        if (threadIdx.x == 0) stf(dw, (((int64_t)co * Cin + ci) * KH) * KW + t, red[0]);
        __syncthreads();
    }
}

template <typename T>
static int attn_bwd_launch(tb_ctx* ctx, const T* q, const T* k, const T* v, const T* o, const T* dout,
                           const float* lse, float* delta, T* dq, T* dk, T* dv, int B, int Hq, int Hkv, int Sq, int Sk,
                           int D, float scale, int causal) {
    const int64_t qrows = (int64_t)B * Hq * Sq, krows = (int64_t)B * Hkv * Sk;
    if (qrows) {
        int rc = launch(ctx, "attn_delta", attn_delta_kernel<T>, dim3((unsigned)((qrows + 7) / 8)), dim3(256), 0, o,
                        dout, delta, qrows, D);
        if (rc) return rc;
        rc = launch(ctx, "attn_bwd_dq", attn_bwd_dq_kernel<T>, dim3((unsigned)((qrows + 7) / 8)), dim3(256), 0, q, k,
                    v, dout, lse, (const float*)delta, dq, B, Hq, Hkv, Sq, Sk, D, scale, causal);
        if (rc) return rc;
    }
    if (krows)
        return launch(ctx, "attn_bwd_dkv", attn_bwd_dkv_kernel<T>, dim3((unsigned)((krows + 7) / 8)), dim3(256), 0, q,
                      k, v, dout, lse, (const float*)delta, dk, dv, B, Hq, Hkv, Sq, Sk, D, scale, causal);
    return TB_OK;
}

static int grid_for_elems(tb_ctx* ctx, int64_t n) {
    const int64_t b = (n + 255) / 256, cap = (int64_t)ctx->num_sms * 16;
    return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

int linear_launch(tb_ctx* ctx, int int8, const void* x, const void* w, const Epi& ep, int M, int N, int K);

}  // namespace tb

using namespace tb;

extern "C" {

int tb_rmsnorm_bwd(tb_ctx* ctx, int dtype, const void* dy, const void* x, const void* w, const float* rrms, void* dx,
                   float* dw, int64_t M, int64_t N, void* workspace, size_t workspace_bytes) {
    if (!ctx || !dy || !x || !w || !rrms || !dx) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0, TB_ERR_SHAPE, "rmsnorm_bwd: M=%lld N=%lld", (long long)M, (long long)N);
    if (dtype != TB_F32 && dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "rmsnorm_bwd: dtype %d", dtype);
    if (M == 0) return TB_OK;
    const size_t need = dw ? colsum_ws_bytes(M, N) : 0;
    TB_REQUIRE(ctx, !dw || (workspace && workspace_bytes >= need), TB_ERR_ARG,
               "rmsnorm_bwd: workspace of %zu bytes required (tb_workspace_bytes)", need);
    const dim3 grid((unsigned)((M + 7) / 8));
    int rc;
    if (dtype == TB_F32)
        rc = launch(ctx, "rmsnorm_bwd", rmsnorm_bwd_dx_kernel<float>, grid, dim3(256), 0, (const float*)dy,
                    (const float*)x, (const float*)w, rrms, (float*)dx, M, N);
    else
        rc = launch(ctx, "rmsnorm_bwd", rmsnorm_bwd_dx_kernel<__nv_bfloat16>, grid, dim3(256), 0,
                    (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, rrms,
                    (__nv_bfloat16*)dx, M, N);
    if (rc || !dw) return rc;
    if (dtype == TB_F32)
        return colsum(ctx, (const float*)dy, (const float*)x, rrms, dw, M, N, (float*)workspace, 1);
    return colsum(ctx, (const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, rrms, dw, M, N, (float*)workspace, 1);
}

int tb_linear_bwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const void* dy, void* dx, void* dw, float* db,
                  int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes) {
    if (!ctx || !x || !w || !dy) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31), TB_ERR_SHAPE,
               "linear_bwd: bad shape");
    if (dtype != TB_F32 && dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "linear_bwd: dtype %d", dtype);
    if (M == 0) return TB_OK;
    if (dtype == TB_BF16)
        TB_REQUIRE(ctx, M % 8 == 0 && N % 8 == 0 && K % 8 == 0, TB_ERR_SHAPE,
                   "linear_bwd bf16: M, N and K must be multiples of 8");
    const size_t need = linear_bwd_ws(dtype, M, N);
    TB_REQUIRE(ctx, workspace && workspace_bytes >= need, TB_ERR_ARG,
               "linear_bwd: workspace of %zu bytes required (tb_workspace_bytes)", need);
    const size_t esz = dtype == TB_F32 ? 4 : 2;
    void* dyT = workspace;
    float* part = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + round256((size_t)M * N * esz));
    // dx = dy w: c[M, K] = a[M, N] b[N, K]
    if (dx) {
        const int rc = tb_matmul_fwd(ctx, dtype, dy, w, dx, M, K, N);
        if (rc) return rc;
    }
    // dw = dy^T x: c[N, K] = dyT[N, M] x[M, K]
    if (dw) {
        const dim3 tg((unsigned)((N + 31) / 32), (unsigned)((M + 31) / 32));
        int rc = dtype == TB_F32 ? launch(ctx, "transpose", transpose_kernel<float>, tg, dim3(256), 0,
                                          (const float*)dy, (float*)dyT, M, N)
                                 : launch(ctx, "transpose", transpose_kernel<__nv_bfloat16>, tg, dim3(256), 0,
                                          (const __nv_bfloat16*)dy, (__nv_bfloat16*)dyT, M, N);
        if (rc) return rc;
        rc = tb_matmul_fwd(ctx, dtype, dyT, x, dw, N, K, M);
        if (rc) return rc;
    }
    if (db) {
        if (dtype == TB_F32)
            return colsum(ctx, (const float*)dy, (const float*)nullptr, nullptr, db, M, N, part, 0);
        return colsum(ctx, (const __nv_bfloat16*)dy, (const __nv_bfloat16*)nullptr, nullptr, db, M, N, part, 0);
    }
    return TB_OK;
}

int tb_attn_bwd(tb_ctx* ctx, int dtype, const void* q, const void* k, const void* v, const void* o, const void* dout,
                const float* lse, void* dq, void* dk, void* dv, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                float scale, int causal, void* workspace, size_t workspace_bytes) {
    if (!ctx || !q || !k || !v || !o || !dout || !lse || !dq || !dk || !dv) return TB_ERR_ARG;
    TB_REQUIRE(ctx, B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Sq >= 0 && Sk >= 0 && D > 0 && D <= 128,
               TB_ERR_SHAPE, "attn_bwd: bad shape (D <= 128, Hq %% Hkv == 0)");
    if (dtype != TB_F32 && dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "attn_bwd: dtype %d", dtype);
    const int64_t qrows = (int64_t)B * Hq * Sq, krows = (int64_t)B * Hkv * Sk;
    if (qrows == 0 && krows == 0) return TB_OK;
    const size_t need = (size_t)qrows * 4;
    TB_REQUIRE(ctx, workspace && workspace_bytes >= need, TB_ERR_ARG,
               "attn_bwd: workspace of %zu bytes required (tb_workspace_bytes)", need);
    float* delta = reinterpret_cast<float*>(workspace);
    if (dtype == TB_F32)
        return attn_bwd_launch(ctx, (const float*)q, (const float*)k, (const float*)v, (const float*)o,
                               (const float*)dout, lse, delta, (float*)dq, (float*)dk, (float*)dv, B, Hq, Hkv, Sq, Sk, D,
                               scale, causal);
    using T = __nv_bfloat16;
    return attn_bwd_launch(ctx, (const T*)q, (const T*)k, (const T*)v, (const T*)o, (const T*)dout, lse, delta, (T*)dq,
                           (T*)dk, (T*)dv, B, Hq, Hkv, Sq, Sk, D, scale, causal);
}

int tb_conv2d_bwd(tb_ctx* ctx, int dtype, const void* dy, const void* x, const void* w, void* dx, void* dw, int B,
                  int Cin, int Cout, int H, int W, int KH, int KW, int stride, int pad) {
    if (!ctx || !dy || !x || !w) return TB_ERR_ARG;
    TB_REQUIRE(ctx, B >= 0 && Cin > 0 && Cout > 0 && H > 0 && W > 0 && KH > 0 && KW > 0 && KH * KW <= 49 &&
                        stride > 0 && pad >= 0 && H + 2 * pad >= KH && W + 2 * pad >= KW,
               TB_ERR_SHAPE, "conv2d_bwd: bad shape (KH * KW <= 49)");
    if (dtype != TB_F32 && dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "conv2d_bwd: dtype %d", dtype);
    if (B == 0) return TB_OK;
    const int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (dx) {
        const int g = grid_for_elems(ctx, (int64_t)B * Cin * H * W);
        const int rc = dtype == TB_F32
                           ? launch(ctx, "conv_bwd_dx", conv_bwd_dx_kernel<float>, dim3(g), dim3(256), 0,
                                    (const float*)dy, (const float*)w, (float*)dx, B, Cin, Cout, H, W, KH, KW, stride,
                                    pad, OH, OW)
                           : launch(ctx, "conv_bwd_dx", conv_bwd_dx_kernel<__nv_bfloat16>, dim3(g), dim3(256), 0,
                                    (const __nv_bfloat16*)dy, (const __nv_bfloat16*)w, (__nv_bfloat16*)dx, B, Cin, Cout,
                                    H, W, KH, KW, stride, pad, OH, OW);
        if (rc) return rc;
    }
    if (dw)
        return dtype == TB_F32 ? launch(ctx, "conv_bwd_dw", conv_bwd_dw_kernel<float>, dim3((unsigned)(Cout * Cin)),
                                        dim3(256), 0, (const float*)dy, (const float*)x, (float*)dw, B, Cin, Cout, H,
                                        W, KH, KW, stride, pad, OH, OW)
                               : launch(ctx, "conv_bwd_dw", conv_bwd_dw_kernel<__nv_bfloat16>,
                                        dim3((unsigned)(Cout * Cin)), dim3(256), 0, (const __nv_bfloat16*)dy,
                                        (const __nv_bfloat16*)x, (__nv_bfloat16*)dw, B, Cin, Cout, H, W, KH, KW, stride,
                                        pad, OH, OW);
    return TB_OK;
}

// Workspace bytes of the backward ops (the forward ones are answered in ctx.cu).
int tb_backward_workspace_bytes(int op, int dtype, const int64_t* shape, int n_shape, size_t* bytes) {
    if (!bytes) return TB_ERR_ARG;
    *bytes = 0;
    switch (op) {
        case TB_OP_RMSNORM_BWD:   // {M, N}
            if (!shape || n_shape != 2) return TB_ERR_ARG;
            *bytes = colsum_ws_bytes(shape[0], shape[1]);
            return TB_OK;
        case TB_OP_LINEAR_BWD:    // {M, N, K}
            if (!shape || n_shape != 3) return TB_ERR_ARG;
            *bytes = linear_bwd_ws(dtype, shape[0], shape[1]);
            return TB_OK;
        case TB_OP_ATTN_BWD:      // {B, Hq, Sq}
            if (!shape || n_shape != 3) return TB_ERR_ARG;
            *bytes = (size_t)shape[0] * shape[1] * shape[2] * 4;
            return TB_OK;
        case TB_OP_CONV2D_BWD:
            return TB_OK;
        default: return TB_ERR_ARG;
    }
}

}  // extern "C"

// conv2d forward (NCHW, groups = 1) with the inference epilogue
// bias -> folded BatchNorm scale/shift -> activation.
//
//  * bf16: implicit GEMM on tcgen05.  The input is first transposed to NHWC
//    with channels padded to a multiple of 8 (caller workspace), the weights
//    reordered to [Cout][KH][KW][Cin_pad].  GEMM view: M = output pixels,
//    N = Cout, K = KH * KW * Cin_pad.  One CTA computes a tile of 16 x 8
//    output pixels (rows h, columns w) x 64 output channels; each K-block is
//    one filter tap (kh, kw) x 64 input channels, fetched by a 4-D TMA box
//    (64 channels, 8 columns, 16 rows, 1 image) whose column / row coordinates
//    are shifted by the tap and may be negative: out-of-range positions read
//    as zero, which is exactly the convolution's zero padding.  The epilogue
//    stages the tile in shared memory as [channel][row][column] and writes it
//    to NCHW with one TMA store.  Unit stride, OW % 8 == 0.
//  * CUDA cores: implicit GEMM with exact f32 FMA accumulation, for f32 I/O
//    (the reference's fp32 kernels, conv2d.rs:44-148 / :643-764, and its 1e-4
//    tolerance) and for the bf16 shapes the tensor-core path does not take.
#include "common.cuh"

namespace tb {

struct ConvEpi {
    const float* bias;
    const float* scale;
    const float* shift;
    int act;   // -1 none, 0 silu, 2 relu
};

__device__ __forceinline__ float conv_epi(const ConvEpi& e, int co, float v) {
    if (e.bias && !e.shift) v += e.bias[co];
    if (e.scale) v *= e.scale[co];
    if (e.shift) v += e.shift[co];
    if (e.act == TB_ACT_RELU) v = v > 0.f ? v : 0.f;
    else if (e.act == TB_ACT_SILU) v = v / (1.0f + expf(-v));
    return v;
}

// ------------------------------------------------------------ layout prep --
// x [B][C][H][W] (f32 or bf16) -> xn [B][H][W][Cp] bf16, channels >= C zero.
template <typename T>
__global__ void nchw_to_nhwc_kernel(const T* __restrict__ x, __nv_bfloat16* __restrict__ xn, int B, int C, int H,
                                    int W, int Cp) {
    __shared__ float tile[32][33];
    const int bh = blockIdx.z;          // b * H + h
    const int b = bh / H, h = bh % H;
    const int c0 = blockIdx.y * 32, w0 = blockIdx.x * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, w = w0 + threadIdx.x;
        float v = 0.f;
        if (c < C && w < W) {
            const T* p = x + (((int64_t)b * C + c) * H + h) * W + w;
            if constexpr (sizeof(T) == 4) v = *p;
            else v = __bfloat162float(*p);
        }
        tile[i][threadIdx.x] = v;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int w = w0 + i, c = c0 + threadIdx.x;
        if (w < W && c < Cp) xn[(((int64_t)b * H + h) * W + w) * Cp + c] = __float2bfloat16_rn(tile[threadIdx.x][i]);
    }
}

// w [Co][C][KH][KW] -> wr [Co][KH][KW][Cp] bf16 (channels >= C zero)
template <typename T>
__global__ void reorder_weights_kernel(const T* __restrict__ w, __nv_bfloat16* __restrict__ wr, int Co, int C, int KH,
                                       int KW, int Cp) {
    const int64_t total = (int64_t)Co * KH * KW * Cp;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % Cp);
        int64_t r = i / Cp;
        const int kw = (int)(r % KW);
        r /= KW;
        const int kh = (int)(r % KH);
        const int co = (int)(r / KH);
        float v = 0.f;
        if (c < C) {
            const T* p = w + (((int64_t)co * C + c) * KH + kh) * KW + kw;
            if constexpr (sizeof(T) == 4) v = *p;
            else v = __bfloat162float(*p);
        }
        wr[i] = __float2bfloat16_rn(v);
    }
}

// ---------------------------------------------------------- tcgen05 conv --
constexpr int CONV_BH = 16, CONV_BW = 8, CONV_BN = 64, CONV_STAGES = 6;
constexpr int CONV_A_BYTES = 128 * 128;            // 128 pixels x 64 channels
constexpr int CONV_B_BYTES = CONV_BN * 128;        // 64 couts x 64 channels
constexpr int CONV_OUT_BYTES = CONV_BN * 128 * 2;  // [64][16][8] bf16
constexpr int CONV_SMEM = CONV_STAGES * (CONV_A_BYTES + CONV_B_BYTES) + CONV_OUT_BYTES + 1024 + 256;

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// grid: (tiles_w * tiles_h * B, ceil(Cout / 64))
__global__ void __launch_bounds__(256, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
               const __grid_constant__ CUtensorMap tmY, ConvEpi ep, int OH, int OW, int Cout, int KH, int KW,
               int Cp, int stride, int pad, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = sA + CONV_STAGES * CONV_A_BYTES;
    __nv_bfloat16* sO = reinterpret_cast<__nv_bfloat16*>(sB + CONV_STAGES * CONV_B_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sO) + CONV_OUT_BYTES);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + CONV_STAGES), accb = smem_u32(bars + 2 * CONV_STAGES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * CONV_STAGES + 1);

    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int tiles_w = (OW + CONV_BW - 1) / CONV_BW, tiles_h = (OH + CONV_BH - 1) / CONV_BH;
    int t = blockIdx.x;
    const int tw = t % tiles_w;
    t /= tiles_w;
    const int th = t % tiles_h;
    const int b = t / tiles_h;
    const int ow0 = tw * CONV_BW, oh0 = th * CONV_BH, n0 = blockIdx.y * CONV_BN;
    const int nc = (Cp + 63) / 64;            // 64-channel chunks per tap
    const int nk = KH * KW * nc;

    if (threadIdx.x == 0) {
        for (int s = 0; s < CONV_STAGES; s++) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        mbar_init(accb, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), CONV_BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmW);
        int issued = 0;
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % CONV_STAGES;
            if (kb >= CONV_STAGES && !mbar_wait(empty0 + 8 * s, ((kb / CONV_STAGES) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) break;
            const int tap = kb / nc, c0 = (kb % nc) * 64;
            const int kh = tap / KW, kw = tap % KW;
            mbar_expect_tx(full0 + 8 * s, CONV_A_BYTES + CONV_B_BYTES);
            tma_load_4d(smem_u32(sA + s * CONV_A_BYTES), &tmX, full0 + 8 * s, c0, ow0 * stride + kw - pad,
                        oh0 * stride + kh - pad, b);
            tma_load_2d(smem_u32(sB + s * CONV_B_BYTES), &tmW, full0 + 8 * s, tap * Cp + c0, n0);
            issued = kb + 1;
        }
        for (int kb = (issued > CONV_STAGES ? issued - CONV_STAGES : 0); kb < issued; kb++)
            mbar_wait(full0 + 8 * (kb % CONV_STAGES), (kb / CONV_STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL);
    } else if (warp == 1 && lane == 0) {
        constexpr uint32_t idesc = idesc_bf16_f32(128, CONV_BN, false, false);
        for (int kb = 0; kb < nk; kb++) {
            const int s = kb % CONV_STAGES;
            if (!mbar_wait(full0 + 8 * s, (kb / CONV_STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
            tc_fence_after();
            const uint32_t a_base = smem_u32(sA + s * CONV_A_BYTES), b_base = smem_u32(sB + s * CONV_B_BYTES);
#pragma unroll
            for (int kk = 0; kk < 4; kk++)
                umma_f16_ss(tmem, sdesc_sw128(a_base + kk * 32, 16, 1024), sdesc_sw128(b_base + kk * 32, 16, 1024),
                            idesc, (kb | kk) != 0);
            umma_commit(empty0 + 8 * s);
        }
        umma_commit(accb);
    }
    __syncwarp();

    // epilogue: thread <-> pixel row r = 32 * (warp % 4) + lane (h = r / 8, w = r % 8),
    // warps 0-3 channels [0, 32), warps 4-7 channels [32, 64)
    bool ok = __all_sync(0xffffffffu, mbar_wait(accb, 0, err, DEV_ERR_TIMEOUT_ACC));
    tc_fence_after();
    const int q = warp & 3, half = warp >> 2;
    const int r = q * 32 + lane;
    float v[32];
    tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + half * 32, v);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; j++) {
        const int co = n0 + half * 32 + j;
        const float o = co < Cout ? conv_epi(ep, co, v[j]) : 0.f;
        sO[(half * 32 + j) * 128 + r] = __float2bfloat16_rn(o);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, CONV_BN);
    if (threadIdx.x == 0 && ok) tma_store_4d(&tmY, smem_u32(sO), ow0, oh0, n0, b);
}

// ------------------------------------------------------------- f32 conv ---
// Implicit GEMM on CUDA cores: 64 output pixels x 64 output channels per CTA,
// K = C * KH * KW in slices of 16, the im2col gather done while loading.
// f32 accumulate for both I/O types (bf16 I/O: strides > 1, widths % 8 != 0).
__device__ __forceinline__ float ldf(const float* p) { return *p; }
__device__ __forceinline__ float ldf(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stf(float* p, float v) { *p = v; }
__device__ __forceinline__ void stf(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(256)
conv_simt_kernel(const T* __restrict__ x, const T* __restrict__ w, ConvEpi ep, T* __restrict__ y, int B,
                 int C, int Co, int H, int W, int KH, int KW, int stride, int pad, int OH, int OW) {
    pdl_trigger();
    pdl_wait();
    __shared__ float sa[16][64 + 4];
    __shared__ float sb[16][64 + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t P = (int64_t)B * OH * OW;
    const int64_t p0 = (int64_t)blockIdx.x * 64;
    const int n0 = blockIdx.y * 64;
    const int K = C * KH * KW;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 64 * 16; i += 256) {
            const int pr = i / 16, kk = i % 16;
            const int64_t p = p0 + pr;
            const int k = k0 + kk;
            float av = 0.f;
            if (p < P && k < K) {
                const int ow = (int)(p % OW);
                const int64_t t2 = p / OW;
                const int oh = (int)(t2 % OH), bb = (int)(t2 / OH);
                const int kw = k % KW, kh = (k / KW) % KH, c = k / (KW * KH);
                const int ih = oh * stride + kh - pad, iw = ow * stride + kw - pad;
                if (ih >= 0 && ih < H && iw >= 0 && iw < W) av = ldf(x + (((int64_t)bb * C + c) * H + ih) * W + iw);
            }
            sa[kk][pr] = av;
            const int co = n0 + pr;
            sb[kk][pr] = (co < Co && k < K) ? ldf(w + (int64_t)co * K + k) : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; kk++) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                av[i] = sa[kk][ty + 16 * i];
                bv[i] = sb[kk][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int64_t p = p0 + ty + 16 * i;
        if (p >= P) continue;
        const int ow = (int)(p % OW);
        const int64_t t2 = p / OW;
        const int oh = (int)(t2 % OH), bb = (int)(t2 / OH);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int co = n0 + tx + 16 * j;
            if (co < Co) stf(y + (((int64_t)bb * Co + co) * OH + oh) * OW + ow, conv_epi(ep, co, acc[i][j]));
        }
    }
}

// ------------------------------------------------------------ batchnorm ---
__global__ void bn_fold_kernel(const float* g, const float* be, const float* mu, const float* var, const float* bias,
                               float eps, float* scale, float* shift, int C) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const float sc = g[c] / sqrtf(var[c] + eps);
    float sh = be[c] - sc * mu[c];
    if (bias) sh += sc * bias[c];
    scale[c] = sc;
    shift[c] = sh;
}

// batch_norm_2d_nchw_forward_inference (nn/norm/batchnorm.rs:574-686).
template <typename T>
__global__ void batchnorm_kernel(const T* __restrict__ x, const float* __restrict__ g, const float* __restrict__ be,
                                 const float* __restrict__ mu, const float* __restrict__ var, T* __restrict__ y,
                                 int64_t total, int C, int64_t HW, float eps) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)((i / HW) % C);
        float v;
        if constexpr (sizeof(T) == 4) v = x[i];
        else v = __bfloat162float(x[i]);
        v = (v - mu[c]) * rsqrtf(var[c] + eps) * g[c] + be[c];
        if constexpr (sizeof(T) == 4) y[i] = v;
        else y[i] = __float2bfloat16_rn(v);
    }
}

struct ConvShape {
    int B, C, Co, H, W, KH, KW, stride, pad, OH, OW, Cp;
};

static size_t conv_ws_bytes(const ConvShape& s) {
    const size_t xn = (size_t)s.B * s.H * s.W * s.Cp * 2;
    const size_t wr = (size_t)s.Co * s.KH * s.KW * s.Cp * 2;
    return ((xn + 255) / 256) * 256 + ((wr + 255) / 256) * 256;
}

static bool conv_shape(int B, int C, int Co, int H, int W, int KH, int KW, int stride, int pad, ConvShape* s) {
    if (B <= 0 || C <= 0 || Co <= 0 || H <= 0 || W <= 0 || KH <= 0 || KW <= 0 || stride <= 0 || pad < 0) return false;
    s->B = B; s->C = C; s->Co = Co; s->H = H; s->W = W; s->KH = KH; s->KW = KW; s->stride = stride; s->pad = pad;
    s->OH = (H + 2 * pad - KH) / stride + 1;
    s->OW = (W + 2 * pad - KW) / stride + 1;
    s->Cp = (C + 7) / 8 * 8;
    return s->OH > 0 && s->OW > 0;
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_conv2d_workspace_size(int dtype, int B, int Cin, int Cout, int H, int W, int KH, int KW, int stride, int pad,
                             size_t* bytes) {
    if (!bytes) return TB_ERR_ARG;
    ConvShape s;
    if (!conv_shape(B, Cin, Cout, H, W, KH, KW, stride, pad, &s)) return TB_ERR_SHAPE;
    *bytes = (dtype == TB_BF16 && stride == 1 && s.OW % 8 == 0) ? conv_ws_bytes(s) : 0;
    return TB_OK;
}

int tb_conv2d_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias, const float* bn_scale,
                  const float* bn_shift, void* y, int B, int Cin, int Cout, int H, int W, int KH, int KW, int stride,
                  int pad, int act, void* workspace, size_t workspace_bytes) {
    if (!ctx || !x || !w || !y) return TB_ERR_ARG;
    ConvShape s;
    TB_REQUIRE(ctx, conv_shape(B, Cin, Cout, H, W, KH, KW, stride, pad, &s), TB_ERR_SHAPE, "conv2d: bad shape");
    TB_REQUIRE(ctx, act == TB_ACT_NONE || act == TB_ACT_RELU || act == TB_ACT_SILU, TB_ERR_ARG, "conv2d: act %d", act);
    ConvEpi ep{bias, bn_scale, bn_shift, act};
    const int64_t P = (int64_t)B * s.OH * s.OW;
    const dim3 sgrid((unsigned)((P + 63) / 64), (unsigned)((Cout + 63) / 64));
    if (dtype == TB_F32)
        return launch(ctx, "conv2d_f32", conv_simt_kernel<float>, sgrid, dim3(256), 0, (const float*)x, (const float*)w,
                      ep, (float*)y, B, Cin, Cout, H, W, KH, KW, stride, pad, s.OH, s.OW);
    if (dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "conv2d: dtype %d", dtype);
    if (stride != 1 || s.OW % 8 != 0)   // tensor-core path: unit stride, output rows of 16-byte multiples
        return launch(ctx, "conv2d_simt_bf16", conv_simt_kernel<__nv_bfloat16>, sgrid, dim3(256), 0,
                      (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, ep, (__nv_bfloat16*)y, B, Cin, Cout, H, W, KH,
                      KW, stride, pad, s.OH, s.OW);
    TB_REQUIRE(ctx, aligned16(y), TB_ERR_ALIGN, "conv2d bf16: y must be 16-byte aligned");
    const size_t need = conv_ws_bytes(s);
    TB_REQUIRE(ctx, workspace && workspace_bytes >= need && aligned16(workspace), TB_ERR_ARG,
               "conv2d bf16: workspace of %zu bytes required (tb_conv2d_workspace_size)", need);
    __nv_bfloat16* xn = reinterpret_cast<__nv_bfloat16*>(workspace);
    __nv_bfloat16* wr = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(workspace) +
                                                         (((size_t)B * H * W * s.Cp * 2 + 255) / 256) * 256);
    {
        dim3 grid((W + 31) / 32, (s.Cp + 31) / 32, B * H);
        int rc = launch(ctx, "nchw_to_nhwc", nchw_to_nhwc_kernel<__nv_bfloat16>, grid, dim3(32, 8), 0,
                        (const __nv_bfloat16*)x, xn, B, Cin, H, W, s.Cp);
        if (rc) return rc;
        const int64_t tot = (int64_t)Cout * KH * KW * s.Cp;
        rc = launch(ctx, "reorder_weights", reorder_weights_kernel<__nv_bfloat16>,
                    dim3((unsigned)((tot + 255) / 256 < 4096 ? (tot + 255) / 256 : 4096)), dim3(256), 0,
                    (const __nv_bfloat16*)w, wr, Cout, Cin, KH, KW, s.Cp);
        if (rc) return rc;
    }
    CUtensorMap mx, mw, my;
    {
        uint64_t dims[4] = {(uint64_t)s.Cp, (uint64_t)W, (uint64_t)H, (uint64_t)B};
        uint64_t strides[3] = {(uint64_t)s.Cp * 2, (uint64_t)W * s.Cp * 2, (uint64_t)H * W * s.Cp * 2};
        uint32_t box[4] = {64, CONV_BW, CONV_BH, 1};
        cuuint32_t es[4] = {1, 1, 1, 1};
        int rc = make_tmap_strided(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, xn, dims, strides, box, es,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        rc = make_tmap_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wr, Cout, (uint64_t)KH * KW * s.Cp,
                          (uint64_t)KH * KW * s.Cp, 64, CONV_BN);
        if (rc) return rc;
        uint64_t ydims[4] = {(uint64_t)s.OW, (uint64_t)s.OH, (uint64_t)Cout, (uint64_t)B};
        uint64_t ystr[3] = {(uint64_t)s.OW * 2, (uint64_t)s.OH * s.OW * 2, (uint64_t)Cout * s.OH * s.OW * 2};
        uint32_t ybox[4] = {CONV_BW, CONV_BH, CONV_BN, 1};
        rc = make_tmap(ctx, &my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, y, ydims, ystr, ybox, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    TB_CUDA_TRY(ctx, cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CONV_SMEM));
    const int tiles = ((s.OW + CONV_BW - 1) / CONV_BW) * ((s.OH + CONV_BH - 1) / CONV_BH) * B;
    dim3 grid((unsigned)tiles, (unsigned)((Cout + CONV_BN - 1) / CONV_BN));
    return launch(ctx, "conv_tc", conv_tc_kernel, grid, dim3(256), CONV_SMEM, mx, mw, my, ep, s.OH, s.OW, Cout, KH,
                  KW, s.Cp, stride, pad, ctx->d_err);
}

int tb_bn_fold(tb_ctx* ctx, const float* gamma, const float* beta, const float* mean, const float* var,
               const float* bias, float eps, float* scale, float* shift, int C) {
    if (!ctx || !gamma || !beta || !mean || !var || !scale || !shift) return TB_ERR_ARG;
    if (C <= 0) return set_error(ctx, TB_ERR_SHAPE, "bn_fold: C=%d", C);
    return launch(ctx, "bn_fold", bn_fold_kernel, dim3((C + 127) / 128), dim3(128), 0, gamma, beta, mean, var, bias,
                  eps, scale, shift, C);
}

int tb_batchnorm_fwd(tb_ctx* ctx, int dtype, const void* x, const float* gamma, const float* beta, const float* mean,
                     const float* var, void* y, int64_t B, int64_t C, int64_t HW, float eps) {
    if (!ctx || !x || !gamma || !beta || !mean || !var || !y) return TB_ERR_ARG;
    TB_REQUIRE(ctx, B >= 0 && C > 0 && HW > 0 && C < (1ll << 31), TB_ERR_SHAPE, "batchnorm: bad shape");
    const int64_t total = B * C * HW;
    if (total == 0) return TB_OK;
    const unsigned grid = (unsigned)((total + 255) / 256 < 8192 ? (total + 255) / 256 : 8192);
    if (dtype == TB_F32)
        return launch(ctx, "batchnorm", batchnorm_kernel<float>, dim3(grid), dim3(256), 0, (const float*)x, gamma, beta,
                      mean, var, (float*)y, total, (int)C, HW, eps);
    if (dtype == TB_BF16)
        return launch(ctx, "batchnorm", batchnorm_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0,
                      (const __nv_bfloat16*)x, gamma, beta, mean, var, (__nv_bfloat16*)y, total, (int)C, HW, eps);
    return set_error(ctx, TB_ERR_UNSUPPORTED, "batchnorm: dtype %d", dtype);
}

}  // extern "C"

// Row argmax that allocates nothing.
//
// A split-row argmax (several CTAs per row, one per slice of the vocabulary,
// combined through a per-row 64-bit key and an arrival counter) needs
// cross-CTA scratch.  This entry point serves callers that cannot allocate
// device memory at all -- e.g. a serving loop whose device memory is owned by
// an external pool -- by keeping that scratch in a file-scope device array.
//
// Scratch: 16 bytes per row (key, counter), TB_ARGMAX_NOALLOC_MAX_ROWS rows,
// resident on every GPU that loads the library until the process exits.
// Every call shares it: each call clears its rows first (stream-ordered), and
// calls that overlap on the GPU (two streams, or two host threads) race.
#include <mutex>

#include "common.cuh"

namespace tb {

static __device__ __align__(256) unsigned long long g_argmax_noalloc_scratch[2 * TB_ARGMAX_NOALLOC_MAX_ROWS];

__device__ __forceinline__ float ld_as_f32(const float* p) { return *p; }
__device__ __forceinline__ float ld_as_f32(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// Grid (M, chunks).  Each CTA reduces its slice of the row to (value, index)
// (greater value wins, equal values keep the lower index, NaN is skipped),
// folds it into the row's key with atomicMax (argmax_key: order-preserving
// bits of the value << 32 | ~index, -0.0 keyed as +0.0), and the last CTA of
// the row writes out[row].
template <typename T>
__global__ void argmax_noalloc_kernel(const T* __restrict__ x, int32_t* __restrict__ out, int64_t N, int chunk,
                                      unsigned long long* scratch) {
    const int row = blockIdx.x;
    const T* xr = x + (int64_t)row * N;
    const int64_t c0 = (int64_t)blockIdx.y * chunk;
    const int64_t c1 = c0 + chunk < N ? c0 + chunk : N;
    float bv = -INFINITY;
    int bi = -1;
    for (int64_t c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
        const float v = ld_as_f32(xr + c);
        if (v != v) continue;
        if (bi < 0 || v > bv) {
            bv = v;
            bi = (int)c;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, bv, o);
        const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
        if (i2 >= 0 && (bi < 0 || v2 > bv || (v2 == bv && i2 < bi))) {
            bv = v2;
            bi = i2;
        }
    }
    __shared__ float sv[32];
    __shared__ int si[32];
    __shared__ int s_last;
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    unsigned long long* key = scratch + 2 * row;
    unsigned* cnt = reinterpret_cast<unsigned*>(scratch + 2 * row + 1);
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x / 32); w++) {
            if (si[w] >= 0 && (bi < 0 || sv[w] > bv || (sv[w] == bv && si[w] < bi))) {
                bv = sv[w];
                bi = si[w];
            }
        }
        if (bi >= 0) atomicMax(key, argmax_key(bv, bi));
        __threadfence();
        s_last = atomicAdd(cnt, 1u) == gridDim.y - 1;
    }
    __syncthreads();
    if (threadIdx.x == 0 && s_last) {
        __threadfence();
        const unsigned long long k = atomicExch(key, 0ull);
        out[row] = k ? argmax_key_index(k) : 0;
        *cnt = 0u;
    }
}

// Device address of the scratch array, looked up once per device with that
// device current (host code must not hand the symbol itself to a kernel).
static int scratch_ptr(tb_ctx* ctx, unsigned long long** out) {
    static std::mutex mu;
    static unsigned long long* ptrs[64] = {};
    if (ctx->device < 0 || ctx->device >= 64) return set_error(ctx, TB_ERR_ARG, "argmax_noalloc: device %d", ctx->device);
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[ctx->device]) {
        int prev = -1;
        TB_CUDA_TRY(ctx, cudaGetDevice(&prev));
        if (prev != ctx->device) TB_CUDA_TRY(ctx, cudaSetDevice(ctx->device));
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_noalloc_scratch);
        if (prev != ctx->device) cudaSetDevice(prev);
        if (e != cudaSuccess)
            return set_error(ctx, TB_ERR_CUDA, "argmax_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
        ptrs[ctx->device] = reinterpret_cast<unsigned long long*>(p);
    }
    *out = ptrs[ctx->device];
    return TB_OK;
}

}  // namespace tb

using namespace tb;

extern "C" int tb_argmax_noalloc_fwd(tb_ctx* ctx, int dtype, const void* x, int32_t* out, int64_t M, int64_t N) {
    if (!ctx || !x || !out) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && M <= TB_ARGMAX_NOALLOC_MAX_ROWS, TB_ERR_SHAPE,
               "argmax_noalloc: M=%lld rows exceeds the static scratch (%d rows)", (long long)M,
               TB_ARGMAX_NOALLOC_MAX_ROWS);
    TB_REQUIRE(ctx, N > 0 && N < (1ll << 31), TB_ERR_SHAPE, "argmax_noalloc: N=%lld", (long long)N);
    if (dtype != TB_F32 && dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "argmax_noalloc: dtype %d", dtype);
    if (M == 0) return TB_OK;
    unsigned long long* scratch = nullptr;
    int rc = scratch_ptr(ctx, &scratch);
    if (rc) return rc;
    // the rows this call uses start from zero, whatever an earlier (possibly failed) call left
    TB_CUDA_TRY(ctx, cudaMemsetAsync(scratch, 0, (size_t)M * 16, ctx->stream));
    // 2048 columns per CTA, widened for rows so long that the chunk count
    // would pass the 65535 limit of gridDim.y
    int64_t chunk = 2048;
    if ((N + chunk - 1) / chunk > 65535) chunk = (N + 65534) / 65535;
    const dim3 grid((unsigned)M, (unsigned)((N + chunk - 1) / chunk));
    if (dtype == TB_F32)
        argmax_noalloc_kernel<float><<<grid, 256, 0, ctx->stream>>>((const float*)x, out, N, (int)chunk, scratch);
    else
        argmax_noalloc_kernel<__nv_bfloat16><<<grid, 256, 0, ctx->stream>>>((const __nv_bfloat16*)x, out, N, (int)chunk,
                                                                        scratch);
    return check_launch(ctx, "argmax_noalloc");
}

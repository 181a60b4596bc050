// Linear layers on B200.
//
//  * gemm_tc_kernel: y[M,N] = x[M,K] w[N,K]^T for prefill-sized M.  One CTA
//    per 128 x BN output tile; warp 0 streams K-blocks of 64 with TMA (128-B
//    swizzle) into a STAGES-deep ring, warp 1 issues tcgen05.mma (M=128, N=BN,
//    K=16, f32 accumulator in TMEM), all 8 warps run the fused epilogue
//    (bias, residual, SwiGLU, bf16/f32 store) straight out of TMEM.
//  * gemv_tc_kernel: decode-sized M (<= 64 tokens).  Swap-AB: the weight rows
//    are the MMA's M dimension (two 128-row halves per CTA), the tokens its N.
//    K is split across the CTAs of a thread-block cluster (up to 16), which
//    exchange their partials over DSMEM; each CTA finishes a slice of the
//    rows.  Weights are bf16, or int8 converted exactly (|q| <= 127) to bf16
//    straight into TMEM by eight converter warps, the MMA taking its A operand
//    from TMEM.  An RMSNorm of the activations can be fused in front.
//  * linear_f32_kernel / matmul_f32_kernel: exact-f32 CUDA-core tiles for the
//    fp32 configurations (the reference's TF32 dot, linear.rs:86, misses the
//    1e-4 fp32 tolerance at K >= 256).
#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "gemm.h"

namespace tb {


// ------------------------------------------------------------ store helpers --
__device__ __forceinline__ void store_row8(void* out, bool f32, int64_t off, const float* v) {
    if (f32) {
        float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + off);
        p[0] = make_float4(v[0], v[1], v[2], v[3]);
        p[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint4 a;
        a.x = pack_bf16x2(v[0], v[1]);
        a.y = pack_bf16x2(v[2], v[3]);
        a.z = pack_bf16x2(v[4], v[5]);
        a.w = pack_bf16x2(v[6], v[7]);
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out) + off) = a;
    }
}

__device__ __forceinline__ void load_row8(const void* p, bool f32, int64_t off, float* v) {
    if (f32) {
        const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + off);
        float4 a = q[0], b = q[1];
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
        uint4 a = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p) + off);
        uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[2 * i] = bf16_lo(w[i]);
            v[2 * i + 1] = bf16_hi(w[i]);
        }
    }
}

// =====================================================================
// Prefill GEMM
// =====================================================================
constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;

template <int BN, int STAGES>
constexpr int gemm_smem_bytes() {
    return STAGES * (GEMM_BM * 128 + BN * 128) + 1024 /*align*/ + 256 /*barriers*/;
}
constexpr int GEMM_THREADS = 384;   // warp 0 TMA, warp 1 MMA, warps 4-11 epilogue

// Persistent: one CTA per SM walks the output tiles (t += gridDim.x) in groups
// of gm 128-row tile rows (gemm_tile): m fastest inside a group, so running
// CTAs share the weight tile, and the group's activation rows (gm x 128 x K,
// at most 32 MB as the launcher picks gm) stay in L2 while every weight tile
// streams past them once per group.  A plain m-fastest walk over all rows
// re-read the activations from DRAM (601 MB for 128 MB of operands on the
// 16384 x 16384 x 2048 gate/up GEMM).  The f32 accumulator
// is double-buffered in TMEM (2 x BN columns): the epilogue of tile i (warps
// 4-11: TMEM lane quarter warp % 4, column half (warp - 4) / 4) overlaps the
// MMAs of tile i + 1.
// B_MN: b operand stored [K, N] (N contiguous), as matmul_forward's B.
// Output tile t -> (row tile mi, column tile ni): groups of gm row tiles (the
// last may be shorter), rows fastest inside a group.
__device__ __forceinline__ void gemm_tile(int t, int mt, int ntl, int gm, int& mi, int& ni) {
    const int grp = t / (gm * ntl), r = t - grp * gm * ntl;
    const int g0 = grp * gm;
    const int rows = min(gm, mt - g0);
    mi = g0 + r % rows;
    ni = r / rows;
}

template <int BN, int STAGES, bool B_MN>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               Epi ep, int M, int N, int K, int gm, int* err) {
    constexpr int A_BYTES = GEMM_BM * 128;
    constexpr int B_BYTES = BN * 128;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* sA = smem;
    uint8_t* sB = smem + STAGES * A_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    const uint32_t accf0 = smem_u32(bars + 2 * STAGES);       // [2] accumulator ready
    const uint32_t acce0 = smem_u32(bars + 2 * STAGES + 2);   // [2] accumulator drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int mt = (M + GEMM_BM - 1) / GEMM_BM, ntl = (N + BN - 1) / BN;
    const int tiles = mt * ntl;
    const int nk = (K + GEMM_BK - 1) / GEMM_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(accf0 + 8 * s, 1);
            mbar_init(acce0 + 8 * s, 8);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- TMA producer.  The weights (B) do not depend on the
        // previous kernel: the first tile's first STAGES K-blocks of them are
        // requested before waiting for it, the activations (A) after.
        if (lane == 0) {
            tma_prefetch_desc(&tmA);
            tma_prefetch_desc(&tmB);
            auto load_b = [&](int s, int kb, int n0) {
                if (!B_MN) {
                    tma_load_2d(smem_u32(sB + s * B_BYTES), &tmB, full0 + 8 * s, kb * GEMM_BK, n0);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / 64; j++)
                        tma_load_2d(smem_u32(sB + s * B_BYTES + j * 64 * 128), &tmB, full0 + 8 * s, n0 + 64 * j,
                                    kb * GEMM_BK);
                }
            };
            int pre = 0;
            if ((int)blockIdx.x < tiles) {
                int mi, ni;
                gemm_tile(blockIdx.x, mt, ntl, gm, mi, ni);
                pre = nk < STAGES ? nk : STAGES;
                for (int kb = 0; kb < pre; kb++) {
                    mbar_expect_tx(full0 + 8 * kb, A_BYTES + B_BYTES);
                    load_b(kb, kb, ni * BN);
                }
                pdl_wait();
                for (int kb = 0; kb < pre; kb++)
                    tma_load_2d(smem_u32(sA + kb * A_BYTES), &tmA, full0 + 8 * kb, kb * GEMM_BK, mi * GEMM_BM);
            }
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
                int mi, ni;
                gemm_tile(t, mt, ntl, gm, mi, ni);
                const int m0 = mi * GEMM_BM, n0 = ni * BN;
                for (int kb = 0; kb < nk; kb++, it++) {
                    if (it < pre) continue;   // requested above
                    const int s = it % STAGES;
                    if (it >= STAGES && !mbar_wait(empty0 + 8 * s, ((it / STAGES) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(full0 + 8 * s, A_BYTES + B_BYTES);
                    tma_load_2d(smem_u32(sA + s * A_BYTES), &tmA, full0 + 8 * s, kb * GEMM_BK, m0);
                    load_b(s, kb, n0);
                }
            }
            // every issued stage has landed before the CTA can exit
            for (int k = (it > STAGES ? it - STAGES : 0); k < it; k++)
                mbar_wait(full0 + 8 * (k % STAGES), (k / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL);
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(GEMM_BM, BN, false, B_MN);
            const uint64_t a_desc0 = sdesc_sw128(smem_u32(sA), 16, 1024);
            const uint64_t b_desc0 = B_MN ? sdesc_sw128(smem_u32(sB), 64 * 128, 1024) : sdesc_sw128(smem_u32(sB), 16, 1024);
            int it = 0, tl = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, tl++) {
                const int ab = tl & 1;
                if (tl >= 2 && !mbar_wait(acce0 + 8 * ab, ((tl >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + ab * BN;
                for (int kb = 0; kb < nk; kb++, it++) {
                    const int s = it % STAGES;
                    if (!mbar_wait(full0 + 8 * s, (it / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = a_desc0 + (uint64_t)((s * A_BYTES) >> 4);
                    const uint64_t bd = b_desc0 + (uint64_t)((s * B_BYTES) >> 4);
#pragma unroll
                    for (int kk = 0; kk < GEMM_BK / 16; kk++)
                        umma_f16_ss(d_tmem, ad + 2 * kk, bd + (B_MN ? kk * 128 : 2 * kk), idesc, (kb | kk) != 0);
                    umma_commit(empty0 + 8 * s);
                }
                umma_commit(accf0 + 8 * ab);
            }
        }
    } else if (warp >= 4) {
        // ---------------- epilogue: TMEM lane quarter q = warp % 4, column half
        pdl_wait();   // the previous kernel is done before any global read or write here
        const int q = warp & 3, half = (warp - 4) >> 2;
        const uint32_t t_lane = tmem + ((uint32_t)(q * 32) << 16);
        const bool f32o = ep.out_f32 != 0;
        const int pos_base = ep.rope_tab ? (ep.pos_ptr ? *ep.pos_ptr : ep.pos_host) : 0;
        bool ok = true;
        int tl = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, tl++) {
            int mi, ni;
            gemm_tile(t, mt, ntl, gm, mi, ni);
            const int m0 = mi * GEMM_BM, n0 = ni * BN;
            const int ab = tl & 1;
            ok = mbar_wait(accf0 + 8 * ab, (tl >> 1) & 1, err, DEV_ERR_TIMEOUT_ACC) && ok;
            tc_fence_after();
            const uint32_t t_row = t_lane + ab * BN;
            const int row = m0 + q * 32 + lane;
            if (ep.rope_tab) {
                // QKV with RoPE and the KV-cache write: the weight rows are permuted per
                // 256-row tile (qkv_perm_row), so columns p < 128 and p + 128 of the tile
                // are dims (i, i + hd/2) of one head, and a chunk of 32 pairs lies in one
                // head.  The projection is rounded to bf16 first, as the unfused path
                // stores it, then rotated (rotate-half); q goes to out in natural order,
                // k and v to the caches at position pos_base + (row % rope_s_new).
                const int hd = ep.perm_hd, hh = hd / 2;
                __nv_bfloat16* outb = reinterpret_cast<__nv_bfloat16*>(ep.out);
#pragma unroll 1
                for (int c = half * 64; c < half * 64 + 64; c += 32) {
                    float a[32], bv[32];
                    tmem_ld32(t_row + c, a);
                    tmem_ld32(t_row + 128 + c, bv);
                    tmem_wait_ld();
                    const int H = (n0 / 256) * (256 / hd) + c / hh, ri0 = c % hh;
                    const int kind = H < ep.rope_hq ? 0
                                   : H < ep.rope_hq + ep.rope_hkv ? 1
                                   : H < ep.rope_hq + 2 * ep.rope_hkv ? 2 : 3;
                    if (!ok || row >= M || kind == 3) continue;
                    const int bs = row / ep.rope_s_new, pos = pos_base + row % ep.rope_s_new;
                    if (pos < 0 || pos >= ep.max_seq) {
                        atomicOr(err, 1 << 5);
                        continue;
                    }
                    __nv_bfloat16* dst;
                    if (kind == 0)
                        dst = outb + (int64_t)row * ep.ldo + (int64_t)H * hd;
                    else if (kind == 1)
                        dst = reinterpret_cast<__nv_bfloat16*>(ep.kcache) +
                              (((int64_t)bs * ep.rope_hkv + (H - ep.rope_hq)) * ep.max_seq + pos) * hd;
                    else
                        dst = reinterpret_cast<__nv_bfloat16*>(ep.vcache) +
                              (((int64_t)bs * ep.rope_hkv + (H - ep.rope_hq - ep.rope_hkv)) * ep.max_seq + pos) * hd;
                    const float2* tab = ep.rope_tab + (int64_t)pos * hh + ri0;
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        float y0[8], y1[8];
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            const float x0 = __bfloat162float(__float2bfloat16_rn(a[j + i]));
                            const float x1 = __bfloat162float(__float2bfloat16_rn(bv[j + i]));
                            if (kind <= 1) {
                                const float2 cs = tab[j + i];
                                y0[i] = x0 * cs.x - x1 * cs.y;
                                y1[i] = x1 * cs.x + x0 * cs.y;
                            } else {
                                y0[i] = x0;
                                y1[i] = x1;
                            }
                        }
                        store_row8(dst, false, ri0 + j, y0);
                        store_row8(dst, false, hh + ri0 + j, y1);
                    }
                }
            } else if (!ep.swiglu) {
#pragma unroll 1
                for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
                    float v[32];
                    tmem_ld32(t_row + c, v);
                    tmem_wait_ld();
                    const int col0 = n0 + c;
                    if (ok && row < M) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            const int col = col0 + j;
                            if (col < N) {
                                if (ep.bias) {
#pragma unroll
                                    for (int i = 0; i < 8; i++) v[j + i] += ep.bias[col + i];
                                }
                                if (ep.resid) {
                                    float r[8];
                                    load_row8(ep.resid, f32o, (int64_t)row * ep.ldr + col, r);
#pragma unroll
                                    for (int i = 0; i < 8; i++) v[j + i] += r[i];
                                }
                                const int64_t ocol = ep.perm_hd ? qkv_unperm_row(col, ep.perm_hd) : col;
                                store_row8(ep.out, f32o, (int64_t)row * ep.ldo + ocol, v + j);
                            }
                        }
                    }
                }
            } else {
                // tile columns [0,128) = gate rows, [128,256) = up rows of the same outputs
#pragma unroll 1
                for (int c = half * 64; c < half * 64 + 64; c += 32) {
                    float g[32], u[32];
                    tmem_ld32(t_row + c, g);
                    tmem_ld32(t_row + 128 + c, u);
                    tmem_wait_ld();
                    const int ocol0 = n0 / 2 + c;
                    if (ok && row < M) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            float o[8];
#pragma unroll
                            for (int i = 0; i < 8; i++) o[i] = silu_f(g[j + i]) * u[j + i];
                            if (ocol0 + j < N / 2) store_row8(ep.out, f32o, (int64_t)row * ep.ldo + ocol0 + j, o);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acce0 + 8 * ab);
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 2 * BN);
}

// =====================================================================
// Decode GEMV (swap-AB, split-K reduced inside a thread-block cluster)
// =====================================================================
// Grid (tiles, CS) with cluster dims (1, CS, 1): the CS CTAs of a cluster
// split the K range of one 256-row weight tile.  Each CTA lays out its f32
// partial tile [NT tokens][256 rows] per owner; CTA rank r receives the
// partials of row pairs [r*128/CS, (r+1)*128/CS) from its peers by DSMEM bulk
// copies, sums them in rank order (deterministic) and runs the epilogue.
//
// Fused RMSNorm (Epi::norm_w set): the raw activation rows and the norm
// gains arrive through the ring with the weights (TMA / bulk copies); the
// converter warps turn each activation tile into bf16(x * w) in place and
// accumulate each token's sum of squares over the CTA's K range.  1/rms is a
// per-token factor of every output, so it is applied in the epilogue once the
// cluster's partial sums are added.
//
// bf16 weights: 288 threads; warp 0 TMA, warps 1 and 8 issue the MMAs of one
// 128-row half each (A and B from shared memory), warps 2-7 build normalised
// activation tiles.  int8 weights: 384 threads; warps 1 and 2 issue, and
// warps 4-11 convert: thread <-> weight row (TMEM lane quarter = warp % 4,
// half = (warp - 4) / 4) reads its 128 int8 of the K block from the 128-B
// swizzled ring (conflict-free), converts them exactly (i8x4_to_bf16x4) and
// stores the 64 bf16 pairs into a TMEM A tile with two tcgen05.st; the MMA
// takes A from TMEM.  int8 K blocks are 128 wide (32 KB of weights) so the
// per-block synchronisation is spread over twice the bytes of a 64-wide one.  Shared-memory traffic per K block is then the TMA
// writes, one read of the int8 tile and the MMAs' reads of the activations
// (no bf16 weight tile written and read back through shared memory).
// MINB: CTAs per SM the kernel is compiled for (registers); the grid is sized
// to the resident CTA slots that shared memory and MINB allow.
template <int NT, int STAGES, bool INT8, int MINB>
struct GemvCfg {
    static constexpr int KB = INT8 ? 128 : 64;      // K per block
    static constexpr int RC = KB / 8;               // 16-B activation chunks per token row per block
    static constexpr int W_BYTES = 256 * 128;       // [256 rows][128 B], 128-B swizzle (bf16 64 K, int8 128 K)
    static constexpr int X_ATOM = NT * 128;         // [NT][64] bf16, one 128-B swizzle atom wide
    static constexpr int X_BYTES = (KB / 64) * X_ATOM;
    static constexpr int G_BYTES = KB * 2;          // fused norm: the gains of the K block (bf16)
    // received partials (reuse the rings): CS slots of NT * 256 / CS values + NT sums of squares
    static constexpr int RED_BYTES = (NT * 256 + 16 * NT) * 4;
    static constexpr int RING = STAGES * (W_BYTES + X_BYTES + G_BYTES);
    static constexpr int BAR_OFF = RING > RED_BYTES ? RING : RED_BYTES;
    static constexpr int SMEM = BAR_OFF + 1024 + 512;
    static constexpr int SLOTS_SMEM = (227 * 1024 + 1024) / (SMEM + 1024);   // per SM, shared memory
    static constexpr int PER_SM = SLOTS_SMEM < MINB ? SLOTS_SMEM : MINB;
    // TMEM: accumulators [half][NT] from column 0; int8: converted A tiles
    // [2 buffers][2 halves][64 columns] from column A_COL
    static constexpr int A_COL = 128;               // int8: [2 buffers][2 halves][KB / 2 columns]
    static constexpr int TMEM_COLS = INT8 ? 512 : ((2 * NT) < 32 ? 32 : (2 * NT));
    static constexpr int THREADS = INT8 ? 384 : 288;
    static constexpr int MMA_W1 = INT8 ? 2 : 8;     // second MMA-issuing warp (the first is warp 1)
    static constexpr int CONV_W0 = INT8 ? 4 : 2;    // first converter warp
    static constexpr int N_CONV = INT8 ? 8 : 6;     // converter warps
    // An int8 CTA allocates all 512 TMEM columns (128 + 2 x 128 used; allocations
    // are powers of two).  Its shared memory (> 114 KB) leaves too little beside it
    // for any other TMEM-using CTA (the GEMV, attention, conv and GEMM kernels all
    // need more than 100 KB), so no TMEM allocation ever waits on a neighbour.
    static_assert(!INT8 || SMEM > 114 * 1024, "int8 GEMV CTAs must not share an SM with another TMEM user");
};

template <int NT, int STAGES, bool INT8, int MINB>
__global__ void __launch_bounds__(GemvCfg<NT, STAGES, INT8, MINB>::THREADS, MINB)
gemv_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
               Epi ep, int Nw, int K, int Mtok, int kb_per_split, int* err) {
    using C = GemvCfg<NT, STAGES, INT8, MINB>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* sW = smem;
    uint8_t* sX = sW + STAGES * C::W_BYTES;
    uint8_t* sG = sX + STAGES * C::X_BYTES;                      // fused norm: [STAGES][KB] gains
    float* red = reinterpret_cast<float*>(smem);   // [NT][256] received partials, after the MMAs
    constexpr int BAR_OFF = C::BAR_OFF;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BAR_OFF);
    const uint32_t full0 = smem_u32(bars);
    const uint32_t empty0 = smem_u32(bars + STAGES);
    const uint32_t cfull0 = smem_u32(bars + 2 * STAGES);       // int8: TMEM A tile [2] converted
    const uint32_t cempty0 = smem_u32(bars + 2 * STAGES + 2);  // int8: TMEM A tile [2] consumed
    const uint32_t accb = smem_u32(bars + 2 * STAGES + 4);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 5);
    const uint32_t recvb = smem_u32(bars + 2 * STAGES + 6);   // partials from the peers have landed
    const uint32_t xrdy0 = smem_u32(bars + 2 * STAGES + 7);   // [STAGES] activation tile normalised
    float* s_ss = reinterpret_cast<float*>(bars + 3 * STAGES + 7);   // [NT] sum of squares, then 1/rms
    const bool NORM = ep.norm_w != nullptr;

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int tile = blockIdx.x, split = blockIdx.y, CS = gridDim.y;
    constexpr int KB = C::KB;
    const int nk_total = (K + KB - 1) / KB;
    const int kb0 = split * kb_per_split;
    const int kb1 = min(nk_total, kb0 + kb_per_split);
    const int nk = kb1 - kb0;
    constexpr int N_CONV_WARPS = C::N_CONV;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, INT8 ? 2 + N_CONV_WARPS : 2);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(cfull0 + 8 * s, N_CONV_WARPS);
            mbar_init(cempty0 + 8 * s, 2);
        }
        mbar_init(accb, 2);
        mbar_init(recvb, 1);
        for (int s = 0; s < STAGES; s++) mbar_init(xrdy0 + 8 * s, N_CONV_WARPS);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmX);
        // Weights (and the fused norm's gains) do not depend on the previous
        // kernel: start streaming the first STAGES K-blocks before waiting for
        // it, then fetch the activations.  Gains: the K block's bytes inside K
        // (a multiple of 16, K % 8 == 0).
        auto g_bytes = [&](int i) { return (uint32_t)(2 * min(KB, K - (kb0 + i) * KB)); };
        const __nv_bfloat16* gains = reinterpret_cast<const __nv_bfloat16*>(ep.norm_w);
        const int pre = nk < STAGES ? nk : STAGES;
        for (int i = 0; i < pre; i++) {
            mbar_expect_tx(full0 + 8 * i, C::W_BYTES + C::X_BYTES + (NORM ? g_bytes(i) : 0));
            tma_load_2d(smem_u32(sW + i * C::W_BYTES), &tmW, full0 + 8 * i, (kb0 + i) * KB, tile * 256);
            if (NORM) bulk_load(smem_u32(sG + i * C::G_BYTES), gains + (kb0 + i) * KB, g_bytes(i), full0 + 8 * i);
        }
        pdl_wait();
        for (int i = 0; i < pre; i++)
            for (int a = 0; a < KB / 64; a++)
                tma_load_2d(smem_u32(sX + i * C::X_BYTES + a * C::X_ATOM), &tmX, full0 + 8 * i, (kb0 + i) * KB + 64 * a, 0);
        int issued = pre;
        for (int i = pre; i < nk; i++) {
            int s = i % STAGES;
            if (!mbar_wait(empty0 + 8 * s, ((i / STAGES) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) break;
            mbar_expect_tx(full0 + 8 * s, C::W_BYTES + C::X_BYTES + (NORM ? g_bytes(i) : 0));
            int kcoord = (kb0 + i) * KB;
            tma_load_2d(smem_u32(sW + s * C::W_BYTES), &tmW, full0 + 8 * s, kcoord, tile * 256);
            if (NORM) bulk_load(smem_u32(sG + s * C::G_BYTES), gains + kcoord, g_bytes(i), full0 + 8 * s);
            for (int a = 0; a < KB / 64; a++)
                tma_load_2d(smem_u32(sX + s * C::X_BYTES + a * C::X_ATOM), &tmX, full0 + 8 * s, kcoord + 64 * a, 0);
            issued = i + 1;
        }
        for (int i = (issued > STAGES ? issued - STAGES : 0); i < issued; i++)
            mbar_wait(full0 + 8 * (i % STAGES), (i / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL);
    } else if ((warp == 1 || warp == C::MMA_W1) && lane == 0) {
        // two issuing threads: warp 1 the weight rows [0, 128) of the tile, the
        // other the rows [128, 256), into separate accumulators
        constexpr uint32_t idesc = idesc_bf16_f32(128, NT, false, false);
        const int h = warp == 1 ? 0 : 1;
        for (int i = 0; i < nk; i++) {
            int s = i % STAGES;
            uint32_t w_base = 0;
            if (INT8) {
                int c = i & 1;
                if (!mbar_wait(cfull0 + 8 * c, (i >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                if (!mbar_wait(full0 + 8 * s, (i / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
            } else {
                if (!mbar_wait(full0 + 8 * s, (i / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
                if (NORM && !mbar_wait(xrdy0 + 8 * s, (i / STAGES) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                w_base = smem_u32(sW + s * C::W_BYTES);
            }
            tc_fence_after();
            uint32_t x_base = smem_u32(sX + s * C::X_BYTES);
#pragma unroll
            for (int kk = 0; kk < KB / 16; kk++) {
                const uint64_t bd = sdesc_sw128(x_base + (kk >> 2) * C::X_ATOM + (kk & 3) * 32, 16, 1024);
                if (INT8) {
                    // A: this half's converted tile, K slice kk = 8 TMEM columns
                    const uint32_t a_tmem = tmem + C::A_COL + (i & 1) * KB + h * (KB / 2) + kk * 8;
                    umma_f16_ts(tmem + h * NT, a_tmem, bd, idesc, (i | kk) != 0);
                } else {
                    const uint64_t ad = sdesc_sw128(w_base + h * 128 * 128 + kk * 32, 16, 1024);
                    umma_f16_ss(tmem + h * NT, ad, bd, idesc, (i | kk) != 0);
                }
            }
            if (INT8) umma_commit(cempty0 + 8 * (i & 1));
            umma_commit(empty0 + 8 * s);
        }
        umma_commit(accb);
    } else if ((INT8 || NORM) && warp >= C::CONV_W0 && warp < C::CONV_W0 + C::N_CONV) {
        // ---------------- converter warps: the normalised activation tile (when
        // the RMSNorm is fused) and int8 -> bf16 weights into TMEM (int8 path)
        constexpr int CT = 32 * C::N_CONV;                  // converter threads
        const int ct = threadIdx.x - 32 * C::CONV_W0;       // 0 .. CT - 1
        constexpr int RC = C::RC;
        constexpr int XI = (NT * RC + CT - 1) / CT;         // 16-B activation chunks per thread per stage
        float ssv[XI];   // sum of squares of this thread's raw activation chunks (one row each)
#pragma unroll
        for (int u = 0; u < XI; u++) ssv[u] = 0.f;
        for (int i = 0; i < nk; i++) {
            int s = i % STAGES, c = i & 1;
            // the stage's weights, raw activations and gains have landed (for the int8
            // path this also means the MMAs of stage i - STAGES are done)
            if ((INT8 || NORM) && !mbar_wait(full0 + 8 * s, (i / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
            if (NORM) {
                // x tile [KB / 64 atoms][NT rows][64 k] bf16, 128-B swizzle, rewritten in
                // place as bf16(x[m,k] * w[k]); rows past the tokens and columns past K
                // arrived as zeros.  The per-token 1/rms is a common factor of each
                // output and is applied in the epilogue.
                uint8_t* xt = sX + s * C::X_BYTES;
                const uint8_t* gt = sG + s * C::G_BYTES;
                const int kbase = (kb0 + i) * KB;
#pragma unroll
                for (int u = 0; u < XI; u++) {
                    const int it = ct + u * CT;
                    if (it < NT * RC) {
                        // token m, physical chunk cc of its row (atom cc / 8, swizzled chunk cc % 8)
                        const int m = it / RC, cc = it % RC;
                        const int kk = 64 * (cc >> 3) + 8 * ((cc & 7) ^ (m & 7));
                        uint4* px = reinterpret_cast<uint4*>(xt + (cc >> 3) * C::X_ATOM + m * 128 + (cc & 7) * 16);
                        const uint4 xv = *px;
                        const uint4 gv = kbase + kk < K ? *reinterpret_cast<const uint4*>(gt + 2 * kk) : make_uint4(0, 0, 0, 0);
                        const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w};
                        const uint32_t ga[4] = {gv.x, gv.y, gv.z, gv.w};
                        uint32_t o[4];
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const float a0 = bf16_lo(xa[j]), a1 = bf16_hi(xa[j]);
                            ssv[u] += a0 * a0 + a1 * a1;
                            o[j] = pack_bf16x2(a0 * bf16_lo(ga[j]), a1 * bf16_hi(ga[j]));
                        }
                        *px = make_uint4(o[0], o[1], o[2], o[3]);
                    }
                }
                if (!INT8) {
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xrdy0 + 8 * s);
                }
            }
            if (INT8) {
                // TMEM A buffer c is free once the MMAs of stage i - 2 are done
                if (i >= 2 && !mbar_wait(cempty0 + 8 * c, ((i >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                tc_fence_after();
                // thread <-> weight row r; the ring holds [256 rows][128 B] with the
                // 128-B swizzle (16-B chunk index ^= row % 8); two halves of 64 K
                const int q = warp & 3, hc = (warp - C::CONV_W0) >> 2;
                const int r = hc * 128 + q * 32 + lane;
                const uint8_t* src = sW + s * C::W_BYTES + r * 128;
                const uint32_t a_dst = tmem + ((uint32_t)(q * 32) << 16) + C::A_COL + c * KB + hc * (KB / 2);
#pragma unroll
                for (int hb = 0; hb < 2; hb++) {
                    uint4 raw[4];
#pragma unroll
                    for (int ch = 0; ch < 4; ch++)
                        raw[ch] = *reinterpret_cast<const uint4*>(src + (((hb * 4 + ch) ^ (r & 7)) << 4));
                    uint32_t o[32];   // column ch * 8 + 2j (+1): K = 64 hb + 16 ch + 4j .. + 3
#pragma unroll
                    for (int ch = 0; ch < 4; ch++) {
                        i8x4_to_bf16x4(raw[ch].x, o[ch * 8 + 0], o[ch * 8 + 1]);
                        i8x4_to_bf16x4(raw[ch].y, o[ch * 8 + 2], o[ch * 8 + 3]);
                        i8x4_to_bf16x4(raw[ch].z, o[ch * 8 + 4], o[ch * 8 + 5]);
                        i8x4_to_bf16x4(raw[ch].w, o[ch * 8 + 6], o[ch * 8 + 7]);
                    }
                    tmem_st32u(a_dst + hb * 32, o);
                }
                tmem_wait_st();
                tc_fence_before();
                if (NORM) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the activation tile
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(cfull0 + 8 * c);
                    mbar_arrive(empty0 + 8 * s);
                }
            }
        }
        if (NORM) {
            // the RC chunks of a row sit in RC consecutive lanes: partial sum of squares
            // of each token row over this CTA's K range
#pragma unroll
            for (int u = 0; u < XI; u++) {
                float v = ssv[u];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                if (RC == 16) v += __shfl_xor_sync(0xffffffffu, v, 8);
                const int it = ct + u * CT;
                if ((lane & (RC - 1)) == 0 && it < NT * RC) s_ss[it / RC] = v;
            }
        }
    }
    __syncwarp();

    // ---------------- accumulator -> registers
    pdl_wait();   // (already satisfied: the activations arrived) before any global write
    bool ok = mbar_wait(accb, 0, err, DEV_ERR_TIMEOUT_ACC);
    ok = __all_sync(0xffffffffu, ok);
    __syncwarp();
    tc_fence_after();
    // Every MMA of this CTA has completed and every TMA landed: its rings may
    // now be overwritten by peers' partials (first half of a split barrier).
    // Relaxed: the rings' last readers and writers are the async proxy's, done
    // as the accumulator barrier shows, and this thread has no shared or global
    // writes the peers need; the mbarrier initialisation was published by its
    // fence.mbarrier_init.release.cluster.  A release arrive waits for the
    // thread's outstanding memory operations, which under the next kernel's
    // weight stream cost 1-2 us per launch (decode step -3.5% without it).
    if (CS > 1) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
    const int q = warp & 3, part = warp >> 2;
    constexpr int TP = NT / 2;   // tokens per thread
    const int l = q * 32 + lane;
    const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16);
    float acc[2][TP];
    const bool ewarp = warp < 8;   // warps 0-7 hold the accumulator; warps 8+ only join the barriers
    if (ewarp) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            if (TP == 8) tmem_ld8(t_row + h * NT + part * TP, acc[h]);
            else if (TP == 16) tmem_ld16(t_row + h * NT + part * TP, acc[h]);
            else tmem_ld32(t_row + h * NT + part * TP, acc[h]);
        }
        tmem_wait_ld();
    }
    if (nk <= 0 || !ok || !ewarp) {
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int t = 0; t < TP; t++) acc[h][t] = 0.f;
    }
    tc_fence_before();
    __syncthreads();   // every MMA has read its smem operands; the rings are free
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);

    const bool f32o = ep.out_f32 != 0;
    auto store = [&](int m, int n, float o) {
        int64_t off = (int64_t)m * ep.ldo + n;
        if (f32o) reinterpret_cast<float*>(ep.out)[off] = o;
        else reinterpret_cast<__nv_bfloat16*>(ep.out)[off] = __float2bfloat16_rn(o);
    };
    // Epilogue of (token m, row pair p): gate/first row p, second row p + 128 of the tile.
    // A thread's row pair is fixed (the CS == 1 path: p = l; the cluster path: 256 is a
    // multiple of P), so its per-pair inputs (scales, bias, RoPE position and angle) are
    // loaded once; per token only the residual is read.
    struct PairK {
        int p, n0, n1;
        bool in0, in1;
        float sc0, sc1, bi0, bi1;
        int kind, hd, hh, H, ri, posb;   // RoPE: kind 0 q, 1 k, 2 v, 3 no head
        float2 cs;
    };
    auto pair_consts = [&](int p) {
        PairK k{};
        k.p = p;
        k.n0 = tile * 256 + p;
        k.n1 = k.n0 + 128;
        k.in0 = k.n0 < Nw;
        k.in1 = k.n1 < Nw;
        k.sc0 = (ep.scale && k.in0) ? ep.scale[k.n0] : 1.f;
        k.sc1 = (ep.scale && k.in1) ? ep.scale[k.n1] : 1.f;
        k.bi0 = (ep.bias && !ep.swiglu && k.in0) ? ep.bias[k.n0] : 0.f;
        k.bi1 = (ep.bias && !ep.swiglu && k.in1) ? ep.bias[k.n1] : 0.f;
        if (ep.rope_tab) {
            k.hd = ep.perm_hd;
            k.hh = k.hd / 2;
            k.H = tile * (256 / k.hd) + p / k.hh;
            k.ri = p % k.hh;
            k.kind = k.H < ep.rope_hq ? 0 : k.H < ep.rope_hq + ep.rope_hkv ? 1 : k.H < ep.rope_hq + 2 * ep.rope_hkv ? 2 : 3;
            k.posb = ep.pos_ptr ? *ep.pos_ptr : ep.pos_host;
            k.cs = make_float2(1.f, 0.f);
            if (ep.rope_s_new == 1 && k.kind <= 1 && k.posb >= 0 && k.posb < ep.max_seq)
                k.cs = ep.rope_tab[(int64_t)k.posb * k.hh + k.ri];
        }
        return k;
    };
    auto load_resid = [&](const PairK& k, int m, float& r0, float& r1) {
        r0 = r1 = 0.f;
        if (!ep.resid || ep.swiglu || ep.rope_tab || m >= Mtok) return;
        const int64_t roff = (int64_t)m * ep.ldr;
        if (f32o) {
            if (k.in0) r0 = reinterpret_cast<const float*>(ep.resid)[roff + k.n0];
            if (k.in1) r1 = reinterpret_cast<const float*>(ep.resid)[roff + k.n1];
        } else {
            if (k.in0) r0 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(ep.resid)[roff + k.n0]);
            if (k.in1) r1 = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(ep.resid)[roff + k.n1]);
        }
    };
    auto finish = [&](const PairK& k, int m, float a0, float a1, float r0, float r1) {
        if (NORM) {
            a0 *= s_ss[m];   // 1 / rms of token m
            a1 *= s_ss[m];
        }
        if (ep.rope_tab) {
            // (a0, a1) = dims (i, i + hd/2) of head slot H; the projection is rounded
            // to bf16 first, as the unfused path stores it, then rotated (rotate-half)
            if (k.kind == 3) return;
            const int b = m / ep.rope_s_new, s = m % ep.rope_s_new;
            const int pos = k.posb + s;
            if (pos < 0 || pos >= ep.max_seq) {
                atomicOr(err, 1 << 5);
                return;
            }
            a0 *= k.sc0;
            a1 *= k.sc1;
            float x0 = __bfloat162float(__float2bfloat16_rn(a0)), x1 = __bfloat162float(__float2bfloat16_rn(a1));
            __nv_bfloat16* dst;
            if (k.kind <= 1) {
                const float2 cs = ep.rope_s_new == 1 ? k.cs : ep.rope_tab[(int64_t)pos * k.hh + k.ri];
                const float y0 = x0 * cs.x - x1 * cs.y, y1 = x1 * cs.x + x0 * cs.y;
                x0 = y0;
                x1 = y1;
            }
            if (k.kind == 0)
                dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (int64_t)m * ep.ldo + (int64_t)k.H * k.hd;
            else if (k.kind == 1)
                dst = reinterpret_cast<__nv_bfloat16*>(ep.kcache) +
                      (((int64_t)b * ep.rope_hkv + (k.H - ep.rope_hq)) * ep.max_seq + pos) * k.hd;
            else
                dst = reinterpret_cast<__nv_bfloat16*>(ep.vcache) +
                      (((int64_t)b * ep.rope_hkv + (k.H - ep.rope_hq - ep.rope_hkv)) * ep.max_seq + pos) * k.hd;
            dst[k.ri] = __float2bfloat16_rn(x0);
            dst[k.ri + k.hh] = __float2bfloat16_rn(x1);
            return;
        }
        if (ep.swiglu) {
            if (k.in1) store(m, tile * 128 + k.p, silu_f(a0 * k.sc0) * (a1 * k.sc1));
            return;
        }
        // acc * scale + bias, then + residual (added only when present, so -0 stays -0)
        float o0 = a0 * k.sc0 + k.bi0, o1 = a1 * k.sc1 + k.bi1;
        if (ep.resid) {
            o0 += r0;
            o1 += r1;
        }
        if (k.in0) store(m, k.n0, o0);
        if (k.in1) store(m, k.n1, o1);
    };

    const float inv_k = 1.0f / (float)K;
    if (CS == 1) {
        if (NORM) {
            if (threadIdx.x < NT) s_ss[threadIdx.x] = rsqrtf(s_ss[threadIdx.x] * inv_k + ep.norm_eps);
            __syncthreads();
        }
        if (ok && ewarp) {
            const PairK k = pair_consts(l);
#pragma unroll
            for (int t = 0; t < TP; t++) {
                const int m = part * TP + t;
                if (m < Mtok) {
                    float r0, r1;
                    load_resid(k, m, r0, r1);
                    finish(k, m, acc[0][t], acc[1][t], r0, r1);
                }
            }
        }
        return;
    }
    // Rank r of the cluster owns row pairs [r*P, (r+1)*P), P = 128 / CS, and
    // receives every peer's partial of them into receive slot [peer rank]
    // (layout [token][pair][2]) of its own ring area.  Each thread pushes its
    // TP tokens of one row pair straight from registers with st.async, which
    // completes on the owner's mbarrier; its own slot is written locally.
    // Owners sum the CS slots in rank order (deterministic).  The split
    // cluster barrier guarantees a peer's rings are idle before it is written.
    // With the norm fused, every slot also carries the sender's NT partial sums
    // of squares; each owner adds them in rank order to form 1 / rms.
    {
        const int P = 128 / CS;
        const int PF = NT * P * 2;                         // partial floats per slot, [token][pair][2]
        const int SF = PF + NT;                            // slot floats (+ sums of squares)
        float* recvf = red;
        const int owner = l / P, pl = l % P;
        if (threadIdx.x == 0) mbar_expect_tx(recvb, (uint32_t)((CS - 1) * (PF + (NORM ? NT : 0)) * 4));
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");   // all peers' rings are free
        if (ewarp) {
            const int off = split * SF + (part * TP * P + pl) * 2;   // token part * TP, pair pl
            if (owner == split) {
#pragma unroll
                for (int t = 0; t < TP; t++)
                    *reinterpret_cast<float2*>(recvf + off + t * P * 2) = make_float2(acc[0][t], acc[1][t]);
            } else {
                uint32_t rdst, rbar;
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rdst) : "r"(smem_u32(recvf + off)), "r"(owner));
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(recvb), "r"(owner));
#pragma unroll
                for (int t = 0; t < TP; t++)
                    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                                     rdst + t * P * 8),
                                 "f"(acc[0][t]), "f"(acc[1][t]), "r"(rbar)
                                 : "memory");
            }
        }
        if (NORM && ewarp) {
            for (int it = threadIdx.x; it < CS * NT; it += 256) {
                const int r = it / NT, m = it % NT;
                const uint32_t dst = smem_u32(recvf + split * SF + PF + m);
                if (r == split) {
                    recvf[split * SF + PF + m] = s_ss[m];
                } else {
                    uint32_t rdst, rbar;
                    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rdst) : "r"(dst), "r"(r));
                    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rbar) : "r"(recvb), "r"(r));
                    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(rdst),
                                 "f"(s_ss[m]), "r"(rbar)
                                 : "memory");
                }
            }
        }
        // this thread's epilogue items: row pair pl2 of the owned slice, tokens
        // m = m_first + u * (ET / P); every thread of the int8 CTA (384, a multiple
        // of P <= 64) takes items, the first 256 otherwise.  Their per-pair constants
        // and first residuals are loaded now, while the partials are in flight.
        constexpr int ET = INT8 ? C::THREADS : 256;
        constexpr int MAXI = 4;
        const bool eth = threadIdx.x < ET;
        const int pl2 = threadIdx.x % P, mstep = ET / P, m0 = threadIdx.x / P;
        PairK kc{};
        float rr0[MAXI], rr1[MAXI];
#pragma unroll
        for (int u = 0; u < MAXI; u++) rr0[u] = rr1[u] = 0.f;
        if (eth) {
            kc = pair_consts(split * P + pl2);
#pragma unroll
            for (int u = 0; u < MAXI; u++)
                if (m0 + u * mstep < NT) load_resid(kc, m0 + u * mstep, rr0[u], rr1[u]);
        }
        const bool got = __all_sync(0xffffffffu, mbar_wait(recvb, 0, err, DEV_ERR_TIMEOUT_MISC));
        __syncthreads();   // the local slot, written by other threads
        if (NORM) {
            if (threadIdx.x < NT) {
                float v[16];   // all loads in flight, then a fixed-order sum
#pragma unroll
                for (int r = 0; r < 16; r++) v[r] = r < CS ? recvf[r * SF + PF + threadIdx.x] : 0.f;
                float t = 0.f;
#pragma unroll
                for (int r = 0; r < 16; r++) t += v[r];
                s_ss[threadIdx.x] = rsqrtf(t * inv_k + ep.norm_eps);
            }
            __syncthreads();
        }
        if (eth && ok && got) {
            const PairK& k = kc;
            for (int u = 0, m = m0; m < NT; u++, m += mstep) {
                float r0 = 0.f, r1 = 0.f;
                if (u >= MAXI) load_resid(k, m, r0, r1);
#pragma unroll
                for (int j = 0; j < MAXI; j++)
                    if (u == j) {
                        r0 = rr0[j];
                        r1 = rr1[j];
                    }
                float2 v[16];   // all loads in flight, then a fixed-order sum
#pragma unroll
                for (int r = 0; r < 16; r++)
                    v[r] = r < CS ? *reinterpret_cast<const float2*>(recvf + r * SF + (m * P + pl2) * 2) : make_float2(0.f, 0.f);
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int r = 0; r < 16; r++) {
                    a0 += v[r].x;
                    a1 += v[r].y;
                }
                if (m < Mtok) finish(k, m, a0, a1, r0, r1);
            }
        }
    }
}

// =====================================================================
// f32 CUDA-core paths (exact f32 FMA accumulate)
// =====================================================================
// 64x64 output tile, 256 threads, 4x4 outputs per thread, K-slices of 32
// (the next slice is loaded into registers while the current one is
// multiplied from shared memory).  Small grids split K over a thread-block
// cluster (gridDim.z CTAs); the partial tiles are summed over DSMEM in rank
// order (deterministic), each rank finishing 64 / splits rows.
// B_KN: b is [K, N] (matmul_forward); else b is [N, K] (linear_forward).
// lda: row stride of a; ldy: row stride of y and of the residual.
template <bool B_KN>
__global__ void __launch_bounds__(256)
gemm_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, const float* __restrict__ bias,
                const float* __restrict__ resid, float* __restrict__ y, int M, int N, int K, int k_per_split,
                int64_t lda, int64_t ldy) {
    __shared__ float sa[2][32][64 + 4];
    __shared__ float sb[2][32][64 + 4];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int split = blockIdx.z, S = gridDim.z;
    const int kbeg = split * k_per_split, kend = min(K, kbeg + k_per_split);
    const int nsl = kend > kbeg ? (kend - kbeg + 31) / 32 : 0;
    float acc[4][4] = {};
    float ra[8], rb[8];
    auto load = [&](int sl) {
        const int k0 = kbeg + sl * 32;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int e = tid + 256 * u;
            {
                const int r = e / 32, kk = e % 32, gm = m0 + r, gk = k0 + kk;
                ra[u] = (gm < M && gk < kend) ? a[(int64_t)gm * lda + gk] : 0.f;
            }
            if (B_KN) {
                const int kr = e / 64, c = e % 64, gn = n0 + c, gk = k0 + kr;
                rb[u] = (gn < N && gk < kend) ? b[(int64_t)gk * N + gn] : 0.f;
            } else {
                const int r = e / 32, kk = e % 32, gn = n0 + r, gk = k0 + kk;
                rb[u] = (gn < N && gk < kend) ? b[(int64_t)gn * K + gk] : 0.f;
            }
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int u = 0; u < 8; u++) {
            const int e = tid + 256 * u;
            sa[buf][e % 32][e / 32] = ra[u];
            if (B_KN) sb[buf][e / 64][e % 64] = rb[u];
            else sb[buf][e % 32][e / 32] = rb[u];
        }
    };
    if (nsl > 0) {
        load(0);
        store(0);
    }
    __syncthreads();
    for (int sl = 0; sl < nsl; sl++) {
        const int buf = sl & 1;
        if (sl + 1 < nsl) load(sl + 1);
#pragma unroll
        for (int kk = 0; kk < 32; kk++) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                av[i] = sa[buf][kk][ty + 16 * i];
                bv[i] = sb[buf][kk][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        if (sl + 1 < nsl) store(buf ^ 1);
        __syncthreads();
    }
    auto finish = [&](int m, int n, float v) {
        if (m >= M || n >= N) return;
        if (bias) v += bias[n];
        if (resid) v += resid[(int64_t)m * ldy + n];
        y[(int64_t)m * ldy + n] = v;
    };
    if (S == 1) {
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) finish(m0 + ty + 16 * i, n0 + tx + 16 * j, acc[i][j]);
        return;
    }
    // partial tile [64][64] -> this CTA's shared memory (sa reused), then rank r
    // sums rows [r * 64 / S, (r + 1) * 64 / S) of all S partials over DSMEM
    float* part = &sa[0][0][0];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) part[(ty + 16 * i) * 64 + tx + 16 * j] = acc[i][j];
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
    const int rows = 64 / S;
    const uint32_t base = smem_u32(part);
    for (int e = tid; e < rows * 64; e += 256) {
        const int r = split * rows + e / 64, c = e % 64;
        float v = 0.f;
        for (int q = 0; q < S; q++) {
            uint32_t addr;
            float t;
            asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(addr) : "r"(base + (uint32_t)(r * 64 + c) * 4), "r"(q));
            asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(t) : "r"(addr) : "memory");
            v += t;
        }
        finish(m0 + r, n0 + c, v);
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Launches gemm_f32_kernel, splitting K over a cluster of up to 8 CTAs when
// the output tiles alone would leave most SMs idle.
template <bool B_KN>
static int launch_gemm_f32(tb_ctx* ctx, const float* a, const float* b, const float* bias, const float* resid, float* y,
                           int M, int N, int K, int64_t lda, int64_t ldy) {
    const int tiles = ((N + 63) / 64) * ((M + 63) / 64);
    int S = 1;
    while (S < 8 && tiles * S * 2 <= ctx->num_sms && K / (S * 2) >= 64) S *= 2;
    const int kps = (K + S - 1) / S;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)((N + 63) / 64), (unsigned)((M + 63) / 64), (unsigned)S);
    lc.blockDim = dim3(256, 1, 1);
    lc.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = S;
    lc.attrs = attr;
    lc.numAttrs = 1;
    TB_CUDA_TRY(ctx, cudaLaunchKernelEx(&lc, gemm_f32_kernel<B_KN>, a, b, bias, resid, y, M, N, K, kps, lda, ldy));
    return check_launch(ctx, "gemm_f32");
}

// ------------------------------------------------------------ host side --
template <int BN, int STAGES, bool B_MN>
static int launch_gemm_tc(tb_ctx* ctx, const void* a, const void* b, const Epi& ep, int M, int N, int K) {
    CUtensorMap ta, tbm;
    int rc = make_tmap_2d(ctx, &ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a, M, K, ep.x_ld ? ep.x_ld : K, 64, GEMM_BM);
    if (rc) return rc;
    if (!B_MN) rc = make_tmap_2d(ctx, &tbm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, N, K, K, 64, BN);
    else rc = make_tmap_2d(ctx, &tbm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b, K, N, N, 64, 64);
    if (rc) return rc;
    constexpr int smem = gemm_smem_bytes<BN, STAGES>();
    auto kern = gemm_tc_kernel<BN, STAGES, B_MN>;
    TB_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int mt = (M + GEMM_BM - 1) / GEMM_BM;
    const int64_t tiles = (int64_t)((N + BN - 1) / BN) * mt;
    const int grid = (int)(tiles < ctx->num_sms ? tiles : ctx->num_sms);
    // row tiles per raster group: the most (a power of two) whose activation
    // rows fit in 32 MB of L2
    const int64_t row_bytes = (int64_t)GEMM_BM * K * 2;
    int gm = 1;
    while (gm * 2 <= mt && (int64_t)gm * 2 * row_bytes <= (32ll << 20)) gm *= 2;
    return launch(ctx, "gemm_tc", kern, dim3(grid), dim3(GEMM_THREADS), smem, ta, tbm, ep, M, N, K, gm, ctx->d_err);
}

// Cluster size (K splits per weight tile): the largest of 8, 4, 2, 1 that
// keeps the grid within two CTAs per SM and every split >= 2 K-blocks.
// Split-K factor: the largest power of two <= max_cs that keeps the grid
// within the resident CTA slots (one wave; with two slots per SM the next
// kernel's CTAs can start streaming their weights early) and gives every CTA
// at least two K-blocks.
static void gemv_split(int slots, int max_cs, int Nw, int K, int KB, int* splits_out, int* kb_per_out) {
    const int tiles = (Nw + 255) / 256;
    const int nk = (K + KB - 1) / KB;
    int cs = max_cs;
    while (cs > 1 && (tiles * cs > slots || nk < 2 * cs)) cs >>= 1;
    int kb_per = (nk + cs - 1) / cs;
    *splits_out = cs;
    *kb_per_out = kb_per;
}

template <int NT, int STAGES, bool INT8, int MINB>
static int launch_gemv_tc(tb_ctx* ctx, const void* x, const void* w, const Epi& ep, int Mtok, int Nw, int K) {
    using C = GemvCfg<NT, STAGES, INT8, MINB>;
    CUtensorMap tw, tx;
    int rc;
    if (INT8) {
        uint64_t dims[2] = {(uint64_t)K, (uint64_t)Nw};
        uint64_t strides[1] = {(uint64_t)K};
        uint32_t box[2] = {128, 256};
        rc = make_tmap(ctx, &tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
    } else {
        rc = make_tmap_2d(ctx, &tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, Nw, K, K, 64, 256);
    }
    if (rc) return rc;
    rc = make_tmap_2d(ctx, &tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, Mtok, K, ep.x_ld ? ep.x_ld : K, 64, NT);
    if (rc) return rc;
    Epi e2 = ep;
    e2.x_ld = ep.x_ld ? ep.x_ld : K;
    e2.norm_x = x;
    auto kern = gemv_tc_kernel<NT, STAGES, INT8, MINB>;
    // bf16: clusters of 16 (non-portable) when the device can co-schedule them,
    // else 8.  int8 (one CTA per SM, converter-bound) is fastest at 8.
    static std::atomic<int> max_cs{INT8 ? 8 : 0};
    if (max_cs.load() == 0) {
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        int n = 0;
        cudaLaunchConfig_t q = {};
        q.gridDim = dim3(1, 16, 1);
        q.blockDim = dim3(C::THREADS, 1, 1);
        q.dynamicSmemBytes = C::SMEM;
        cudaLaunchAttribute qa[1];
        qa[0].id = cudaLaunchAttributeClusterDimension;
        qa[0].val.clusterDim.x = 1;
        qa[0].val.clusterDim.y = 16;
        qa[0].val.clusterDim.z = 1;
        q.attrs = qa;
        q.numAttrs = 1;
        const bool ok16 = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess &&
                          cudaOccupancyMaxActiveClusters(&n, kern, &q) == cudaSuccess && n >= 1;
        cudaGetLastError();
        max_cs.store(ok16 ? 16 : 8);
    }
    int cs, kb_per;
    gemv_split(C::PER_SM * ctx->num_sms, max_cs.load(), Nw, K, C::KB, &cs, &kb_per);
    const int tiles = (Nw + 255) / 256;
    TB_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(tiles, cs, 1);
    lc.blockDim = dim3(C::THREADS, 1, 1);
    lc.dynamicSmemBytes = C::SMEM;
    lc.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cs;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (ctx->pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        lc.numAttrs = 2;
    }
    TB_CUDA_TRY(ctx, cudaLaunchKernelEx(&lc, kern, tw, tx, e2, Nw, K, Mtok, kb_per, ctx->d_err));
    return check_launch(ctx, "gemv_tc");
}

template <bool INT8>
static int dispatch_gemv(tb_ctx* ctx, const void* x, const void* w, const Epi& ep, int M, int N, int K) {
    // <= 32 tokens: 3-stage rings (~105 KB) let two CTAs share an SM, so the
    // next layer's GEMV can start streaming weights (PDL) beside this one.
    // (Measured on C4 and not kept: 2-stage rings with three CTAs per SM -6%;
    // one CTA per SM with 6-stage rings for grids of <= 148 CTAs -13%.)
    if (M <= 16) return launch_gemv_tc<16, INT8 ? 5 : 3, INT8, INT8 ? 1 : 2>(ctx, x, w, ep, M, N, K);
    if (M <= 32) return launch_gemv_tc<32, INT8 ? 5 : 3, INT8, INT8 ? 1 : 2>(ctx, x, w, ep, M, N, K);
    return launch_gemv_tc<64, INT8 ? 4 : 5, INT8, 1>(ctx, x, w, ep, M, N, K);
}

int linear_launch(tb_ctx* ctx, int int8, const void* x, const void* w, const Epi& ep, int M, int N, int K) {
    if (ep.perm_hd) {
        if ((ep.perm_hd != 64 && ep.perm_hd != 128) || N % 256 || ep.bias || ep.resid || ep.swiglu || ep.out_f32 ||
            (ep.rope_tab && ep.rope_s_new <= 0) || (!ep.rope_tab && (M <= 64 || int8)))
            return set_error(ctx, TB_ERR_UNSUPPORTED, "linear: permuted QKV epilogue configuration");
    }
    if (ep.norm_w && (M > 64 || K % 8 || ep.x_ld % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
                      (reinterpret_cast<uintptr_t>(ep.norm_w) & 15)))
        return set_error(ctx, TB_ERR_UNSUPPORTED,
                         "linear: fused norm needs <= 64 tokens, K and row stride %% 8, 16-B alignment");
    if (ep.x_ld && ep.x_ld != K && (ep.x_ld < K || ep.x_ld % 8 || (reinterpret_cast<uintptr_t>(x) & 15)))
        return set_error(ctx, TB_ERR_ALIGN, "linear: row stride of x must be >= K and a multiple of 8 elements");
    if (int8) {
        if (M > 64) return set_error(ctx, TB_ERR_UNSUPPORTED, "int8 linear: at most 64 tokens");
        return dispatch_gemv<true>(ctx, x, w, ep, M, N, K);
    }
    if (M <= 64) return dispatch_gemv<false>(ctx, x, w, ep, M, N, K);
    if (N <= 128 && !ep.swiglu) return launch_gemm_tc<128, 6, false>(ctx, x, w, ep, M, N, K);
    return launch_gemm_tc<256, 4, false>(ctx, x, w, ep, M, N, K);
}

}  // namespace tb

using namespace tb;

extern "C" {

int tb_linear_fwd_strided(tb_ctx* ctx, int dtype, const void* x, int64_t ldx, const void* w, const float* bias,
                          const void* residual, void* y, int64_t ldy, int64_t M, int64_t N, int64_t K, int flags) {
    if (!ctx || !x || !w || !y) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
               TB_ERR_SHAPE, "linear: bad shape M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
    const bool swiglu = (flags & TB_EPI_SWIGLU) != 0;
    const int64_t ncols = swiglu ? N / 2 : N;
    TB_REQUIRE(ctx, ldx >= K && ldy >= ncols, TB_ERR_SHAPE, "linear: row strides ldx=%lld < K or ldy=%lld < %lld",
               (long long)ldx, (long long)ldy, (long long)ncols);
    if (M == 0) return TB_OK;
    if ((flags & TB_EPI_BIAS) && !bias) return set_error(ctx, TB_ERR_ARG, "linear: TB_EPI_BIAS without bias");
    if ((flags & TB_EPI_RESIDUAL) && !residual) return set_error(ctx, TB_ERR_ARG, "linear: TB_EPI_RESIDUAL without residual");
    if (dtype == TB_F32) {
        if (swiglu) return set_error(ctx, TB_ERR_UNSUPPORTED, "linear f32: SwiGLU epilogue is bf16-only");
        return launch_gemm_f32<false>(ctx, (const float*)x, (const float*)w, (flags & TB_EPI_BIAS) ? bias : nullptr,
                                      (flags & TB_EPI_RESIDUAL) ? (const float*)residual : nullptr, (float*)y, (int)M,
                                      (int)N, (int)K, ldx, ldy);
    }
    if (dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "linear: dtype %d", dtype);
    TB_REQUIRE(ctx, K % 8 == 0 && N % 8 == 0, TB_ERR_SHAPE, "linear bf16: K and N must be multiples of 8");
    TB_REQUIRE(ctx, aligned16(x) && aligned16(w) && aligned16(y) && (!residual || aligned16(residual)),
               TB_ERR_ALIGN, "linear bf16: pointers must be 16-byte aligned");
    TB_REQUIRE(ctx, ldx % 8 == 0 && ldy % 8 == 0, TB_ERR_ALIGN,
               "linear bf16: row strides must be multiples of 8 elements (16 bytes)");
    if (swiglu) {
        TB_REQUIRE(ctx, N % 256 == 0, TB_ERR_SHAPE, "linear SwiGLU: N must be a multiple of 256");
        TB_REQUIRE(ctx, !(flags & (TB_EPI_BIAS | TB_EPI_RESIDUAL)), TB_ERR_UNSUPPORTED,
                   "linear SwiGLU: no bias/residual");
    }
    Epi ep{};
    ep.out = y;
    ep.out_f32 = (flags & TB_EPI_OUT_F32) ? 1 : 0;
    ep.ldo = ldy;
    ep.bias = (flags & TB_EPI_BIAS) ? bias : nullptr;
    ep.resid = (flags & TB_EPI_RESIDUAL) ? residual : nullptr;
    ep.ldr = ldy;
    ep.swiglu = swiglu ? 1 : 0;
    ep.x_ld = ldx;
    return linear_launch(ctx, 0, x, w, ep, (int)M, (int)N, (int)K);
}

int tb_linear_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias,
                  const void* residual, void* y, int64_t M, int64_t N, int64_t K, int flags) {
    const int64_t ncols = (flags & TB_EPI_SWIGLU) ? N / 2 : N;
    return tb_linear_fwd_strided(ctx, dtype, x, K, w, bias, residual, y, ncols, M, N, K, flags);
}

int tb_matmul_fwd(tb_ctx* ctx, int dtype, const void* a, const void* b, void* c, int64_t M, int64_t N, int64_t K) {
    if (!ctx || !a || !b || !c) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && N > 0 && K > 0 && M < (1ll << 31) && N < (1ll << 31) && K < (1ll << 31),
               TB_ERR_SHAPE, "matmul: bad shape");
    if (M == 0) return TB_OK;
    if (dtype == TB_F32) {
        return launch_gemm_f32<true>(ctx, (const float*)a, (const float*)b, nullptr, nullptr, (float*)c, (int)M, (int)N,
                                     (int)K, K, N);
    }
    if (dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "matmul: dtype %d", dtype);
    TB_REQUIRE(ctx, K % 8 == 0 && N % 8 == 0, TB_ERR_SHAPE, "matmul bf16: K and N must be multiples of 8");
    TB_REQUIRE(ctx, aligned16(a) && aligned16(b) && aligned16(c), TB_ERR_ALIGN, "matmul bf16: alignment");
    Epi ep{};
    ep.out = c;
    ep.ldo = N;
    return launch_gemm_tc<256, 4, true>(ctx, a, b, ep, (int)M, (int)N, (int)K);
}

int tb_int8_linear_fwd(tb_ctx* ctx, const void* x, const int8_t* q, const float* scale,
                       const void* residual, void* y, int64_t M, int64_t N, int64_t K, int flags) {
    if (!ctx || !x || !q || !scale || !y) return TB_ERR_ARG;
    TB_REQUIRE(ctx, M >= 0 && M <= 64 && N > 0 && K > 0 && N < (1ll << 31) && K < (1ll << 31), TB_ERR_SHAPE,
               "int8 linear: 0 <= M <= 64 tokens (decode GEMV path)");
    if (M == 0) return TB_OK;
    TB_REQUIRE(ctx, K % 16 == 0 && N % 8 == 0, TB_ERR_SHAPE, "int8 linear: K %% 16 and N %% 8 must be 0");
    TB_REQUIRE(ctx, aligned16(x) && aligned16(q), TB_ERR_ALIGN, "int8 linear: alignment");
    if ((flags & TB_EPI_RESIDUAL) && !residual) return set_error(ctx, TB_ERR_ARG, "int8 linear: residual missing");
    const bool swiglu = (flags & TB_EPI_SWIGLU) != 0;
    if (swiglu) TB_REQUIRE(ctx, N % 256 == 0, TB_ERR_SHAPE, "int8 SwiGLU: N %% 256");
    Epi ep{};
    ep.out = y;
    ep.out_f32 = (flags & TB_EPI_OUT_F32) ? 1 : 0;
    ep.ldo = swiglu ? N / 2 : N;
    ep.resid = (flags & TB_EPI_RESIDUAL) ? residual : nullptr;
    ep.ldr = N;
    ep.scale = scale;
    ep.swiglu = swiglu ? 1 : 0;
    return linear_launch(ctx, 1, x, q, ep, (int)M, (int)N, (int)K);
}

}  // extern "C"

// Attention forward on B200.
//
//  * attn_tc_kernel<D>: flash-style forward for bf16 Q/K/V, D in {64, 128}.
//    One CTA per (128-query tile, head, batch).  Warp 0 streams K and V tiles
//    of 128 keys with TMA (two-stage ring), warp 1 issues tcgen05.mma:
//    S = Q K^T into one of two TMEM score buffers, then O += P V into a TMEM
//    accumulator.  Warps 2-5 own one query row per thread: they read the row
//    of S from TMEM, run the online softmax in the exp2 domain, rescale O in
//    TMEM when the running max grows, and write P (bf16) into a 128-B
//    swizzled shared-memory tile that the next MMA reads as its A operand.
//    The same online-softmax recurrence as flash_attention2_forward
//    (nn/attention/flash_attn2.rs:98-140), over 128-key tiles instead of one
//    key at a time, plus the causal mask and GQA head mapping.
//  * attn_decode_kernel: decode against a KV cache (few queries, long
//    context).  Split over the context; the last CTA of a (batch, kv-head)
//    group merges the partial (max, sum, output) triples.
//  * attn_f32_kernel: exact f32 path (fixtures, fp32 configurations).
#include <math.h>

#include "common.cuh"
#include "attention.h"

namespace tb {

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <int D>
struct AttnCfg {
    static constexpr int BM = 128, BN = 128;
    static constexpr int TILE = 128 * D * 2;           // Q, K or V tile bytes
    static constexpr int P_BYTES = 128 * 128 * 2;
    static constexpr int SMEM = TILE /*Q*/ + 2 * TILE /*K*/ + 2 * TILE /*V*/ + P_BYTES + 1024 + 256;
    static constexpr int O_COL = 256;                  // TMEM columns: S0 [0,128), S1 [128,256), O
};

template <int D>
__global__ void __launch_bounds__(192, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, AttnOut out, int Hq, int Hkv, int Sq, int Sk,
               float scale_log2, int causal, int* err) {
    using C = AttnCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + C::TILE;
    uint8_t* sV = sK + 2 * C::TILE;
    uint8_t* sP = sV + 2 * C::TILE;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::P_BYTES);
    const uint32_t q_full = smem_u32(bars + 0);
    const uint32_t k_full0 = smem_u32(bars + 1);     // [2]
    const uint32_t v_full0 = smem_u32(bars + 3);     // [2]
    const uint32_t kv_empty0 = smem_u32(bars + 5);   // [2]
    const uint32_t s_full0 = smem_u32(bars + 7);     // [2]
    const uint32_t p_full = smem_u32(bars + 9);
    const uint32_t o_done = smem_u32(bars + 10);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);

    pdl_trigger();
    pdl_wait();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int q_tile = gridDim.x - 1 - blockIdx.x;   // heaviest causal tiles first
    const int h = blockIdx.y, b = blockIdx.z;
    const int hk = h / (Hq / Hkv);
    const int q0 = q_tile * C::BM;
    const int diag = Sk - Sq;                         // causal: key j visible to query i iff j <= i + diag
    int n_tiles = (Sk + C::BN - 1) / C::BN;
    if (causal) {
        int last_key = q0 + C::BM - 1 + diag;
        int nt_c = last_key < 0 ? 0 : last_key / C::BN + 1;
        n_tiles = min(n_tiles, nt_c);
    }
    constexpr int DB = D / 64;                        // 64-wide d blocks per tile

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(k_full0 + 8 * s, 1);
            mbar_init(v_full0 + 8 * s, 1);
            mbar_init(kv_empty0 + 8 * s, 1);
            mbar_init(s_full0 + 8 * s, 1);
        }
        mbar_init(p_full, 128);
        mbar_init(o_done, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0 && n_tiles > 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_expect_tx(q_full, C::TILE);
            for (int d = 0; d < DB; d++) tma_load_4d(smem_u32(sQ + d * 16384), &tmQ, q_full, 64 * d, h, q0, b);
            int issued = 0;
            for (int j = 0; j < n_tiles; j++) {
                int st = j & 1;
                if (j >= 2 && !mbar_wait(kv_empty0 + 8 * st, ((j >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) break;
                mbar_expect_tx(k_full0 + 8 * st, C::TILE);
                for (int d = 0; d < DB; d++)
                    tma_load_4d(smem_u32(sK + st * C::TILE + d * 16384), &tmK, k_full0 + 8 * st, 64 * d, hk, j * C::BN, b);
                mbar_expect_tx(v_full0 + 8 * st, C::TILE);
                for (int d = 0; d < DB; d++)
                    tma_load_4d(smem_u32(sV + st * C::TILE + d * 16384), &tmV, v_full0 + 8 * st, 64 * d, hk, j * C::BN, b);
                issued = j + 1;
            }
            mbar_wait(q_full, 0, err, DEV_ERR_TIMEOUT_FULL);
            for (int j = (issued > 2 ? issued - 2 : 0); j < issued; j++) {
                mbar_wait(k_full0 + 8 * (j & 1), (j >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL);
                mbar_wait(v_full0 + 8 * (j & 1), (j >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && n_tiles > 0) {
            constexpr uint32_t idesc_s = idesc_bf16_f32(128, C::BN, false, false);
            constexpr uint32_t idesc_o = idesc_bf16_f32(128, D, false, true);
            const uint32_t q_base = smem_u32(sQ), p_base = smem_u32(sP);
            bool ok = mbar_wait(q_full, 0, err, DEV_ERR_TIMEOUT_FULL);
            for (int j = 0; ok && j <= n_tiles; j++) {
                if (j < n_tiles) {
                    int st = j & 1;
                    if (!mbar_wait(k_full0 + 8 * st, (j >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
                    tc_fence_after();
                    const uint32_t k_base = smem_u32(sK + st * C::TILE);
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                        umma_f16_ss(tmem + st * 128, sdesc_sw128(q_base + off, 16, 1024),
                                    sdesc_sw128(k_base + off, 16, 1024), idesc_s, kk != 0);
                    }
                    umma_commit(s_full0 + 8 * st);
                }
                if (j > 0) {
                    const int jp = j - 1, st = jp & 1;
                    if (!mbar_wait(p_full, jp & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                    if (!mbar_wait(v_full0 + 8 * st, (jp >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
                    tc_fence_after();
                    const uint32_t v_base = smem_u32(sV + st * C::TILE);
#pragma unroll
                    for (int kk = 0; kk < C::BN / 16; kk++) {
                        uint64_t ad = sdesc_sw128(p_base + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
                        uint64_t bd = sdesc_sw128(v_base + kk * 16 * 128, 16384, 1024);
                        umma_f16_ss(tmem + C::O_COL, ad, bd, idesc_o, (jp | kk) != 0);
                    }
                    umma_commit(kv_empty0 + 8 * st);
                    umma_commit(o_done);
                }
            }
        }
    } else {
        // ---------------- softmax warps 2..5: thread <-> query row
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const int qi = q0 + r;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        float m_run = -INFINITY, l_run = 0.f;
        bool ok = true;
        for (int j = 0; j < n_tiles; j++) {
            const int sb = j & 1;
            ok = mbar_wait(s_full0 + 8 * sb, (j >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            float s[128];
#pragma unroll
            for (int c = 0; c < 4; c++) tmem_ld32(t_lane + sb * 128 + c * 32, s + c * 32);
            tmem_wait_ld();
            const int k0 = j * C::BN;
            const int lim = causal ? min(Sk - 1, qi + diag) : Sk - 1;   // last visible key
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 128; c++) {
                float v = (k0 + c <= lim) ? s[c] * scale_log2 : -INFINITY;
                s[c] = v;
                mx = fmaxf(mx, v);
            }
            const float m_new = fmaxf(m_run, mx);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = ex2(m_run - m_use);   // m_run = -inf -> 0
            float rs = 0.f;
#pragma unroll
            for (int c = 0; c < 128; c++) {
                float p = ex2(s[c] - m_use);
                s[c] = p;
                rs += p;
            }
            l_run = l_run * alpha + rs;
            m_run = m_new;
            if (j > 0) {
                ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, err, DEV_ERR_TIMEOUT_MISC));
                if (!ok) break;
                tc_fence_after();
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                    for (int c = 0; c < D; c += 16) {
                        float o[16];
                        tmem_ld16(t_lane + C::O_COL + c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i++) o[i] *= alpha;
                        tmem_st16(t_lane + C::O_COL + c, o);
                    }
                    tmem_wait_st();
                }
            }
            // P row -> shared memory, 128-B swizzled K-major (keys) tile
            uint8_t* prow = sP + r * 128;
#pragma unroll
            for (int ch = 0; ch < 16; ch++) {
                const int kc = ch >> 3, c8 = ch & 7;
                uint4 v;
                v.x = pack_bf16x2(s[ch * 8 + 0], s[ch * 8 + 1]);
                v.y = pack_bf16x2(s[ch * 8 + 2], s[ch * 8 + 3]);
                v.z = pack_bf16x2(s[ch * 8 + 4], s[ch * 8 + 5]);
                v.w = pack_bf16x2(s[ch * 8 + 6], s[ch * 8 + 7]);
                *reinterpret_cast<uint4*>(prow + kc * 16384 + ((c8 ^ (r & 7)) << 4)) = v;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (ok && n_tiles > 0) {
            ok = __all_sync(0xffffffffu, mbar_wait(o_done, (n_tiles - 1) & 1, err, DEV_ERR_TIMEOUT_ACC));
        }
        if (ok) {
            tc_fence_after();
            const float inv_l = (l_run > 0.f) ? 1.0f / l_run : 0.f;
            const bool valid = qi < Sq;
            const int64_t obase = (int64_t)b * out.o_sb + (int64_t)h * out.o_sh + (int64_t)qi * out.o_ss;
#pragma unroll 1
            for (int c = 0; c < D; c += 32) {
                float o[32];
                if (n_tiles > 0) {
                    tmem_ld32(t_lane + C::O_COL + c, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int i = 0; i < 32; i++) o[i] = 0.f;
                }
                if (valid) {
                    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out.o) + obase + c;
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint4 v;
                        v.x = pack_bf16x2(o[i] * inv_l, o[i + 1] * inv_l);
                        v.y = pack_bf16x2(o[i + 2] * inv_l, o[i + 3] * inv_l);
                        v.z = pack_bf16x2(o[i + 4] * inv_l, o[i + 5] * inv_l);
                        v.w = pack_bf16x2(o[i + 6] * inv_l, o[i + 7] * inv_l);
                        *reinterpret_cast<uint4*>(dst + i) = v;
                    }
                }
            }
            if (valid && out.lse) {
                float lse = (l_run > 0.f) ? (m_run + log2f(l_run)) * kLn2 : -INFINITY;
                out.lse[((int64_t)b * Hq + h) * Sq + qi] = lse;
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// -------------------------------------------------------------- decode -----
// Decode attention against the KV cache: a few queries, a long context.
// Grid (B * Hkv, DEC_CTAS) in clusters of (1, DEC_CTAS, 1), 4 warps per CTA:
// the 4 * DEC_CTAS warps of a cluster split the context of one (batch, kv
// head) group into `chunk`-key ranges (a multiple of 32).  A warp streams its
// range in 32-key slabs: one lane issues 1-D bulk async copies (TMA engine)
// of the slab's contiguous K and V rows into the warp's double-buffered
// shared memory, so the next slab is in flight while this one is processed.
// Lane j scores key j against the G = Hq / Hkv queries (broadcast from shared
// memory; the K row is read in a lane-rotated chunk order, conflict-free),
// the slab's max / exp / sum run on warp shuffles (online softmax), and the
// P V product gives each lane D/32 output dims of every head.  Partials
// (max, sum, o) stay in shared memory; after a cluster barrier CTA rank r
// merges output dims [r*D/DEC_CTAS, ...) of every head over DSMEM, in fixed
// order (deterministic).  D = 64 or 128, G in {1, 2, 4, 8}.
constexpr int DEC_CTAS = 2;                 // cluster size (8 warp-splits per group: one wave at 2 CTAs per SM)
constexpr int DEC_WARPS = 4;                // warps per CTA
constexpr int DEC_SPLITS = DEC_CTAS * DEC_WARPS;

__device__ __forceinline__ void dec_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float dec_ld_dsmem(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote));
    return v;
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

template <int D>
struct DecSmem {
    static constexpr int SLAB = 32 * D * 2;                        // bytes of K (or V) per slab
    static constexpr int KV = DEC_WARPS * 2 * 2 * SLAB;            // [warp][buf][K|V]
    static constexpr int BYTES = KV + 8 * D * 4 /*sq*/ + DEC_WARPS * 32 * 8 * 4 /*sp*/ +
                                 DEC_WARPS * 8 * (D + 2) * 4 /*partials*/ + DEC_WARPS * 2 * 8 /*bars*/ + 128;
};

template <int D, int G>
__global__ void __launch_bounds__(128)
attn_decode_kernel(DecodeArgs a, int* err) {
    constexpr int DPL = D / 32;                       // output dims per lane
    using SM = DecSmem<D>;
    extern __shared__ __align__(128) uint8_t dsm[];
    uint8_t* kv = dsm;                                              // [warp][buf][K|V][32][D] bf16
    float (*sq)[D] = reinterpret_cast<float (*)[D]>(dsm + SM::KV);
    float (*sp)[32][8] = reinterpret_cast<float (*)[32][8]>(dsm + SM::KV + 8 * D * 4);
    float* sparts = reinterpret_cast<float*>(dsm + SM::KV + 8 * D * 4 + DEC_WARPS * 32 * 8 * 4);   // [warp][8][D+2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(dsm + SM::KV + 8 * D * 4 + DEC_WARPS * 32 * 8 * 4 +
                                                 DEC_WARPS * 8 * (D + 2) * 4);

    pdl_trigger();
    const int bg = blockIdx.x, cr = blockIdx.y;
    const int b = bg / a.Hkv, g = bg % a.Hkv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t bar0 = smem_u32(&bars[warp * 2]), bar1 = smem_u32(&bars[warp * 2 + 1]);
    if (lane == 0) {
        mbar_init(bar0, 1);
        mbar_init(bar1, 1);
        fence_barrier_init();
    }
    __syncwarp();
    pdl_wait();
    const int L = a.len_ptr ? (*a.len_ptr + a.len) : a.len;
    const int split = cr * DEC_WARPS + warp;
    const int kbeg = split * a.chunk;
    const int kend = min(L, kbeg + a.chunk);
    const int nslab = kend > kbeg ? (kend - kbeg + 31) / 32 : 0;
    const __nv_bfloat16* kbase = a.k + (int64_t)b * a.kv_sb + (int64_t)g * a.kv_sh;
    const __nv_bfloat16* vbase = a.v + (int64_t)b * a.kv_sb + (int64_t)g * a.kv_sh;
    uint8_t* wkv = kv + warp * 2 * 2 * SM::SLAB;

    auto issue = [&](int i) {   // lane 0 only
        const int k0 = kbeg + 32 * i;
        const int nk = min(32, kend - k0);
        const uint32_t bytes = (uint32_t)(nk * D * 2);
        const uint32_t bar = (i & 1) ? bar1 : bar0;
        uint8_t* buf = wkv + (i & 1) * 2 * SM::SLAB;
        mbar_expect_tx(bar, 2 * bytes);
        bulk_g2s(smem_u32(buf), kbase + (int64_t)k0 * a.kv_ss, bytes, bar);
        bulk_g2s(smem_u32(buf + SM::SLAB), vbase + (int64_t)k0 * a.kv_ss, bytes, bar);
    };
    if (lane == 0) {
        if (nslab > 0) issue(0);
        if (nslab > 1) issue(1);
    }
    for (int i = tid; i < 8 * D; i += 128) {
        const int gg = i / D, d = i % D;
        sq[gg][d] = (gg < G) ? __bfloat162float(a.q[(int64_t)b * a.q_sb + (int64_t)(g * G + gg) * a.q_sh + d]) * a.scale_log2
                             : 0.f;
    }
    __syncthreads();

    float m_run[G], l_run[G], o[G][DPL];
#pragma unroll
    for (int gg = 0; gg < G; gg++) {
        m_run[gg] = -INFINITY;
        l_run[gg] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; j++) o[gg][j] = 0.f;
    }
    bool ok = true;
    for (int i = 0; i < nslab; i++) {
        const int k0 = kbeg + 32 * i;
        const int nk = min(32, kend - k0);
        const bool mine = lane < nk;
        ok = __all_sync(0xffffffffu, mbar_wait((i & 1) ? bar1 : bar0, (i >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL));
        if (!ok) break;
        const __nv_bfloat16* sk = reinterpret_cast<const __nv_bfloat16*>(wkv + (i & 1) * 2 * SM::SLAB);
        const __nv_bfloat16* sv = sk + 32 * D;
        // ---- scores of this lane's key (chunks visited in lane-rotated order)
        float s[G];
#pragma unroll
        for (int gg = 0; gg < G; gg++) s[gg] = 0.f;
        if (mine) {
            const uint4* kr = reinterpret_cast<const uint4*>(sk + lane * D);
#pragma unroll
            for (int cc = 0; cc < D / 8; cc++) {
                const int c = (cc + lane) & (D / 8 - 1);
                const uint4 kw = kr[c];
                const uint32_t w[4] = {kw.x, kw.y, kw.z, kw.w};
                float kf[8];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    kf[2 * j] = bf16_lo(w[j]);
                    kf[2 * j + 1] = bf16_hi(w[j]);
                }
#pragma unroll
                for (int gg = 0; gg < G; gg++) {
                    const float4 q0 = *reinterpret_cast<const float4*>(&sq[gg][c * 8]);
                    const float4 q1 = *reinterpret_cast<const float4*>(&sq[gg][c * 8 + 4]);
                    s[gg] = fmaf(q0.x, kf[0], s[gg]);
                    s[gg] = fmaf(q0.y, kf[1], s[gg]);
                    s[gg] = fmaf(q0.z, kf[2], s[gg]);
                    s[gg] = fmaf(q0.w, kf[3], s[gg]);
                    s[gg] = fmaf(q1.x, kf[4], s[gg]);
                    s[gg] = fmaf(q1.y, kf[5], s[gg]);
                    s[gg] = fmaf(q1.z, kf[6], s[gg]);
                    s[gg] = fmaf(q1.w, kf[7], s[gg]);
                }
            }
        }
        // ---- online softmax per head over the slab
#pragma unroll
        for (int gg = 0; gg < G; gg++) {
            const float sv_ = mine ? s[gg] : -INFINITY;
            float mx = sv_;
#pragma unroll
            for (int of = 16; of > 0; of >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, of));
            const float m_new = fmaxf(m_run[gg], mx);
            const float alpha = ex2(m_run[gg] - m_new);
            const float p = mine ? ex2(sv_ - m_new) : 0.f;
            float sum = p;
#pragma unroll
            for (int of = 16; of > 0; of >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, of);
            l_run[gg] = l_run[gg] * alpha + sum;
            m_run[gg] = m_new;
#pragma unroll
            for (int j = 0; j < DPL; j++) o[gg][j] *= alpha;
            sp[warp][lane][gg] = p;
        }
        __syncwarp();
        // ---- P V for this lane's dims
        for (int j = 0; j < nk; j++) {
            float vf[DPL];
            const __nv_bfloat16* vr = sv + j * D + lane * DPL;
            if (DPL == 2) {
                const uint32_t w = *reinterpret_cast<const uint32_t*>(vr);
                vf[0] = bf16_lo(w);
                vf[1] = bf16_hi(w);
            } else {
                const uint2 w = *reinterpret_cast<const uint2*>(vr);
                vf[0] = bf16_lo(w.x);
                vf[1] = bf16_hi(w.x);
                vf[DPL - 2] = bf16_lo(w.y);
                vf[DPL - 1] = bf16_hi(w.y);
            }
            const float4 p0 = *reinterpret_cast<const float4*>(&sp[warp][j][0]);
            const float4 p1 = *reinterpret_cast<const float4*>(&sp[warp][j][4]);
            const float pj[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
            for (int gg = 0; gg < G; gg++)
#pragma unroll
                for (int q = 0; q < DPL; q++) o[gg][q] = fmaf(pj[gg], vf[q], o[gg][q]);
        }
        __syncwarp();
        if (lane == 0 && i + 2 < nslab) issue(i + 2);   // this buffer has been read by every lane
    }

    // ---- partial of this warp -> shared memory ([warp][head][D + 2])
    float* wp = sparts + warp * 8 * (D + 2);
#pragma unroll
    for (int gg = 0; gg < G; gg++) {
#pragma unroll
        for (int q = 0; q < DPL; q++) wp[gg * (D + 2) + lane * DPL + q] = ok ? o[gg][q] : 0.f;
        if (lane == 0) {
            wp[gg * (D + 2) + D] = ok ? m_run[gg] : -INFINITY;
            wp[gg * (D + 2) + D + 1] = ok ? l_run[gg] : 0.f;
        }
    }
    __syncthreads();
    dec_cluster_sync();
    {
        constexpr int DS = D / DEC_CTAS;              // dims merged by this CTA per head
        const int gg = tid / DS, d = cr * DS + tid % DS;
        if (gg < G) {
            float mv[DEC_SPLITS], lv[DEC_SPLITS], ov[DEC_SPLITS];
#pragma unroll
            for (int r = 0; r < DEC_CTAS; r++) {
#pragma unroll
                for (int w = 0; w < DEC_WARPS; w++) {
                    const float* pw = sparts + (w * 8 + gg) * (D + 2);
                    mv[r * DEC_WARPS + w] = dec_ld_dsmem(smem_u32(pw + D), r);
                    lv[r * DEC_WARPS + w] = dec_ld_dsmem(smem_u32(pw + D + 1), r);
                    ov[r * DEC_WARPS + w] = dec_ld_dsmem(smem_u32(pw + d), r);
                }
            }
            float M = -INFINITY;
#pragma unroll
            for (int i = 0; i < DEC_SPLITS; i++) M = fmaxf(M, mv[i]);
            float l = 0.f, acc = 0.f;
#pragma unroll
            for (int i = 0; i < DEC_SPLITS; i++) {
                const float w = (mv[i] == -INFINITY) ? 0.f : ex2(mv[i] - M);
                l += lv[i] * w;
                acc += ov[i] * w;
            }
            a.o[(int64_t)b * a.o_sb + (int64_t)(g * G + gg) * a.o_sh + d] = __float2bfloat16_rn(l > 0.f ? acc / l : 0.f);
            if (d == 0 && a.lse) a.lse[(int64_t)b * a.Hq + g * G + gg] = l > 0.f ? (M + log2f(l)) * kLn2 : -INFINITY;
        }
    }
    dec_cluster_sync();   // peers may still be reading this CTA's partials
}

// ---------------------------------------------------------------- f32 ------
// One warp per query row, exact f32 two-pass softmax over visible keys.
__global__ void attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                const float* __restrict__ v, float* __restrict__ o, float* __restrict__ lse,
                                int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale, int causal) {
    int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    int lane = threadIdx.x & 31;
    if (row >= (int64_t)B * Hq * Sq) return;
    int i = (int)(row % Sq);
    int64_t bh = row / Sq;
    int h = (int)(bh % Hq), b = (int)(bh / Hq);
    int hk = h / (Hq / Hkv);
    const float* qr = q + row * D;
    const float* kb = k + ((int64_t)b * Hkv + hk) * Sk * D;
    const float* vb = v + ((int64_t)b * Hkv + hk) * Sk * D;
    int jmax = causal ? min(Sk - 1, i + (Sk - Sq)) : Sk - 1;
    float qv[4];
    for (int t = 0; t < 4; t++) qv[t] = (lane + 32 * t < D) ? qr[lane + 32 * t] : 0.f;
    float m = -INFINITY;
    for (int j = 0; j <= jmax; j++) {
        float s = 0.f;
        for (int t = 0; t < 4; t++)
            if (lane + 32 * t < D) s = fmaf(qv[t], kb[(int64_t)j * D + lane + 32 * t], s);
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) s += __shfl_xor_sync(0xffffffffu, s, of);
        m = fmaxf(m, s * scale);
    }
    float l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j <= jmax; j++) {
        float s = 0.f;
        for (int t = 0; t < 4; t++)
            if (lane + 32 * t < D) s = fmaf(qv[t], kb[(int64_t)j * D + lane + 32 * t], s);
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) s += __shfl_xor_sync(0xffffffffu, s, of);
        float p = expf(s * scale - m);
        l += p;
        for (int t = 0; t < 4; t++)
            if (lane + 32 * t < D) acc[t] = fmaf(p, vb[(int64_t)j * D + lane + 32 * t], acc[t]);
    }
    float* orow = o + row * D;
    for (int t = 0; t < 4; t++)
        if (lane + 32 * t < D) orow[lane + 32 * t] = (jmax >= 0) ? acc[t] / l : 0.f;
    if (lse && lane == 0) lse[row] = (jmax >= 0) ? m + logf(l) : -INFINITY;
}

// ------------------------------------------------------------ host side ----
static int tmap_heads(tb_ctx* ctx, CUtensorMap* m, const void* base, int D, int H, int S, int B,
                      int64_t sh, int64_t ss, int64_t sb) {
    // dims (d, h, s, b), box (64, 1, 128, 1); strides in elements -> bytes
    uint64_t dims[4] = {(uint64_t)D, (uint64_t)H, (uint64_t)S, (uint64_t)B};
    uint64_t strides[3] = {(uint64_t)sh * 2, (uint64_t)ss * 2, (uint64_t)sb * 2};
    uint32_t box[4] = {64, 1, 128, 1};
    return make_tmap(ctx, m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, base, dims, strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

int attn_tc_launch(tb_ctx* ctx, const AttnTensors& t, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                   float scale, int causal) {
    CUtensorMap mq, mk, mv;
    int rc = tmap_heads(ctx, &mq, t.q, D, Hq, Sq, B, t.q_sh, t.q_ss, t.q_sb);
    if (!rc) rc = tmap_heads(ctx, &mk, t.k, D, Hkv, t.kv_len_alloc, B, t.kv_sh, t.kv_ss, t.kv_sb);
    if (!rc) rc = tmap_heads(ctx, &mv, t.v, D, Hkv, t.kv_len_alloc, B, t.kv_sh, t.kv_ss, t.kv_sb);
    if (rc) return rc;
    AttnOut out{t.o, t.o_sh, t.o_ss, t.o_sb, t.lse};
    dim3 grid((Sq + 127) / 128, Hq, B);
    const float sl2 = scale * kLog2e;
    if (D == 64) {
        // 512 TMEM columns per CTA: keep one CTA per SM (the padding does that).
        constexpr int smem = AttnCfg<64>::SMEM > 120 * 1024 ? AttnCfg<64>::SMEM : 120 * 1024;
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return launch(ctx, "attn_tc", attn_tc_kernel<64>, grid, dim3(192), smem, mq, mk, mv, out, Hq, Hkv, Sq, Sk, sl2, causal, ctx->d_err);
    } else {
        constexpr int smem = AttnCfg<128>::SMEM;
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return launch(ctx, "attn_tc", attn_tc_kernel<128>, grid, dim3(192), smem, mq, mk, mv, out, Hq, Hkv, Sq, Sk, sl2, causal, ctx->d_err);
    }
    return check_launch(ctx, "attn_tc");
}

// Keys per warp: the context split DEC_SPLITS ways, rounded up to a multiple of 32.
static int decode_chunk(int max_len) {
    int c = (max_len + DEC_SPLITS - 1) / DEC_SPLITS;
    c = (c + 31) / 32 * 32;
    return c < 32 ? 32 : c;
}

int attn_decode_launch(tb_ctx* ctx, DecodeArgs a, int B, int D, int max_len) {
    a.chunk = decode_chunk(max_len);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(B * a.Hkv, DEC_CTAS, 1);
    lc.blockDim = dim3(128, 1, 1);
    lc.dynamicSmemBytes = 0;
    lc.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = DEC_CTAS;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (ctx->pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        lc.numAttrs = 2;
    }
    const int G = a.Hq / a.Hkv;
    cudaError_t e = cudaErrorInvalidValue;
#define TB_DEC_CASE(DD, GG)                                                                                     \
    if (D == DD && G == GG) {                                                                                   \
        lc.dynamicSmemBytes = DecSmem<DD>::BYTES;                                                               \
        cudaFuncSetAttribute(attn_decode_kernel<DD, GG>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecSmem<DD>::BYTES); \
        e = cudaLaunchKernelEx(&lc, attn_decode_kernel<DD, GG>, a, ctx->d_err);                                 \
    }
    TB_DEC_CASE(64, 1) TB_DEC_CASE(64, 2) TB_DEC_CASE(64, 4) TB_DEC_CASE(64, 8)
    TB_DEC_CASE(128, 1) TB_DEC_CASE(128, 2) TB_DEC_CASE(128, 4) TB_DEC_CASE(128, 8)
#undef TB_DEC_CASE
    if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "attn_decode launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace tb

using namespace tb;

extern "C" int tb_attn_fwd(tb_ctx* ctx, int dtype, const void* q, const void* k, const void* v, void* o,
                           float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale, int causal) {
    if (!ctx || !q || !k || !v || !o) return TB_ERR_ARG;
    TB_REQUIRE(ctx, B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && Sq >= 0 && Sk >= 0 && D > 0,
               TB_ERR_SHAPE, "attn: bad shape");
    if (B == 0 || Sq == 0) return TB_OK;
    if (dtype == TB_F32) {
        TB_REQUIRE(ctx, D <= 128, TB_ERR_SHAPE, "attn f32: D <= 128");
        int64_t rows = (int64_t)B * Hq * Sq;
        attn_f32_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, ctx->stream>>>(
            (const float*)q, (const float*)k, (const float*)v, (float*)o, lse, B, Hq, Hkv, Sq, Sk, D, scale, causal);
        return check_launch(ctx, "attn_f32");
    }
    if (dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "attn: dtype %d", dtype);
    TB_REQUIRE(ctx, D == 64 || D == 128, TB_ERR_SHAPE, "attn bf16: D must be 64 or 128");
    TB_REQUIRE(ctx, aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o), TB_ERR_ALIGN, "attn: alignment");
    if (Sk == 0) return set_error(ctx, TB_ERR_SHAPE, "attn bf16: Sk must be > 0");
    AttnTensors t{};
    t.q = q; t.q_sh = (int64_t)Sq * D; t.q_ss = D; t.q_sb = (int64_t)Hq * Sq * D;
    t.k = k; t.v = v; t.kv_sh = (int64_t)Sk * D; t.kv_ss = D; t.kv_sb = (int64_t)Hkv * Sk * D;
    t.kv_len_alloc = Sk;
    t.o = o; t.o_sh = (int64_t)Sq * D; t.o_ss = D; t.o_sb = (int64_t)Hq * Sq * D;
    t.lse = lse;
    const int grp = Hq / Hkv;
    if (Sq == 1 && (grp == 1 || grp == 2 || grp == 4 || grp == 8)) {
        // single-query decode: split-KV CUDA-core kernel
        DecodeArgs a{};
        a.q = (const __nv_bfloat16*)q; a.q_sb = t.q_sb; a.q_sh = t.q_sh;
        a.k = (const __nv_bfloat16*)k; a.v = (const __nv_bfloat16*)v;
        a.kv_sb = t.kv_sb; a.kv_sh = t.kv_sh; a.kv_ss = t.kv_ss;
        a.o = (__nv_bfloat16*)o; a.o_sb = t.o_sb; a.o_sh = t.o_sh;
        a.lse = lse; a.Hq = Hq; a.Hkv = Hkv; a.len = Sk; a.len_ptr = nullptr;
        a.scale_log2 = scale * kLog2e;
        return attn_decode_launch(ctx, a, B, D, Sk);
    }
    return attn_tc_launch(ctx, t, B, Hq, Hkv, Sq, Sk, D, scale, causal);
}

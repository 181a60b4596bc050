// Attention forward on B200.
//
//  * attn_tc_kernel<D>: flash-style forward for bf16 Q/K/V, D in {64, 128}.
//    Persistent, one CTA per SM; each item is two 128-query tiles of one
//    (head, batch) taken in turn (a heavy and a light one when causal).  Warps 0 and 3 stream K and V tiles of 128
//    keys with TMA (two-stage rings; warp 0 also loads Q), warp 1 issues
//    S = Q K^T into one of two TMEM score buffers, warp 2 issues O += P V, so
//    neither MMA stream queues behind the other.  Eight softmax warps, two
//    per TMEM lane quarter, each take 64 of a tile's 128 keys for their rows
//    with their own running max, row sum and TMEM O accumulator (merged once
//    at the end): they read S from TMEM, run the online softmax in the exp2
//    domain, rescale O in TMEM only when the max passes the reference by 2^8,
//    and write P (bf16) into TMEM over the S columns it came from, where the
//    P.V MMA reads it as its A operand.
//    The same online-softmax recurrence as flash_attention2_forward
//    (nn/attention/flash_attn2.rs:98-140), over 128-key tiles instead of one
//    key at a time, plus the causal mask and GQA head mapping.
//  * attn_decode_tc_kernel: decode against a KV cache (few queries, long
//    context) on tcgen05, split over the context, splits merged over DSMEM.
//  * attn_f32_kernel: exact f32 path (fixtures, fp32 configurations).
#include <math.h>

#include "common.cuh"
#include "attention.h"

namespace tb {

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));   // pure: free to schedule
    return y;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// One CTA per SM walks items, an item being a pair of 128-query tiles of one
// (head, image) taken in turn (a heavy and a light one when causal, so items
// carry equal work); its rings and barrier phases run on across tiles and
// items, so each tile's loads and first MMAs overlap the previous tile's
// epilogue, and launch, TMEM allocation and pipeline fill are paid once per SM.  Warp 0 streams Q
// and K tiles and warp 3 V
// tiles (TMA, 2-stage rings), warp 1 issues S = Q K^T (M = 128 queries,
// N = 128 keys) into one of two TMEM buffers and warp 2 issues O += P V
// (N = D), each on its own issuing thread, so S of the next tile never
// queues behind P V of this one.  Softmax warps 4-11: two per row quarter, one query row and half
// of each tile's keys per thread (exp2 domain); each half has its own running
// max, sum and O accumulator, merged at the end.  A
// row's reference max is raised (and its O row and sum rescaled) only when a
// tile's max passes it by 2^8; P = 2^(s - m) <= 256 is otherwise used as is,
// so a tile normally needs no wait on the previous P V.  P is bf16 in TMEM over
// the S columns it came from (the A operand of P V; no shared-memory round trip or
// async-proxy fence), V the MN-major B operand; an S buffer takes the next S once
// the P V that read its P has completed.
template <int D>
struct AttnCfg {
    static constexpr int BM = 128, BN = 128;
    static constexpr int TILE = 128 * D * 2;           // Q, K or V tile bytes
    static constexpr int XCH_BYTES = 2 * 128 * 2 * 4;  // (max, sum) of both key halves per row
    static constexpr int SMEM = TILE /*Q*/ + 2 * TILE /*K*/ + 2 * TILE /*V*/ + XCH_BYTES + 1024 + 256;
    static constexpr int O_COL = 256;                  // TMEM columns: S0 [0,128), S1 [128,256), O_0, O_1 (D each)
    static constexpr float RESCALE_LOG2 = 8.f;
};

constexpr int ATTN_THREADS = 384;   // warps 0/3 TMA, 1 S MMA, 2 P.V MMA, 4-11 softmax

template <int D>
__global__ void __launch_bounds__(ATTN_THREADS, 1)
attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
               const __grid_constant__ CUtensorMap tmV, AttnOut out, int B, int Hq, int Hkv, int Sq, int Sk,
               float scale_log2, int causal, int* err) {
    using C = AttnCfg<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + C::TILE;
    uint8_t* sV = sK + 2 * C::TILE;
    float* xch = reinterpret_cast<float*>(sV + 2 * C::TILE);   // [2 halves][128 rows][2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * C::TILE + C::XCH_BYTES);
    const uint32_t q_full = smem_u32(bars + 0);
    const uint32_t k_full0 = smem_u32(bars + 1), v_full0 = smem_u32(bars + 3);      // [2]
    const uint32_t k_empty0 = smem_u32(bars + 5), v_empty0 = smem_u32(bars + 7);    // [2]
    const uint32_t s_full0 = smem_u32(bars + 9), s_free0 = smem_u32(bars + 11);     // [2]
    const uint32_t p_full0 = smem_u32(bars + 13), p_free0 = smem_u32(bars + 15);    // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
    const uint32_t q_empty = smem_u32(bars + 18);   // the S MMAs of a query tile have read Q
    const uint32_t o_free = smem_u32(bars + 19);    // a query tile's O has been read out of TMEM

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int diag = Sk - Sq;                         // causal: key j visible to query i iff j <= i + diag
    // Persistent: one CTA per SM takes the items it = blockIdx.x, + gridDim.x, ...
    // An item is a pair of query tiles of one (head, image), taken one after the
    // other: causal pairs a heavy tile with a light one (equal work per item),
    // otherwise two neighbours.  Items run pair-fastest, then head, then image,
    // so the items in flight together share their K / V tiles in L2.
    const int nq_all = (Sq + C::BM - 1) / C::BM;
    const int n_pairs = (nq_all + 1) / 2;
    const int n_items = n_pairs * Hq * B;
    struct Item {
        int h, b, hk, nqt, qt0, qt1;
        __device__ int qt(int qi) const { return qi ? qt1 : qt0; }
    };
    auto item_of = [&](int it) {
        Item m;
        const int x = it % n_pairs;
        m.h = (it / n_pairs) % Hq;
        m.b = it / (n_pairs * Hq);
        m.hk = m.h / (Hq / Hkv);
        if (causal) {
            m.qt0 = nq_all - 1 - x;
            m.qt1 = x;
            m.nqt = m.qt1 < m.qt0 ? 2 : 1;
        } else {
            m.qt0 = 2 * x;
            m.qt1 = 2 * x + 1;
            m.nqt = m.qt1 < nq_all ? 2 : 1;
        }
        return m;
    };
    auto tiles_of = [&](int qt) {   // key tiles a query tile needs
        int n = (Sk + C::BN - 1) / C::BN;
        if (causal) {
            const int last_key = qt * C::BM + C::BM - 1 + diag;
            n = min(n, last_key < 0 ? 0 : last_key / C::BN + 1);
        }
        return n;
    };
    constexpr int DB = D / 64;                        // 64-wide d blocks per tile

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(o_free, 8);
        for (int s = 0; s < 2; s++) {
            mbar_init(k_full0 + 8 * s, 1);
            mbar_init(v_full0 + 8 * s, 1);
            mbar_init(k_empty0 + 8 * s, 1);
            mbar_init(v_empty0 + 8 * s, 1);
            mbar_init(s_full0 + 8 * s, 1);
            mbar_init(s_free0 + 8 * s, 1);
            mbar_init(p_full0 + 8 * s, 8);
            mbar_init(p_free0 + 8 * s, 1);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();

    // Every ring and barrier continues across the query tiles and items: g counts key
    // tiles over the whole CTA (stage / buffer g & 1, phase g >> 1) and gq query tiles
    // (Q and O hand-offs, phase gq & 1), so each barrier's phases are waited on in order.
    if (warp == 0 || warp == 3) {
        // ---------------- producers: warp 0 Q and K tiles, warp 3 V tiles
        if (lane == 0) {
            const bool isK = warp == 0;
            const CUtensorMap* tm = isK ? &tmK : &tmV;
            uint8_t* ring = isK ? sK : sV;
            const uint32_t full0 = isK ? k_full0 : v_full0, empty0 = isK ? k_empty0 : v_empty0;
            tma_prefetch_desc(tm);
            if (isK) tma_prefetch_desc(&tmQ);
            int g = 0, gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
                const Item m = item_of(it);
                for (int qi = 0; ok && qi < m.nqt; qi++, gq++) {
                    const int nt = tiles_of(m.qt(qi));
                    if (isK) {
                        // Q of the next query tile once the S MMAs have read the previous one
                        if (gq > 0 && !mbar_wait(q_empty, (gq - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(q_full, C::TILE);
                        for (int d = 0; d < DB; d++)
                            tma_load_4d(smem_u32(sQ + d * 16384), &tmQ, q_full, 64 * d, m.h, m.qt(qi) * C::BM, m.b);
                    }
                    for (int j = 0; j < nt; j++, g++) {
                        const int st = g & 1;
                        if (g >= 2 && !mbar_wait(empty0 + 8 * st, ((g >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(full0 + 8 * st, C::TILE);
                        for (int d = 0; d < DB; d++)
                            tma_load_4d(smem_u32(ring + st * C::TILE + d * 16384), tm, full0 + 8 * st, 64 * d, m.hk,
                                        j * C::BN, m.b);
                    }
                }
            }
            // every load this CTA issued has landed before it can exit (a Q load is
            // counted in gq once issued)
            if (isK && gq > 0) mbar_wait(q_full, (gq - 1) & 1, err, DEV_ERR_TIMEOUT_FULL);
            for (int j = (g > 2 ? g - 2 : 0); j < g; j++)
                mbar_wait(full0 + 8 * (j & 1), (j >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL);
        }
    } else if (warp == 1) {
        // ---------------- S = Q K^T issuer
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_bf16_f32(128, C::BN, false, false);
            const uint64_t q_desc = sdesc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t k_desc = sdesc_sw128(smem_u32(sK), 16, 1024);
            int g = 0, gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
              const Item m = item_of(it);
              for (int qi = 0; ok && qi < m.nqt; qi++, gq++) {
                const int nt = tiles_of(m.qt(qi));
                ok = mbar_wait(q_full, gq & 1, err, DEV_ERR_TIMEOUT_FULL);
                for (int j = 0; ok && j < nt; j++, g++) {
                    const int st = g & 1;
                    if (!mbar_wait(k_full0 + 8 * st, (g >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL) ||
                        (g >= 2 && !mbar_wait(s_free0 + 8 * st, ((g >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC))) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t kd = k_desc + (uint64_t)((st * C::TILE) >> 4);
#pragma unroll
                    for (int kk = 0; kk < D / 16; kk++) {
                        const uint32_t off = ((kk >> 2) * 16384 + (kk & 3) * 32) >> 4;
                        umma_f16_ss(tmem + st * 128, q_desc + off, kd + off, idesc_s, kk != 0);
                    }
                    umma_commit(k_empty0 + 8 * st);
                    umma_commit(s_full0 + 8 * st);
                }
                umma_commit(q_empty);   // Q may be replaced once these S MMAs have completed
              }
            }
        }
    } else if (warp == 2) {
        // ---------------- O += P V issuer
        if (lane == 0) {
            constexpr uint32_t idesc_o = idesc_bf16_f32(128, D, false, true);
            const uint64_t v_desc = sdesc_sw128(smem_u32(sV), 16384, 1024);
            int g = 0, gq = 0;
            bool ok = true;
            for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x) {
              const Item m = item_of(it);
              for (int qi = 0; ok && qi < m.nqt; qi++, gq++) {
                const int nt = tiles_of(m.qt(qi));
                // O of the previous query tile must have been read out before it is overwritten
                if (gq > 0) ok = mbar_wait(o_free, (gq - 1) & 1, err, DEV_ERR_TIMEOUT_MISC);
                for (int j = 0; ok && j < nt; j++, g++) {
                    const int st = g & 1;
                    if (!mbar_wait(p_full0 + 8 * st, (g >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC) ||
                        !mbar_wait(v_full0 + 8 * st, (g >> 1) & 1, err, DEV_ERR_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t vd = v_desc + (uint64_t)((st * C::TILE) >> 4);
                    // keys 0-63 accumulate into O_0 (columns O_COL..), keys 64-127 into O_1 (O_COL + D..);
                    // P of key half hf is bf16 in TMEM (two keys per column) over the first
                    // 32 columns of that half's S: S buffer st, columns 64 hf .. 64 hf + 31
#pragma unroll
                    for (int kk = 0; kk < C::BN / 16; kk++)
                        umma_f16_ts(tmem + C::O_COL + (kk >> 2) * D, tmem + st * 128 + (kk >> 2) * 64 + (kk & 3) * 8,
                                    vd + ((kk * 16 * 128) >> 4), idesc_o, (j | (kk & 3)) != 0);
                    umma_commit(v_empty0 + 8 * st);
                    umma_commit(p_free0 + 8 * st);   // P V of this tile done (O may be rescaled / read)
                    umma_commit(s_free0 + 8 * st);   // S buffer st (holding P) may be overwritten
                }
              }
            }
        }
    } else if (warp >= 4) {
        // ---------------- softmax warps 4..11: thread <-> query row r (TMEM lane quarter
        // warp % 4) and key columns [64 * hf, 64 * hf + 64) of every tile (hf = (warp - 4) / 4).
        // Each half keeps its own reference max, row sum and O accumulator (O_hf); the
        // two are merged once at the end of each query tile, so no exchange is needed per tile.
        const int quarter = warp & 3, hf = (warp - 4) >> 2;
        const int r = quarter * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        const uint32_t o_col = C::O_COL + hf * D;
        int g = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
          const Item m = item_of(it);
          const int h = m.h, b = m.b;
          for (int qi = 0; qi < m.nqt; qi++) {
            const int q0 = m.qt(qi) * C::BM;
            const int n_tiles = tiles_of(m.qt(qi));
            const int qrow = q0 + r;
            const int lim = causal ? min(Sk - 1, qrow + diag) : Sk - 1;   // last visible key
            float m_ref = -INFINITY, l_run = 0.f;
            for (int j = 0; j < n_tiles; j++, g++) {
                const int sb = g & 1;
                ok = mbar_wait(s_full0 + 8 * sb, (g >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC) && ok;
                tc_fence_after();
                float s[64];
                tmem_ld32(t_lane + sb * 128 + hf * 64, s);
                tmem_ld32(t_lane + sb * 128 + hf * 64 + 32, s + 32);
                tmem_wait_ld();
                const int k0 = j * C::BN + hf * 64;
                // 8 independent max chains (latency, not issue, bounds this loop otherwise)
                float mx8[8];
#pragma unroll
                for (int u = 0; u < 8; u++) mx8[u] = -INFINITY;
                // every key of this half visible (and a positive scale): the max of the raw
                // scores, scaled once; the scale is folded into the exponent's FMA below
                const bool raw = k0 + 63 <= lim && scale_log2 > 0.f;
                if (raw) {
#pragma unroll
                    for (int c = 0; c < 64; c++) mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
                } else {
#pragma unroll
                    for (int c = 0; c < 64; c++) {
                        const float v = (k0 + c <= lim) ? s[c] * scale_log2 : -INFINITY;
                        s[c] = v;
                        mx8[c & 7] = fmaxf(mx8[c & 7], v);
                    }
                }
                float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                 fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
                if (raw) mx *= scale_log2;
                float alpha = 1.f;
                if (mx > m_ref + C::RESCALE_LOG2) {   // raise the reference max (m_ref = -inf: first visible tile)
                    alpha = ex2(m_ref - mx);           // -inf -> 0
                    m_ref = mx;
                    l_run *= alpha;
                }
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
                    // O_hf holds P V of this query tile's tiles < j: rescale once P V_{g-1} is done
                    ok = mbar_wait(p_free0 + 8 * ((g - 1) & 1), ((g - 1) >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC) && ok;
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < D; c += 16) {
                        float o[16];
                        tmem_ld16(t_lane + o_col + c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i++) o[i] *= alpha;
                        tmem_st16(t_lane + o_col + c, o);
                    }
                    tmem_wait_st();
                }
                const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
                float rs8[8];
#pragma unroll
                for (int u = 0; u < 8; u++) rs8[u] = 0.f;
                if (raw) {
#pragma unroll
                    for (int c = 0; c < 64; c++) {
                        const float p = ex2(fmaf(s[c], scale_log2, -m_use));
                        s[c] = p;
                        rs8[c & 7] += p;
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 64; c++) {
                        const float p = ex2(s[c] - m_use);   // s = -inf -> 0
                        s[c] = p;
                        rs8[c & 7] += p;
                    }
                }
                l_run += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
                // P row half -> TMEM over this half's own S columns (already read): key
                // 2c in the low and 2c + 1 in the high half of column c, the A operand of P V
                uint32_t pk[32];
#pragma unroll
                for (int c = 0; c < 32; c++) pk[c] = pack_bf16x2(s[2 * c], s[2 * c + 1]);
                tmem_st32u(t_lane + sb * 128 + hf * 64, pk);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(p_full0 + 8 * sb);
            }
            // this query tile's last P V (g - 1) has completed O; exchange (max, sum) of the
            // two halves
            if (n_tiles > 0)
                ok = mbar_wait(p_free0 + 8 * ((g - 1) & 1), ((g - 1) >> 1) & 1, err, DEV_ERR_TIMEOUT_ACC) && ok;
            xch[(hf * 128 + r) * 2] = m_ref;
            xch[(hf * 128 + r) * 2 + 1] = l_run;
            asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
            const float m_o = xch[((hf ^ 1) * 128 + r) * 2], l_o = xch[((hf ^ 1) * 128 + r) * 2 + 1];
            // both halves have read the exchange before the next query tile writes it
            asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
            const float M = fmaxf(m_ref, m_o);
            const float w_a = (hf == 0 ? m_ref : m_o) == -INFINITY ? 0.f : ex2((hf == 0 ? m_ref : m_o) - M);
            const float w_b = (hf == 0 ? m_o : m_ref) == -INFINITY ? 0.f : ex2((hf == 0 ? m_o : m_ref) - M);
            const float l_tot = (hf == 0 ? l_run : l_o) * w_a + (hf == 0 ? l_o : l_run) * w_b;
            ok = __all_sync(0xffffffffu, ok);
            if (ok) {
                tc_fence_after();
                const float inv_l = (l_tot > 0.f) ? 1.0f / l_tot : 0.f;
                const float ca = w_a * inv_l, cb = w_b * inv_l;
                const bool valid = qrow < Sq;
                const int64_t obase = (int64_t)b * out.o_sb + (int64_t)h * out.o_sh + (int64_t)qrow * out.o_ss;
#pragma unroll 1
                for (int c = hf * (D / 2); c < (hf + 1) * (D / 2); c += 32) {
                    float oa[32], ob[32];
                    if (n_tiles > 0) {
                        tmem_ld32(t_lane + C::O_COL + c, oa);
                        tmem_ld32(t_lane + C::O_COL + D + c, ob);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; i++) oa[i] = ob[i] = 0.f;
                    }
                    if (valid) {
                        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(out.o) + obase + c;
#pragma unroll
                        for (int i = 0; i < 32; i += 8) {
                            float o[8];
#pragma unroll
                            for (int e = 0; e < 8; e++) o[e] = oa[i + e] * ca + ob[i + e] * cb;
                            uint4 v;
                            v.x = pack_bf16x2(o[0], o[1]);
                            v.y = pack_bf16x2(o[2], o[3]);
                            v.z = pack_bf16x2(o[4], o[5]);
                            v.w = pack_bf16x2(o[6], o[7]);
                            *reinterpret_cast<uint4*>(dst + i) = v;
                        }
                    }
                }
                if (valid && out.lse && hf == 0) {
                    const float lse = (l_tot > 0.f) ? (M + log2f(l_tot)) * kLn2 : -INFINITY;
                    out.lse[((int64_t)b * Hq + h) * Sq + qrow] = lse;
                }
            }
            // O has been read: the next query tile's first P V may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(o_free);
          }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

// -------------------------------------------------------------- decode -----
// Decode attention against the KV cache on tcgen05 (few queries, long
// context).  One CTA per (batch, kv head, split); the G = Hq / Hkv query heads
// that share the kv head are the queries.  Per 128-key tile j:
//   S^T = K_j Q^T   (M = 128 keys, N = 16 query rows, K = D)   -> TMEM S[j & 1]
//   softmax         (thread t of warps 2-5 <-> key t: one TMEM lane)
//   O  += P_j V_j   (M = 128, N = D, K = 128 keys)              -> TMEM O
// P_j holds 8 query rows x 128 keys (2 KB, double-buffered); its descriptor
// repeats those 8 rows over the MMA's 128 (row-group stride 0), and only O
// rows 0..G-1 are read back.  Roles: warp 0 streams K tiles and warp 6 V
// tiles (TMA, NS-stage rings), warp 1 issues the S MMAs and warp 7 the P V
// MMAs, so S_{j+1} never queues behind P V_j.  The softmax keeps a reference
// max per query that is raised (and O and the row sums rescaled) only when a
// tile's max exceeds it by more than 8 in log2 units; otherwise
// P = 2^(s - m) <= 256 is used as is and no wait on P V_{j-1} is needed.
// Row sums stay per thread until the end.  Splits of one group form a
// cluster and merge (max, sum, o) over DSMEM in a fixed order.
template <int D>
struct DecTcCfg {
    static constexpr int NS = D == 64 ? 3 : 2;          // K / V ring stages
    static constexpr int TILE = 128 * D * 2;            // K or V tile bytes
    static constexpr int P_BYTES = 2048;                // [8 rows][128 keys] bf16: two 64-key atoms
    static constexpr int Q_BYTES = 16 * D * 2;          // [16 rows][D] bf16, rows >= G zero
    static constexpr int PART = 8 * (D + 2) * 4;        // merge partial (max, sum, o) per query
    static constexpr int SMEM = 2 * NS * TILE + 2 * P_BYTES + Q_BYTES + PART + 1024 + 1024;
    static constexpr int O_COL = 32;                    // TMEM: S^T buffers at 0 and 16, O at 32
    static constexpr int TMEM_COLS = (32 + D) <= 128 ? 128 : 256;
    static constexpr float RESCALE_LOG2 = 8.f;          // raise the reference max past this margin
    static constexpr int PREFETCH_TILES = 8;            // cache tiles per split warmed in L2 before the wait
};

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

// Named barrier over the 128 softmax threads.  After a timed-out wait the
// softmax loop still runs to its end (every later wait returns at once), so
// all four warps always reach the same barriers.
__device__ __forceinline__ void softmax_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The same barrier, returning whether `v` holds for any of the 128 threads.
__device__ __forceinline__ bool softmax_bar_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.or.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

template <int D>
__global__ void __launch_bounds__(256, D == 64 ? 2 : 1)
attn_decode_tc_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                      DecodeArgs a, int* err) {
    using C = DecTcCfg<D>;
    constexpr int NS = C::NS, DB = D / 64;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* sK = smem;                        // [NS] K tiles
    uint8_t* sV = sK + NS * C::TILE;           // [NS] V tiles
    uint8_t* sP = sV + NS * C::TILE;           // [2] P tiles
    uint8_t* sQ = sP + 2 * C::P_BYTES;
    float* spart = reinterpret_cast<float*>(sQ + C::Q_BYTES);   // [8][D+2]
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(spart) + C::PART);
    const uint32_t k_full0 = smem_u32(bars), v_full0 = smem_u32(bars + NS);
    const uint32_t k_empty0 = smem_u32(bars + 2 * NS), v_empty0 = smem_u32(bars + 3 * NS);
    const uint32_t s_full0 = smem_u32(bars + 4 * NS), s_free0 = smem_u32(bars + 4 * NS + 2);
    const uint32_t p_full0 = smem_u32(bars + 4 * NS + 4), p_free0 = smem_u32(bars + 4 * NS + 6);
    const uint32_t q_full = smem_u32(bars + 4 * NS + 8);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4 * NS + 9);
    float* sred = reinterpret_cast<float*>(bars + 4 * NS + 10);   // [2 tiles][4 warps][8 queries]
    float* ssum = sred + 64;                                       // [4 warps][8 queries]

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int G = a.Hq / a.Hkv;
    const int bg = blockIdx.x, split = blockIdx.y, nsp = gridDim.y;
    const int b = bg / a.Hkv, g = bg % a.Hkv;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(k_full0 + 8 * s, 1);
            mbar_init(v_full0 + 8 * s, 1);
            mbar_init(k_empty0 + 8 * s, 1);
            mbar_init(v_empty0 + 8 * s, 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(s_full0 + 8 * s, 1);
            mbar_init(s_free0 + 8 * s, 4);
            mbar_init(p_full0 + 8 * s, 4);
            mbar_init(p_free0 + 8 * s, 1);
        }
        mbar_init(q_full, 4);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if ((warp == 0 || warp == 6) && lane == 0) {
        // Before the previous kernel has finished: warm L2 with this split's first
        // cache tiles (K by warp 0, V by warp 6).  The length read here is only a
        // hint (it may still be the previous step's); the tiles are loaded for real
        // after the wait, and rows written meanwhile are seen there, not here.
        const int hint = a.len_ptr ? (*reinterpret_cast<const volatile int*>(a.len_ptr) + a.len) : a.len;
        const int kb = split * a.chunk;
        const int ke = min(hint, kb + a.chunk);
        const int nt = ke > kb ? min((ke - kb + 127) / 128, C::PREFETCH_TILES) : 0;
        const CUtensorMap* tm = warp == 0 ? &tmK : &tmV;
        const int64_t r0 = ((int64_t)b * a.Hkv + g) * a.kv_rows + kb;
        for (int j = 0; j < nt; j++)
            for (int d = 0; d < DB; d++) tma_prefetch_l2_2d(tm, 64 * d, (int)(r0 + 128 * j));
    }
    pdl_wait();
    const int L = a.len_ptr ? (*a.len_ptr + a.len) : a.len;
    const int kbeg = split * a.chunk;
    const int kend = min(L, kbeg + a.chunk);
    const int n_tiles = kend > kbeg ? (kend - kbeg + 127) / 128 : 0;
    const int64_t row0 = ((int64_t)b * a.Hkv + g) * a.kv_rows;   // first cache row of this group

    if (warp == 0 || warp == 6) {
        // ---------------- producers: warp 0 K tiles, warp 6 V tiles
        if (lane == 0 && n_tiles > 0) {
            const bool isK = warp == 0;
            const CUtensorMap* tm = isK ? &tmK : &tmV;
            uint8_t* ring = isK ? sK : sV;
            const uint32_t full0 = isK ? k_full0 : v_full0, empty0 = isK ? k_empty0 : v_empty0;
            tma_prefetch_desc(tm);
            int issued = 0;
            for (int j = 0; j < n_tiles; j++) {
                const int st = j % NS;
                if (j >= NS && !mbar_wait(empty0 + 8 * st, ((j / NS) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) break;
                const int r = (int)(row0 + kbeg + 128 * j);
                mbar_expect_tx(full0 + 8 * st, C::TILE);
                for (int d = 0; d < DB; d++) tma_load_2d(smem_u32(ring + st * C::TILE + d * 16384), tm, full0 + 8 * st, 64 * d, r);
                issued = j + 1;
            }
            // every load this CTA issued has landed before it can exit
            for (int j = (issued > NS ? issued - NS : 0); j < issued; j++)
                mbar_wait(full0 + 8 * (j % NS), (j / NS) & 1, err, DEV_ERR_TIMEOUT_FULL);
        }
    } else if (warp == 1) {
        // ---------------- S^T = K Q^T issuer
        if (lane == 0 && n_tiles > 0) {
            constexpr uint32_t idesc_s = idesc_bf16_f32(128, 16, false, false);
            const uint32_t q_base = smem_u32(sQ);
            bool ok = mbar_wait(q_full, 0, err, DEV_ERR_TIMEOUT_MISC);
            for (int j = 0; ok && j < n_tiles; j++) {
                const int st = j % NS, sb = j & 1;
                if (!mbar_wait(k_full0 + 8 * st, (j / NS) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
                if (j >= 2 && !mbar_wait(s_free0 + 8 * sb, ((j - 2) >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                tc_fence_after();
                const uint32_t k_base = smem_u32(sK + st * C::TILE);
#pragma unroll
                for (int kk = 0; kk < D / 16; kk++) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    const uint32_t qoff = (kk >> 2) * 2048 + (kk & 3) * 32;
                    umma_f16_ss(tmem + sb * 16, sdesc_sw128(k_base + off, 16, 1024), sdesc_sw128(q_base + qoff, 16, 1024),
                                idesc_s, kk != 0);
                }
                umma_commit(k_empty0 + 8 * st);
                umma_commit(s_full0 + 8 * sb);
            }
        }
    } else if (warp == 7) {
        // ---------------- O += P V issuer
        if (lane == 0 && n_tiles > 0) {
            constexpr uint32_t idesc_o = idesc_bf16_f32(128, D, false, true);
            const uint32_t p_base = smem_u32(sP);
            for (int j = 0; j < n_tiles; j++) {
                const int st = j % NS, pb = j & 1;
                if (!mbar_wait(p_full0 + 8 * pb, (j >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                if (!mbar_wait(v_full0 + 8 * st, (j / NS) & 1, err, DEV_ERR_TIMEOUT_FULL)) break;
                tc_fence_after();
                const uint32_t v_base = smem_u32(sV + st * C::TILE);
#pragma unroll
                for (int kk = 0; kk < 8; kk++) {
                    // 8 P rows repeated over the 128 MMA rows: row-group stride 0
                    const uint64_t ad = sdesc_sw128(p_base + pb * C::P_BYTES + (kk >> 2) * 1024 + (kk & 3) * 32, 16, 0);
                    const uint64_t bd = sdesc_sw128(v_base + kk * 16 * 128, 16384, 1024);
                    umma_f16_ss(tmem + C::O_COL, ad, bd, idesc_o, (j | kk) != 0);
                }
                umma_commit(v_empty0 + 8 * st);
                umma_commit(p_free0 + 8 * pb);
            }
        }
    } else {
        // ---------------- softmax warps 2..5: thread <-> key row of the tile
        const int sw = warp - 2;                          // 0..3
        const int quarter = warp & 3;                     // TMEM lane quarter of this warp
        const int kr = quarter * 32 + lane;               // key row within the tile
        const int tid = threadIdx.x - 64;                 // 0..127
        const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
        // Q -> smem [16 rows][D], 128-B swizzle, rows >= G zero; both P tiles -> zero
        for (int i = tid; i < 16 * (D / 8); i += 128) {
            const int r = i / (D / 8), c = i % (D / 8);   // row, 16-byte chunk
            uint4 v = make_uint4(0, 0, 0, 0);
            if (r < G) v = *reinterpret_cast<const uint4*>(a.q + (int64_t)b * a.q_sb + (int64_t)(g * G + r) * a.q_sh + c * 8);
            const int cc = c & 7, atom = c >> 3;
            *reinterpret_cast<uint4*>(sQ + atom * 2048 + r * 128 + ((cc ^ (r & 7)) << 4)) = v;
        }
        for (int i = tid; i < 2 * C::P_BYTES / 16; i += 128) reinterpret_cast<uint4*>(sP)[i] = make_uint4(0, 0, 0, 0);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);

        float m_ref[8], lsum[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
            m_ref[q] = -INFINITY;
            lsum[q] = 0.f;
        }
        bool ok = true;
        for (int j = 0; j < n_tiles; j++) {
            const int sb = j & 1;
            ok = mbar_wait(s_full0 + 8 * sb, (j >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC) && ok;
            tc_fence_after();
            float s[8];
            tmem_ld8(t_lane + sb * 16, s);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(s_free0 + 8 * sb);   // S buffer sb may be overwritten
            const bool valid = kbeg + 128 * j + kr < kend;
            bool over = false;   // a score of this thread passes its query's reference max by the margin
#pragma unroll
            for (int q = 0; q < 8; q++) {
                s[q] = (valid && q < G) ? s[q] * a.scale_log2 : -INFINITY;
                over |= s[q] > m_ref[q] + C::RESCALE_LOG2;
            }
            // Common case: no score passes the margin, one barrier and no max
            // reduction.  Otherwise (always on the first tile) reduce the tile max
            // per query and raise the reference max where it passes the margin.
            float alpha[8];
            bool any = false;
#pragma unroll
            for (int q = 0; q < 8; q++) alpha[q] = 1.f;
            if (softmax_bar_or(over)) {
                float* red = sred + sb * 32;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    if (q < G) {
                        float m = s[q];
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                        if (lane == 0) red[sw * 8 + q] = m;
                    }
                }
                softmax_bar();
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    if (q < G) {
                        const float tm = fmaxf(fmaxf(red[q], red[8 + q]), fmaxf(red[16 + q], red[24 + q]));
                        if (tm > m_ref[q] + C::RESCALE_LOG2) {
                            alpha[q] = ex2(m_ref[q] - tm);   // m_ref = -inf -> 0
                            m_ref[q] = tm;
                            lsum[q] *= alpha[q];
                            any = true;
                        }
                    }
                }
            }
            if (any && j > 0 && quarter == 0) {
                // O holds P V of tiles < j: rescale rows 0..G-1 once P V_{j-1} is done
                ok = mbar_wait(p_free0 + 8 * ((j - 1) & 1), ((j - 1) >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC) && ok;
                tc_fence_after();
                float my_alpha = 1.f;
#pragma unroll
                for (int q = 0; q < 8; q++)
                    if (lane == q) my_alpha = alpha[q];
#pragma unroll 1
                for (int c = 0; c < D; c += 16) {
                    float o[16];
                    tmem_ld16(t_lane + C::O_COL + c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i++) o[i] *= my_alpha;
                    tmem_st16(t_lane + C::O_COL + c, o);
                }
                tmem_wait_st();
            }
            float p[8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                p[q] = q < G ? ex2(s[q] - m_ref[q]) : 0.f;   // s = -inf -> 0
                lsum[q] += p[q];
            }
            // P_j (bf16) into the swizzled K-major tile: row q, key column kr; the
            // buffer is free once P V_{j-2} is done
            const int pb = j & 1;
            if (j >= 2) ok = mbar_wait(p_free0 + 8 * pb, ((j - 2) >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC) && ok;
            {
                uint8_t* pt = sP + pb * C::P_BYTES + (kr >> 6) * 1024;
                const int kc = kr & 63;
#pragma unroll
                for (int q = 0; q < 8; q++)
                    if (q < G)
                        *reinterpret_cast<__nv_bfloat16*>(pt + q * 128 + (((kc >> 3) ^ q) << 4) + (kc & 7) * 2) =
                            __float2bfloat16_rn(p[q]);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(p_full0 + 8 * pb);
        }
        // row sums over the 128 key threads
#pragma unroll
        for (int q = 0; q < 8; q++) {
            if (q < G) {
                float v = lsum[q];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane == 0) ssum[sw * 8 + q] = v;
            }
        }
        softmax_bar();
        // partial (max, sum, unnormalised o) of this split: warp 4 (TMEM quarter 0), lanes < G
        if (quarter == 0) {
            if (n_tiles > 0)
                ok = mbar_wait(p_free0 + 8 * ((n_tiles - 1) & 1), ((n_tiles - 1) >> 1) & 1, err, DEV_ERR_TIMEOUT_ACC) && ok;
            ok = __all_sync(0xffffffffu, ok);
            tc_fence_after();
            float my_m = -INFINITY, my_l = 0.f;
#pragma unroll
            for (int q = 0; q < 8; q++)
                if (lane == q && q < G) {
                    my_m = m_ref[q];
                    my_l = ssum[q] + ssum[8 + q] + ssum[16 + q] + ssum[24 + q];
                }
#pragma unroll 1
            for (int c = 0; c < D; c += 16) {
                float o[16];
                if (n_tiles > 0 && ok) {
                    tmem_ld16(t_lane + C::O_COL + c, o);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i++) o[i] = 0.f;
                }
                if (lane < G)
#pragma unroll
                    for (int i = 0; i < 16; i++) spart[lane * (D + 2) + c + i] = o[i];
            }
            if (lane < G) {
                spart[lane * (D + 2) + D] = (n_tiles > 0 && ok) ? my_m : -INFINITY;
                spart[lane * (D + 2) + D + 1] = (n_tiles > 0 && ok) ? my_l : 0.f;
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
    // ---- merge the splits (cluster over blockIdx.y) and write O / LSE
    if (nsp > 1) dec_cluster_sync();
    const int DS = D / nsp;                               // dims merged by this CTA per query
    for (int i = threadIdx.x; i < G * DS; i += 256) {
        const int q = i / DS, d = split * DS + i % DS;
        float M = -INFINITY, l = 0.f, o = 0.f;
        if (nsp == 1) {
            M = spart[q * (D + 2) + D];
            l = spart[q * (D + 2) + D + 1];
            o = spart[q * (D + 2) + d];
        } else {
            float mv[8], lv[8], ov[8];
            const uint32_t base = smem_u32(spart + q * (D + 2));
#pragma unroll
            for (int r = 0; r < 8; r++) {
                if (r < nsp) {
                    mv[r] = dec_ld_dsmem(base + D * 4, r);
                    lv[r] = dec_ld_dsmem(base + (D + 1) * 4, r);
                    ov[r] = dec_ld_dsmem(base + d * 4, r);
                }
            }
#pragma unroll
            for (int r = 0; r < 8; r++)
                if (r < nsp) M = fmaxf(M, mv[r]);
#pragma unroll
            for (int r = 0; r < 8; r++) {
                if (r < nsp) {
                    const float w = (mv[r] == -INFINITY) ? 0.f : ex2(mv[r] - M);
                    l += lv[r] * w;
                    o += ov[r] * w;
                }
            }
        }
        a.o[(int64_t)b * a.o_sb + (int64_t)(g * G + q) * a.o_sh + d] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
        if (d == 0 && a.lse) a.lse[(int64_t)b * a.Hq + g * G + q] = l > 0.f ? (M + log2f(l)) * kLn2 : -INFINITY;
    }
    if (nsp > 1) dec_cluster_sync();   // peers may still be reading this CTA's partial
}

// ---------------------------------------------------------------- f32 ------
// One warp per query row, f32 throughout.  Keys go 32 at a time, lane j
// computing the full dot product of key j (q staged in shared memory); an
// online softmax (running max, rescaled sum and output) merges the chunks,
// and the output dims are spread over the lanes for P V.  Tensors are
// addressed through (head, position, batch) strides in elements (d is
// contiguous); lse is [B, Hq, Sq].
struct F32Strides {
    int64_t q_sh, q_ss, q_sb, kv_sh, kv_ss, kv_sb, o_sh, o_ss, o_sb;
};

__global__ void __launch_bounds__(256)
attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                float* __restrict__ o, float* __restrict__ lse, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                float scale, int causal, F32Strides st) {
    __shared__ float sq[8][128];
    const int w = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * 8 + w;
    const bool live = row < (int64_t)B * Hq * Sq;
    int i = 0, h = 0, b = 0;
    if (live) {
        i = (int)(row % Sq);
        const int64_t bh = row / Sq;
        h = (int)(bh % Hq);
        b = (int)(bh / Hq);
        const float* qr = q + (int64_t)b * st.q_sb + (int64_t)h * st.q_sh + (int64_t)i * st.q_ss;
        for (int d = lane; d < D; d += 32) sq[w][d] = qr[d];
    }
    __syncwarp();
    if (!live) return;
    const int hk = h / (Hq / Hkv);
    const float* kb = k + (int64_t)b * st.kv_sb + (int64_t)hk * st.kv_sh;
    const float* vb = v + (int64_t)b * st.kv_sb + (int64_t)hk * st.kv_sh;
    const bool vec = (D & 3) == 0 && (reinterpret_cast<uintptr_t>(kb) & 15) == 0 && (st.kv_ss & 3) == 0;
    const int jmax = causal ? min(Sk - 1, i + (Sk - Sq)) : Sk - 1;
    float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 <= jmax; j0 += 32) {
        const int j = j0 + lane;
        float sc = -INFINITY;
        if (j <= jmax) {
            const float* kr = kb + (int64_t)j * st.kv_ss;
            float dot = 0.f;
            if (vec) {   // 16-byte rows
#pragma unroll 8
                for (int d = 0; d < D; d += 4) {
                    const float4 kv = *reinterpret_cast<const float4*>(kr + d);
                    dot = fmaf(sq[w][d], kv.x, dot);
                    dot = fmaf(sq[w][d + 1], kv.y, dot);
                    dot = fmaf(sq[w][d + 2], kv.z, dot);
                    dot = fmaf(sq[w][d + 3], kv.w, dot);
                }
            } else {
                for (int d = 0; d < D; d++) dot = fmaf(sq[w][d], kr[d], dot);
            }
            sc = dot * scale;
        }
        float cm = sc;
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, of));
        const float m_new = fmaxf(m, cm);          // finite: key j0 <= jmax is visible
        const float alpha = expf(m - m_new);       // m = -inf on the first chunk -> 0
        const float p = (j <= jmax) ? expf(sc - m_new) : 0.f;
        float ps = p;
#pragma unroll
        for (int of = 16; of > 0; of >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, of);
        l = l * alpha + ps;
#pragma unroll
        for (int t = 0; t < 4; t++) acc[t] *= alpha;
        const int nj = min(32, jmax - j0 + 1);
        for (int jb = 0; jb < nj; jb += 8) {
            // 8 value rows in flight at once
            float vv[8][4];
#pragma unroll
            for (int u = 0; u < 8; u++)
#pragma unroll
                for (int t = 0; t < 4; t++)
                    vv[u][t] = (jb + u < nj && lane + 32 * t < D) ? vb[(int64_t)(j0 + jb + u) * st.kv_ss + lane + 32 * t] : 0.f;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float pj = __shfl_sync(0xffffffffu, p, (jb + u) & 31);
#pragma unroll
                for (int t = 0; t < 4; t++) acc[t] = fmaf(pj, vv[u][t], acc[t]);
            }
        }
        m = m_new;
    }
    float* orow = o + (int64_t)b * st.o_sb + (int64_t)h * st.o_sh + (int64_t)i * st.o_ss;
    for (int t = 0; t < 4; t++)
        if (lane + 32 * t < D) orow[lane + 32 * t] = (jmax >= 0) ? acc[t] / l : 0.f;
    if (lse && lane == 0) lse[row] = (jmax >= 0) ? m + logf(l) : -INFINITY;
}

// ------------------------------------------------------------ host side ----
int attn_f32_launch(tb_ctx* ctx, const AttnTensors& t, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale,
                    int causal) {
    if (D > 128) return set_error(ctx, TB_ERR_SHAPE, "attn f32: D <= 128");
    const int64_t rows = (int64_t)B * Hq * Sq;
    if (rows == 0) return TB_OK;
    const F32Strides st{t.q_sh, t.q_ss, t.q_sb, t.kv_sh, t.kv_ss, t.kv_sb, t.o_sh, t.o_ss, t.o_sb};
    attn_f32_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, ctx->stream>>>(
        (const float*)t.q, (const float*)t.k, (const float*)t.v, (float*)t.o, t.lse, B, Hq, Hkv, Sq, Sk, D, scale,
        causal, st);
    return check_launch(ctx, "attn_f32");
}

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
    // persistent: one CTA per SM (512 TMEM columns each) over the items, an item
    // being two query tiles of one (head, image), a heavy and a light one when causal
    const int64_t items = (int64_t)(((Sq + 127) / 128 + 1) / 2) * Hq * B;
    if (items >= (1ll << 31)) return set_error(ctx, TB_ERR_SHAPE, "attention: too many query tiles");
    dim3 grid((unsigned)std::min<int64_t>(items, ctx->num_sms));
    const float sl2 = scale * kLog2e;
    if (D == 64) {
        // 512 TMEM columns per CTA: keep one CTA per SM (the padding does that).
        constexpr int smem = AttnCfg<64>::SMEM > 120 * 1024 ? AttnCfg<64>::SMEM : 120 * 1024;
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return launch(ctx, "attn_tc", attn_tc_kernel<64>, grid, dim3(ATTN_THREADS), smem, mq, mk, mv, out, B, Hq, Hkv, Sq, Sk, sl2, causal, ctx->d_err);
    } else {
        constexpr int smem = AttnCfg<128>::SMEM;
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return launch(ctx, "attn_tc", attn_tc_kernel<128>, grid, dim3(ATTN_THREADS), smem, mq, mk, mv, out, B, Hq, Hkv, Sq, Sk, sl2, causal, ctx->d_err);
    }
    return check_launch(ctx, "attn_tc");
}

// Splits per (batch, kv head) group: the largest of 8, 4, 2, 1 that keeps the
// grid within the resident CTA slots and leaves every split >= 1 key tile.
int attn_decode_launch(tb_ctx* ctx, DecodeArgs a, int B, int D, int max_len) {
    const int G = a.Hq / a.Hkv;
    if (a.Hq % a.Hkv != 0 || G < 1 || G > 8) return set_error(ctx, TB_ERR_SHAPE, "attn_decode: group size %d", G);
    if (a.kv_ss != D || a.kv_sh != (int64_t)a.kv_rows * D || a.kv_sb != (int64_t)a.Hkv * a.kv_rows * D)
        return set_error(ctx, TB_ERR_SHAPE, "attn_decode: K/V must be contiguous [B][Hkv][rows][D]");
    const int groups = B * a.Hkv;
    const int tiles = (max_len + 127) / 128;
    const int slots = (D == 64 ? 2 : 1) * ctx->num_sms;
    int nsp = 8;
    while (nsp > 1 && (groups * nsp > slots || nsp > tiles)) nsp >>= 1;
    a.chunk = ((tiles + nsp - 1) / nsp) * 128;
    CUtensorMap mk, mv;
    const uint64_t rows = (uint64_t)B * a.Hkv * a.kv_rows;
    int rc = make_tmap_2d(ctx, &mk, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.k, rows, D, D, 64, 128);
    if (!rc) rc = make_tmap_2d(ctx, &mv, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.v, rows, D, D, 64, 128);
    if (rc) return rc;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(groups, nsp, 1);
    lc.blockDim = dim3(256, 1, 1);
    lc.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = nsp;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (ctx->pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        lc.numAttrs = 2;
    }
    cudaError_t e;
    if (D == 64) {
        lc.dynamicSmemBytes = DecTcCfg<64>::SMEM;
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_decode_tc_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecTcCfg<64>::SMEM));
        e = cudaLaunchKernelEx(&lc, attn_decode_tc_kernel<64>, mk, mv, a, ctx->d_err);
    } else {
        lc.dynamicSmemBytes = DecTcCfg<128>::SMEM;
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(attn_decode_tc_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, DecTcCfg<128>::SMEM));
        e = cudaLaunchKernelEx(&lc, attn_decode_tc_kernel<128>, mk, mv, a, ctx->d_err);
    }
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
        AttnTensors t{};
        t.q = q;
        t.q_ss = D, t.q_sh = (int64_t)Sq * D, t.q_sb = (int64_t)Hq * Sq * D;
        t.k = k;
        t.v = v;
        t.kv_ss = D, t.kv_sh = (int64_t)Sk * D, t.kv_sb = (int64_t)Hkv * Sk * D;
        t.o = o;
        t.o_ss = D, t.o_sh = (int64_t)Sq * D, t.o_sb = (int64_t)Hq * Sq * D;
        t.lse = lse;
        return attn_f32_launch(ctx, t, B, Hq, Hkv, Sq, Sk, D, scale, causal);
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
    if (Sq == 1 && grp <= 8) {
        // single-query decode: split-KV CUDA-core kernel
        DecodeArgs a{};
        a.q = (const __nv_bfloat16*)q; a.q_sb = t.q_sb; a.q_sh = t.q_sh;
        a.k = (const __nv_bfloat16*)k; a.v = (const __nv_bfloat16*)v;
        a.kv_sb = t.kv_sb; a.kv_sh = t.kv_sh; a.kv_ss = t.kv_ss;
        a.o = (__nv_bfloat16*)o; a.o_sb = t.o_sb; a.o_sh = t.o_sh;
        a.lse = lse; a.Hq = Hq; a.Hkv = Hkv; a.len = Sk; a.len_ptr = nullptr; a.kv_rows = Sk;
        a.scale_log2 = scale * kLog2e;
        return attn_decode_launch(ctx, a, B, D, Sk);
    }
    return attn_tc_launch(ctx, t, B, Hq, Hkv, Sq, Sk, D, scale, causal);
}

// Persistent decode chain: consecutive decode GEMVs of a layer in one launch.
//
// A decode step streams every weight matrix once for a handful of tokens, so
// each GEMV is HBM-bound, and a separate launch per GEMV spends several
// microseconds per matrix outside its weight stream (the split-K reduction,
// the epilogue, the next launch's start-up).  This kernel runs a chain of
// GEMVs -- e.g. the output projection (+ residual), gate/up (fused RMSNorm,
// SwiGLU), down (+ residual) and the next layer's QKV projection (fused
// RMSNorm, RoPE, KV-cache write) -- as phases of one persistent grid, one CTA
// per SM.  Weights never depend on the previous phase, so each CTA's weight
// producer streams straight on into the next phase's tiles while the current
// phase is still being reduced.
//
// Work split: the grid is NC thread-block clusters of CS CTAs.  A phase's
// 256-row weight tiles are dealt to the clusters in turn (phases with fewer
// tiles than clusters start where the previous phase stopped, so they fall on
// different clusters); the CS CTAs of a cluster split each tile's K range.
// The split-K partial sums are reduced inside the cluster over distributed
// shared memory: rank r owns the row pairs [r*P, (r+1)*P), P = 128 / CS, and
// every rank pushes its partials of those pairs into the owner's receive
// buffer with st.async (completing on the owner's mbarrier); owners add the
// CS slots in rank order (deterministic) and run the epilogue.  Receive
// buffers are double-buffered; an owner frees a buffer by arriving on each
// sender's mbarrier.
//
// Handoffs between phases (a phase's x, or its residual, written by an
// earlier phase) use flagged words: such an output is also stored as 8-byte
// words (f32 value, 32-bit flag) with single stores, and the readers poll the
// words until the flag of this launch and phase appears (epoch * 8 + phase +
// 1; the epoch advances at the end of every launch) -- one L2 round trip, no
// fence on the writer's side.  Outputs are also written in their normal
// layout for the kernels after this one, except where a later phase of the
// same launch rewrites the same buffer.
//
// All CTAs are resident (grid = the clusters that fit, one CTA per SM by
// shared memory), and every wait is bounded: a wait that gives up sets the
// device error word and every other wait then returns at once.  The last CTA
// to finish advances the epoch for the next launch.
//
// Roles (16 warps): warp 0 streams weights (and the norm gains) with TMA,
// warps 1 and 2 issue the MMAs of one 128-row half each into double-buffered
// TMEM accumulators, warp 3 loads activation tiles that come from before the
// launch (TMA) and owns the TMEM allocation, warps 4-11 run the exchange and
// the epilogue and warps 12-15 build the activation tiles that come from an
// earlier phase (from flagged words) and apply the fused RMSNorm (bf16(x * w),
// with each token's sum of squares).
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "decode_chain.h"
#include "gemv_epi.cuh"

namespace tb {

namespace {

struct PhaseInfo {
    Epi ep;
    int Nw, K, nk, tiles, ncols;
    int base;               // the first cluster of the phase's tiles
    int norm;
    int x_src;              // -1: x is from before the launch (TMA); else the phase that wrote it
    int r_src;              // -1: the residual is from before the launch; else the phase that wrote it
    int std_out;            // store y in its normal layout (no later phase rewrites it)
    int ll_out;             // store y as flagged words too (a later phase reads it)
    uint64_t* ll;           // this phase's flagged output [Mtok][ncols]
    const uint64_t* x_ll;   // x as flagged words [Mtok][K] (x_src >= 0)
    const uint64_t* r_ll;   // the residual as flagged words [Mtok][ncols] (r_src >= 0)
};

struct ChainPhaseParams {
    CUtensorMap tmW;   // [Nw][K] bf16, box 64 x 256, 128-B swizzle
    CUtensorMap tmX;   // [Mtok][K] bf16, box 64 x NT, 128-B swizzle (x_src < 0)
    PhaseInfo info;
};

struct ChainParams {
    ChainPhaseParams ph[kChainMaxPhases];
    int nph, Mtok, cs;
    int* err;
    unsigned* sync;   // [0] CTAs finished, [1] epoch
};

constexpr int kConvWarps = 4;
constexpr int kEpiThreads = 256;
constexpr unsigned long long kDrainNs = 10000000ull;   // copies still in flight when a CTA gives up

__device__ __forceinline__ void named_bar(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Barrier over n threads that also ANDs a predicate across them.
__device__ __forceinline__ bool named_bar_and(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_rank(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}

// ------------------------------------------------------------ flagged words
__device__ __forceinline__ uint64_t ll_word(float v, uint32_t flag) {
    return ((uint64_t)flag << 32) | (uint64_t)__float_as_uint(v);
}
__device__ __forceinline__ bool ll_ok(uint64_t w, uint32_t flag) { return (uint32_t)(w >> 32) == flag; }
__device__ __forceinline__ float ll_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ void st_ll(uint64_t* p, uint64_t w) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_ll(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void ld_ll2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Bounded re-polling: a reader loads a batch of flagged words at once and,
// only if a flag is missing, loads the whole batch again until every flag is
// there.  again() returns false (the error word set) once the wait exceeds
// the limit, or at once if another CTA has flagged an error.
struct Repoll {
    unsigned long long t0 = 0;
    uint32_t spins = 0;
    __device__ __forceinline__ bool again(int* err) {
        if (t0 == 0) t0 = globaltimer();
        if ((++spins & 15u) == 0) {
            if (*(volatile int*)err != 0) return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                atomicOr(err, DEV_ERR_TIMEOUT_MISC);
                return false;
            }
        }
        return true;
    }
};

// Wait for a phase without looking at the error word: used only to let this
// CTA's own copies and MMAs finish before it exits.
__device__ void drain_wait(uint32_t bar, uint32_t parity, unsigned long long deadline) {
    while (!mbar_try_wait(bar, parity) && globaltimer() < deadline) {
    }
}

// ------------------------------------------------------------------- items
// A cluster's tiles in a phase: base-rotated cluster index g', tiles g',
// g' + NC, ...; every rank takes the K blocks [r*nk/CS, (r+1)*nk/CS) of each.
struct Cursor {
    int t;
};
struct Item {
    int t, kb0, kb1;
};

__device__ __forceinline__ Cursor item_begin(const PhaseInfo& ph, int cluster, int nc) {
    return Cursor{(cluster - ph.base % nc + nc) % nc};
}

__device__ __forceinline__ bool item_next(const PhaseInfo& ph, Cursor& cur, Item& it, int nc, int rank, int cs) {
    if (cur.t >= ph.tiles) return false;
    it.t = cur.t;
    it.kb0 = rank * ph.nk / cs;
    it.kb1 = (rank + 1) * ph.nk / cs;
    cur.t += nc;
    return true;
}

// ------------------------------------------------------------- epilogue I/O
// Epilogue of (token m, pair): RoPE phases store q / k / v in their normal
// layout only; others store y normally (std_out) and / or as flagged words.
__device__ __forceinline__ void chain_finish(const PhaseInfo& ph, const EpiPair& k, int tile, int m, float a0,
                                             float a1, float r0, float r1, uint32_t flag, int* err) {
    const Epi& ep = ph.ep;
    if (ep.rope_tab) {
        epi_finish_bf16(ep, k, tile, m, a0, a1, r0, r1, err);
        return;
    }
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(ep.out) + (int64_t)m * ep.ldo;
    uint64_t* ll = ph.ll + (int64_t)m * ph.ncols;
    if (ep.swiglu) {
        if (!k.in1) return;
        const __nv_bfloat16 o = __float2bfloat16_rn(silu_f(a0 * k.sc0) * (a1 * k.sc1));
        const int c = tile * 128 + k.p;
        if (ph.std_out) out[c] = o;
        if (ph.ll_out) st_ll(ll + c, ll_word(__bfloat162float(o), flag));
        return;
    }
    float o0 = a0 * k.sc0 + k.bi0, o1 = a1 * k.sc1 + k.bi1;
    if (ep.resid) {
        o0 += r0;
        o1 += r1;
    }
    const __nv_bfloat16 b0 = __float2bfloat16_rn(o0), b1 = __float2bfloat16_rn(o1);
    if (k.in0) {
        if (ph.std_out) out[k.n0] = b0;
        if (ph.ll_out) st_ll(ll + k.n0, ll_word(__bfloat162float(b0), flag));
    }
    if (k.in1) {
        if (ph.std_out) out[k.n1] = b1;
        if (ph.ll_out) st_ll(ll + k.n1, ll_word(__bfloat162float(b1), flag));
    }
}

template <int NT, int STAGES, int RBUF>
struct ChainCfg {
    static constexpr int W_BYTES = 256 * 128;   // [256 rows][64 bf16], 128-B swizzle
    static constexpr int X_BYTES = NT * 128;    // [NT][64 bf16], one swizzle atom wide
    static constexpr int G_BYTES = 128;         // the block's 64 norm gains
    // a message from one rank to one owner: [NT tokens][P pairs][2] partials, then
    // the sender's NT sums of squares; an owner's buffer holds CS of them (<= 8)
    static constexpr int RECV_F = NT * 256 + 8 * NT;
    static constexpr int OFF_X = STAGES * W_BYTES;
    static constexpr int OFF_G = OFF_X + STAGES * X_BYTES;
    static constexpr int OFF_RECV = OFF_G + STAGES * G_BYTES;
    static constexpr int OFF_BAR = OFF_RECV + RBUF * RECV_F * 4;
    static constexpr int N_BARS = 3 * STAGES + 9 + 2 * RBUF;
    static constexpr int OFF_SLOT = OFF_BAR + N_BARS * 8;
    static constexpr int OFF_SS = OFF_SLOT + 16;            // [2][NT] item sums of squares
    static constexpr int OFF_RINV = OFF_SS + 2 * NT * 4;     // [NT] 1/rms of the owned slice
    static constexpr int OFF_INFO = (OFF_RINV + NT * 4 + 15) & ~15;
    static constexpr int SMEM = OFF_INFO + kChainMaxPhases * (int)sizeof(PhaseInfo) + 1024;
    static constexpr int THREADS = 512;
    static constexpr int TMEM_COLS = 4 * NT < 32 ? 32 : 4 * NT;   // [2 buffers][2 halves][NT]
    static_assert(SMEM <= 227 * 1024, "shared memory");
    static_assert(SMEM > 114 * 1024, "one CTA per SM: the grid's CTAs wait on one another");
};

template <int NT, int STAGES, int RBUF>
__global__ void __launch_bounds__(512, 1) decode_chain_kernel(const __grid_constant__ ChainParams P) {
    using C = ChainCfg<NT, STAGES, RBUF>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    uint8_t* sW = smem;
    uint8_t* sX = smem + C::OFF_X;
    uint8_t* sG = smem + C::OFF_G;
    float* recv = reinterpret_cast<float*>(smem + C::OFF_RECV);   // [RBUF][RECV_F]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    const uint32_t full0 = smem_u32(bars);                  // [STAGES] weights (+ TMA activations) landed
    const uint32_t empty0 = smem_u32(bars + STAGES);        // [STAGES] MMAs done with the stage
    const uint32_t xrdy0 = smem_u32(bars + 2 * STAGES);     // [STAGES] activation tile ready for the MMA
    const uint32_t accf0 = smem_u32(bars + 3 * STAGES);     // [2] accumulator complete
    const uint32_t acce0 = accf0 + 16;                      // [2] accumulator read out
    const uint32_t ssf0 = accf0 + 32;                       // [2] item sums of squares written
    const uint32_t sse0 = accf0 + 48;                       // [2] item sums of squares read
    const uint32_t mmad = accf0 + 64;                       // every MMA of the CTA done
    const uint32_t rfull0 = accf0 + 72;                     // [RBUF] peers' messages landed
    const uint32_t rfree0 = rfull0 + 8 * RBUF;              // [RBUF] every owner has read my last messages
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::OFF_SLOT);
    float* s_ss = reinterpret_cast<float*>(smem + C::OFF_SS);
    float* s_rinv = reinterpret_cast<float*>(smem + C::OFF_RINV);
    PhaseInfo* info = reinterpret_cast<PhaseInfo*>(smem + C::OFF_INFO);

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int nph = P.nph, Mtok = P.Mtok, CS = P.cs;
    const int rank = (int)(blockIdx.x % (unsigned)CS), cluster = (int)(blockIdx.x / (unsigned)CS);
    const int NC = (int)(gridDim.x / (unsigned)CS);
    const int PP = 128 / CS;                                 // row pairs an owner reduces
    const int MSG_F = NT * PP * 2 + NT;                      // floats per message
    int* err = P.err;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(full0 + 8 * s, 2);   // the weight and the activation producer
            mbar_init(empty0 + 8 * s, 2);  // the two MMA issuers
            mbar_init(xrdy0 + 8 * s, kConvWarps);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(accf0 + 8 * b, 2);
            mbar_init(acce0 + 8 * b, kEpiThreads / 32);
            mbar_init(ssf0 + 8 * b, kConvWarps);
            mbar_init(sse0 + 8 * b, kEpiThreads / 32);
        }
        mbar_init(mmad, 2);
        for (int b = 0; b < RBUF; b++) {
            mbar_init(rfull0 + 8 * b, 1);
            mbar_init(rfree0 + 8 * b, CS > 1 ? CS - 1 : 1);
        }
        fence_barrier_init();
        // arm every receive buffer for its first messages
        if (CS > 1)
            for (int b = 0; b < RBUF; b++) mbar_expect_tx(rfull0 + 8 * b, (uint32_t)((CS - 1) * MSG_F * 4));
    }
    if (threadIdx.x < nph) info[threadIdx.x] = P.ph[threadIdx.x].info;
    if (warp == 3) tmem_alloc(smem_u32(tmem_slot), C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (CS > 1) cluster_sync_all();   // the peers' barriers exist before any message
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---------------- weight producer: runs ahead across phases
        if (lane == 0) {
            for (int p = 0; p < nph; p++) tma_prefetch_desc(&P.ph[p].tmW);
            int blk = 0;
            bool ok = true;
            for (int p = 0; p < nph && ok; p++) {
                const PhaseInfo& ph = info[p];
                const __nv_bfloat16* gains = reinterpret_cast<const __nv_bfloat16*>(ph.ep.norm_w);
                Cursor cur = item_begin(ph, cluster, NC);
                Item it;
                while (ok && item_next(ph, cur, it, NC, rank, CS)) {
                    for (int kb = it.kb0; kb < it.kb1; kb++, blk++) {
                        const int s = blk % STAGES;
                        if (blk >= STAGES && !mbar_wait(empty0 + 8 * s, ((blk / STAGES) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(full0 + 8 * s, C::W_BYTES + (ph.norm ? C::G_BYTES : 0));
                        tma_load_2d(smem_u32(sW + s * C::W_BYTES), &P.ph[p].tmW, full0 + 8 * s, kb * 64, it.t * 256);
                        if (ph.norm) bulk_load(smem_u32(sG + s * C::G_BYTES), gains + kb * 64, C::G_BYTES, full0 + 8 * s);
                    }
                }
            }
            // the last stages' copies have landed before the CTA may exit
            const unsigned long long dl = globaltimer() + kDrainNs;
            for (int i = blk > STAGES ? blk - STAGES : 0; i < blk; i++)
                drain_wait(full0 + 8 * (i % STAGES), (i / STAGES) & 1, dl);
        }
    } else if (warp == 1 || warp == 2) {
        // ---------------- MMA issuers: rows [0, 128) / [128, 256) of each tile
        if (lane == 0) {
            const int h = warp - 1;
            constexpr uint32_t idesc = idesc_bf16_f32(128, NT, false, false);
            int blk = 0, j = 0;
            bool ok = true;
            for (int p = 0; p < nph && ok; p++) {
                const PhaseInfo& ph = info[p];
                Cursor cur = item_begin(ph, cluster, NC);
                Item it;
                while (ok && item_next(ph, cur, it, NC, rank, CS)) {
                    const int buf = j & 1;
                    if (j >= 2 && !mbar_wait(acce0 + 8 * buf, ((j >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)((buf * 2 + h) * NT);
                    for (int kb = it.kb0; kb < it.kb1; kb++, blk++) {
                        const int s = blk % STAGES;
                        const uint32_t par = (blk / STAGES) & 1;
                        if (!mbar_wait(full0 + 8 * s, par, err, DEV_ERR_TIMEOUT_FULL) ||
                            !mbar_wait(xrdy0 + 8 * s, par, err, DEV_ERR_TIMEOUT_MISC)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t wb = smem_u32(sW + s * C::W_BYTES) + h * 128 * 128;
                        const uint32_t xb = smem_u32(sX + s * C::X_BYTES);
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_f16_ss(d, sdesc_sw128(wb + kk * 32, 16, 1024), sdesc_sw128(xb + kk * 32, 16, 1024), idesc,
                                        (kb > it.kb0 || kk > 0) ? 1u : 0u);
                        umma_commit(empty0 + 8 * s);
                    }
                    if (!ok) break;
                    umma_commit(accf0 + 8 * buf);
                    j++;
                }
            }
            umma_commit(mmad);
        }
    } else if (warp == 3) {
        // ---------------- activations from before the launch (TMA); for an
        // earlier phase's output the converters build the tile, and this warp
        // only keeps the stage barrier's arrival count
        if (lane == 0) {
            for (int p = 0; p < nph; p++)
                if (info[p].x_src < 0) tma_prefetch_desc(&P.ph[p].tmX);
            pdl_wait();   // the previous kernel's output
            int blk = 0;
            bool ok = true;
            for (int p = 0; p < nph && ok; p++) {
                const PhaseInfo& ph = info[p];
                Cursor cur = item_begin(ph, cluster, NC);
                Item it;
                while (ok && item_next(ph, cur, it, NC, rank, CS)) {
                    for (int kb = it.kb0; kb < it.kb1; kb++, blk++) {
                        const int s = blk % STAGES;
                        if (blk >= STAGES && !mbar_wait(empty0 + 8 * s, ((blk / STAGES) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        if (ph.x_src < 0) {
                            mbar_expect_tx(full0 + 8 * s, C::X_BYTES);
                            tma_load_2d(smem_u32(sX + s * C::X_BYTES), &P.ph[p].tmX, full0 + 8 * s, kb * 64, 0);
                        } else {
                            mbar_arrive(full0 + 8 * s);
                        }
                    }
                }
            }
        }
    } else if (warp < 12) {
        // ---------------- exchange and epilogue warps.  Per tile: read the
        // accumulator out; push each owner its row pairs (st.async into the
        // owner's receive buffer); as owner, add the CS messages in rank order and
        // run the epilogue on the owned pairs; free the buffer on every sender.
        pdl_wait();
        const uint32_t ep_base = *(volatile const unsigned*)(P.sync + 1) * 8u + 1u;   // flag of phase 0
        const int e = threadIdx.x - 128;
        const int q = warp & 3, part = (warp - 4) >> 2, l = q * 32 + lane;
        constexpr int TP = NT / 2;
        const uint32_t t_row = tmem + ((uint32_t)(q * 32) << 16);
        const int owner = l / PP, pl = l % PP;
        bool ok = true;
        int j = 0;
        for (int p = 0; p < nph && ok; p++) {
            const PhaseInfo& ph = info[p];
            const Epi& ep = ph.ep;
            const uint32_t flag = ep_base + (uint32_t)p;
            const uint32_t rflag = ep_base + (uint32_t)(ph.r_src < 0 ? 0 : ph.r_src);
            const int posb = epi_posb(ep);
            Cursor cur = item_begin(ph, cluster, NC);
            Item it;
            while (item_next(ph, cur, it, NC, rank, CS)) {
                const int buf = j & 1, rb = j % RBUF, ru = j / RBUF;
                ok = named_bar_and(1, kEpiThreads, mbar_wait(accf0 + 8 * buf, (j >> 1) & 1, err, DEV_ERR_TIMEOUT_ACC));
                if (!ok) break;
                tc_fence_after();
                float acc[2][TP];
#pragma unroll
                for (int h = 0; h < 2; h++) {
                    const uint32_t ta = t_row + (uint32_t)((buf * 2 + h) * NT + part * TP);
                    if (TP == 8) tmem_ld8(ta, acc[h]);
                    else if (TP == 16) tmem_ld16(ta, acc[h]);
                    else tmem_ld32(ta, acc[h]);
                }
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acce0 + 8 * buf);
                // this item's per-token sums of squares (fused norm)
                const bool sok = mbar_wait(ssf0 + 8 * buf, (j >> 1) & 1, err, DEV_ERR_TIMEOUT_MISC);
                float ss_tok[TP];
                float ss_e = 0.f;
#pragma unroll
                for (int t = 0; t < TP; t++) ss_tok[t] = ph.norm ? s_ss[buf * NT + part * TP + t] : 0.f;
                if (e < NT) ss_e = ph.norm ? s_ss[buf * NT + e] : 0.f;
                __syncwarp();
                if (lane == 0) mbar_arrive(sse0 + 8 * buf);
                j++;
                if (CS == 1) {
                    ok = named_bar_and(1, kEpiThreads, sok);
                    if (!ok) break;
                    // one CTA holds the tile's whole K range: finish from registers
                    EpiPair kp = epi_pair(ep, it.t, ph.Nw, l, posb);
                    kp.cs = epi_rope_cs(ep, kp);
#pragma unroll
                    for (int t = 0; t < TP; t++) {
                        const int m = part * TP + t;
                        if (m < Mtok) {
                            const float rs = ph.norm ? rsqrtf(ss_tok[t] * (1.0f / (float)ph.K) + ep.norm_eps) : 1.f;
                            float r0 = 0.f, r1 = 0.f;
                            if (ep.resid && ph.r_src >= 0) {
                                const uint64_t* rr = ph.r_ll + (int64_t)m * ph.ncols;
                                uint64_t w0 = (uint64_t)rflag << 32, w1 = w0;
                                Repoll rp;
                                do {
                                    if (kp.in0) w0 = ld_ll(rr + kp.n0);
                                    if (kp.in1) w1 = ld_ll(rr + kp.n1);
                                } while (!(ll_ok(w0, rflag) && ll_ok(w1, rflag)) && rp.again(err));
                                r0 = ll_val(w0);
                                r1 = ll_val(w1);
                            } else {
                                epi_resid_bf16(ep, kp, m, Mtok, r0, r1);
                            }
                            chain_finish(ph, kp, it.t, m, acc[0][t] * rs, acc[1][t] * rs, r0, r1, flag, err);
                        }
                    }
                    continue;
                }
                // ---- send: my partials of owner o's pairs into o's buffer rb, slot [rank]
                bool fok = true;
                if (ru >= 1) fok = mbar_wait(rfree0 + 8 * rb, (ru - 1) & 1, err, DEV_ERR_TIMEOUT_MISC);
                ok = named_bar_and(1, kEpiThreads, sok && fok);
                if (!ok) break;
                {
                    float* slot = recv + rb * C::RECV_F + rank * MSG_F;
                    const uint32_t loc = smem_u32(slot + (part * TP * PP + pl) * 2);
                    if (owner == rank) {
#pragma unroll
                        for (int t = 0; t < TP; t++)
                            *reinterpret_cast<float2*>(slot + ((part * TP + t) * PP + pl) * 2) = make_float2(acc[0][t], acc[1][t]);
                    } else {
                        const uint32_t rdst = map_rank(loc, owner), rbar = map_rank(rfull0 + 8 * rb, owner);
#pragma unroll
                        for (int t = 0; t < TP; t++)
                            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(
                                             rdst + t * PP * 8),
                                         "f"(acc[0][t]), "f"(acc[1][t]), "r"(rbar)
                                         : "memory");
                    }
                }
                // sums of squares (zeros without the norm): thread e < NT sends
                // token e's to every owner
                if (e < NT) {
                    for (int o = 0; o < CS; o++) {
                        float* slot = recv + rb * C::RECV_F + rank * MSG_F + NT * PP * 2 + e;
                        if (o == rank) {
                            *slot = ss_e;
                        } else {
                            const uint32_t rdst = map_rank(smem_u32(slot), o), rbar = map_rank(rfull0 + 8 * rb, o);
                            asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(rdst),
                                         "f"(ss_e), "r"(rbar)
                                         : "memory");
                        }
                    }
                }
                // ---- receive: owned pairs [rank*PP, (rank+1)*PP) of tile it.t.  The
                // residuals and RoPE angles of my items are loaded while the
                // messages are in flight.
                const int nitems = PP * Mtok;
                float pr0[4], pr1[4];
                float2 pcs[4];
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    pr0[u] = pr1[u] = 0.f;
                    pcs[u] = make_float2(1.f, 0.f);
                    const int idx = e + u * kEpiThreads;
                    if (idx < nitems) {
                        const int m = idx / PP;
                        const EpiPair kp = epi_pair(ep, it.t, ph.Nw, rank * PP + idx % PP, posb);
                        pcs[u] = epi_rope_cs(ep, kp);
                        if (ep.resid && ph.r_src >= 0) {
                            const uint64_t* rr = ph.r_ll + (int64_t)m * ph.ncols;
                            uint64_t w0 = (uint64_t)rflag << 32, w1 = w0;
                            Repoll rp;
                            do {
                                if (kp.in0) w0 = ld_ll(rr + kp.n0);
                                if (kp.in1) w1 = ld_ll(rr + kp.n1);
                            } while (!(ll_ok(w0, rflag) && ll_ok(w1, rflag)) && rp.again(err));
                            pr0[u] = ll_val(w0);
                            pr1[u] = ll_val(w1);
                        } else {
                            epi_resid_bf16(ep, kp, m, Mtok, pr0[u], pr1[u]);
                        }
                    }
                }
                const bool got = mbar_wait(rfull0 + 8 * rb, ru & 1, err, DEV_ERR_TIMEOUT_MISC);
                ok = named_bar_and(1, kEpiThreads, got);   // (also: my own slot's stores are visible)
                if (!ok) break;
                const float* rbuf = recv + rb * C::RECV_F;
                if (ph.norm) {
                    if (e < NT) {
                        float v[8];
#pragma unroll
                        for (int r = 0; r < 8; r++) v[r] = r < CS ? rbuf[r * MSG_F + NT * PP * 2 + e] : 0.f;
                        float s = 0.f;
#pragma unroll
                        for (int r = 0; r < 8; r++) s += v[r];
                        s_rinv[e] = rsqrtf(s * (1.0f / (float)ph.K) + ep.norm_eps);
                    }
                    named_bar(1, kEpiThreads);
                }
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int idx = e + u * kEpiThreads;
                    if (idx < nitems) {
                        const int m = idx / PP, pi = idx % PP;
                        float2 v[8];
#pragma unroll
                        for (int r = 0; r < 8; r++)
                            v[r] = r < CS ? *reinterpret_cast<const float2*>(rbuf + r * MSG_F + (m * PP + pi) * 2) : make_float2(0.f, 0.f);
                        float a0 = 0.f, a1 = 0.f;
#pragma unroll
                        for (int r = 0; r < 8; r++) {
                            a0 += v[r].x;
                            a1 += v[r].y;
                        }
                        EpiPair kp = epi_pair(ep, it.t, ph.Nw, rank * PP + pi, posb);
                        kp.cs = pcs[u];
                        const float rs = ph.norm ? s_rinv[m] : 1.f;
                        chain_finish(ph, kp, it.t, m, a0 * rs, a1 * rs, pr0[u], pr1[u], flag, err);
                    }
                }
                // ---- every read of buffer rb is done: re-arm it, then free it on
                // every sender (their next message into it may follow).  The arrive
                // is relaxed: it orders nothing but this CTA's reads of the buffer,
                // which have returned their values (a release would first wait for
                // this thread's global stores to drain).
                named_bar(1, kEpiThreads);
                if (e == 0) {
                    mbar_expect_tx(rfull0 + 8 * rb, (uint32_t)((CS - 1) * MSG_F * 4));
                    for (int o = 0; o < CS; o++)
                        if (o != rank)
                            asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                                             map_rank(rfree0 + 8 * rb, o))
                                         : "memory");
                }
                __syncwarp();
            }
        }
    } else {
        // ---------------- converter warps: activation tiles of earlier phases
        // (from flagged words) and the fused RMSNorm
        pdl_wait();
        const uint32_t ep_base = *(volatile const unsigned*)(P.sync + 1) * 8u + 1u;
        constexpr int CT = 32 * kConvWarps;
        constexpr int RC = 8;                                  // 16-B chunks per token row of a block
        constexpr int XI = (NT * RC + CT - 1) / CT;
        const int ct = threadIdx.x - 384;
        int blk = 0, j = 0;
        bool ok = true;
        for (int p = 0; p < nph && ok; p++) {
            const PhaseInfo& ph = info[p];
            const uint32_t xflag = ep_base + (uint32_t)(ph.x_src < 0 ? 0 : ph.x_src);
            Cursor cur = item_begin(ph, cluster, NC);
            Item it;
            while (ok && item_next(ph, cur, it, NC, rank, CS)) {
                float ssv[XI];
#pragma unroll
                for (int u = 0; u < XI; u++) ssv[u] = 0.f;
                for (int kb = it.kb0; kb < it.kb1; kb++, blk++) {
                    const int s = blk % STAGES;
                    ok = __all_sync(0xffffffffu, mbar_wait(full0 + 8 * s, (blk / STAGES) & 1, err, DEV_ERR_TIMEOUT_FULL));
                    if (!ok) break;
                    if (ph.norm || ph.x_src >= 0) {
                        // x tile [NT rows][64 k] bf16, 128-B swizzle: chunk cc of row m holds
                        // k = 8 * (cc ^ (m & 7)) .. + 7.  From flagged words (rows past the
                        // tokens are zero), or the TMA tile rewritten in place; with the norm
                        // fused, bf16(x[m,k] * w[k]) and the sum of squares of x.
                        uint8_t* xt = sX + s * C::X_BYTES;
                        const uint8_t* gt = sG + s * C::G_BYTES;
#pragma unroll
                        for (int u = 0; u < XI; u++) {
                            const int itc = ct + u * CT;
                            if (itc < NT * RC) {
                                const int m = itc / RC, cc = itc % RC;
                                const int kk = 8 * (cc ^ (m & 7));
                                uint4* px = reinterpret_cast<uint4*>(xt + m * 128 + cc * 16);
                                float xv[8];
                                if (ph.x_src >= 0) {
                                    if (m < Mtok) {
                                        const uint64_t* src = ph.x_ll + (int64_t)m * ph.K + kb * 64 + kk;
                                        uint64_t w[8];
                                        bool good;
                                        Repoll rp;
                                        do {
                                            good = true;
#pragma unroll
                                            for (int i = 0; i < 8; i += 2) {
                                                ld_ll2(src + i, w[i], w[i + 1]);
                                                good = good && ll_ok(w[i], xflag) && ll_ok(w[i + 1], xflag);
                                            }
                                        } while (!good && rp.again(err));
#pragma unroll
                                        for (int i = 0; i < 8; i++) xv[i] = ll_val(w[i]);
                                    } else {
#pragma unroll
                                        for (int i = 0; i < 8; i++) xv[i] = 0.f;
                                    }
                                } else {
                                    const uint4 raw = *px;
                                    const uint32_t xa[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
                                    for (int i = 0; i < 4; i++) {
                                        xv[2 * i] = bf16_lo(xa[i]);
                                        xv[2 * i + 1] = bf16_hi(xa[i]);
                                    }
                                }
                                uint32_t o[4];
                                if (ph.norm) {
                                    const uint4 gv = *reinterpret_cast<const uint4*>(gt + 2 * kk);
                                    const uint32_t ga[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
                                    for (int i = 0; i < 4; i++) {
                                        ssv[u] += xv[2 * i] * xv[2 * i] + xv[2 * i + 1] * xv[2 * i + 1];
                                        o[i] = pack_bf16x2(xv[2 * i] * bf16_lo(ga[i]), xv[2 * i + 1] * bf16_hi(ga[i]));
                                    }
                                } else {
#pragma unroll
                                    for (int i = 0; i < 4; i++) o[i] = pack_bf16x2(xv[2 * i], xv[2 * i + 1]);
                                }
                                *px = make_uint4(o[0], o[1], o[2], o[3]);
                            }
                        }
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(xrdy0 + 8 * s);
                }
                if (!ok) break;
                const int buf = j & 1;
                if (j >= 2) {
                    ok = __all_sync(0xffffffffu, mbar_wait(sse0 + 8 * buf, ((j >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC));
                    if (!ok) break;
                }
                if (ph.norm) {
                    // the RC chunks of a token row sit in RC consecutive lanes
#pragma unroll
                    for (int u = 0; u < XI; u++) {
                        float v = ssv[u];
                        v += __shfl_xor_sync(0xffffffffu, v, 1);
                        v += __shfl_xor_sync(0xffffffffu, v, 2);
                        v += __shfl_xor_sync(0xffffffffu, v, 4);
                        const int itc = ct + u * CT;
                        if ((lane & (RC - 1)) == 0 && itc < NT * RC) s_ss[buf * NT + itc / RC] = v;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(ssf0 + 8 * buf);
                j++;
            }
        }
    }

    // ---------------- exit: every peer is done with this CTA's shared memory
    // (messages, frees) before it leaves; free TMEM once every MMA is done; the
    // last CTA to leave advances the epoch for the next launch
    __syncwarp();
    pdl_wait();
    tc_fence_before();
    __syncthreads();
    if (CS > 1) cluster_sync_all();
    if (warp == 3) {
        drain_wait(mmad, 0, globaltimer() + kDrainNs);
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(P.sync, 1u);
        if (prev == gridDim.x - 1) {
            atomicAdd(P.sync + 1, 1u);
            atomicExch(P.sync, 0u);
        }
    }
}

// Chain layout decisions made on the host from the steps' pointers.
struct PhasePlan {
    int x_src, r_src, std_out, ll_out, ncols;
};

int plan_phases(tb_ctx* ctx, const ChainStep* steps, int n, PhasePlan* pl) {
    for (int i = 0; i < n; i++) {
        const ChainStep& s = steps[i];
        PhasePlan& q = pl[i];
        q.ncols = s.ep.swiglu ? s.Nw / 2 : s.Nw;
        q.x_src = q.r_src = -1;
        q.ll_out = 0;
        for (int j = i - 1; j >= 0 && (q.x_src < 0 || q.r_src < 0); j--) {
            const ChainStep& o = steps[j];
            if (q.x_src < 0 && o.ep.out == s.x) {
                if (s.K != pl[j].ncols || s.x_ld != o.ep.ldo)
                    return set_error(ctx, TB_ERR_UNSUPPORTED, "decode chain: step %d reads step %d's output with another shape", i, j);
                q.x_src = j;
            }
            if (q.r_src < 0 && s.ep.resid && o.ep.out == s.ep.resid) {
                if (q.ncols != pl[j].ncols || s.ep.ldr != o.ep.ldo)
                    return set_error(ctx, TB_ERR_UNSUPPORTED, "decode chain: step %d's residual is step %d's output with another shape", i, j);
                q.r_src = j;
            }
        }
        q.std_out = 1;
        for (int k = i + 1; k < n; k++)
            if (steps[k].ep.out == s.ep.out) {
                if (pl[i].ncols != (steps[k].ep.swiglu ? steps[k].Nw / 2 : steps[k].Nw) || steps[k].ep.ldo != s.ep.ldo)
                    return set_error(ctx, TB_ERR_UNSUPPORTED, "decode chain: steps %d and %d write one buffer with different shapes", i, k);
                q.std_out = 0;   // a later phase rewrites every value
            }
    }
    for (int i = 0; i < n; i++) {
        if (pl[i].x_src >= 0) pl[pl[i].x_src].ll_out = 1;
        if (pl[i].r_src >= 0) pl[pl[i].r_src].ll_out = 1;
    }
    for (int i = 0; i < n; i++)
        if (pl[i].ll_out && steps[i].ep.rope_tab)
            return set_error(ctx, TB_ERR_UNSUPPORTED, "decode chain: a RoPE phase's output cannot feed a later phase");
    return TB_OK;
}

template <int NT, int STAGES, int RBUF>
int launch_chain(tb_ctx* ctx, const ChainStep* steps, int n, int Mtok, const ChainScratch& scr) {
    using C = ChainCfg<NT, STAGES, RBUF>;
    PhasePlan pl[kChainMaxPhases];
    int rc = plan_phases(ctx, steps, n, pl);
    if (rc) return rc;
    // cluster size: the largest of 8, 4, 2, 1 that leaves every rank a K block
    int cs = 8;
    for (int i = 0; i < n; i++)
        while (cs > 1 && steps[i].K / 64 < cs) cs >>= 1;
    auto kern = decode_chain_kernel<NT, STAGES, RBUF>;
    TB_CUDA_TRY(ctx, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    // clusters that can be resident at once (all of the grid waits on one another)
    static std::mutex mu;
    static int nc_cache[4] = {0, 0, 0, 0};
    const int ci = cs == 8 ? 3 : cs == 4 ? 2 : cs == 2 ? 1 : 0;
    int nc;
    {
        std::lock_guard<std::mutex> g(mu);
        if (!nc_cache[ci]) {
            cudaLaunchConfig_t q = {};
            q.gridDim = dim3((unsigned)cs, 1, 1);
            q.blockDim = dim3(C::THREADS, 1, 1);
            q.dynamicSmemBytes = C::SMEM;
            cudaLaunchAttribute qa[1];
            qa[0].id = cudaLaunchAttributeClusterDimension;
            qa[0].val.clusterDim.x = (unsigned)cs;
            qa[0].val.clusterDim.y = 1;
            qa[0].val.clusterDim.z = 1;
            q.attrs = qa;
            q.numAttrs = 1;
            int m = 0;
            if (cudaOccupancyMaxActiveClusters(&m, kern, &q) != cudaSuccess || m < 1) {
                cudaGetLastError();
                return set_error(ctx, TB_ERR_CUDA, "decode chain: no resident cluster of %d CTAs", cs);
            }
            nc_cache[ci] = m * cs > ctx->num_sms ? ctx->num_sms / cs : m;
        }
        nc = nc_cache[ci];
    }
    ChainParams prm;
    memset(&prm, 0, sizeof(prm));
    size_t ll_used = 0;
    int base = 0;
    for (int i = 0; i < n; i++) {
        const ChainStep& s = steps[i];
        rc = make_tmap_2d(ctx, &prm.ph[i].tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.w, s.Nw, s.K, s.K, 64, 256);
        if (rc) return rc;
        if (pl[i].x_src < 0) {
            rc = make_tmap_2d(ctx, &prm.ph[i].tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, s.x, Mtok, s.K, s.x_ld, 64, NT);
            if (rc) return rc;
        }
        PhaseInfo& ph = prm.ph[i].info;
        ph.ep = s.ep;
        ph.Nw = s.Nw;
        ph.K = s.K;
        ph.nk = s.K / 64;
        ph.tiles = s.Nw / 256;
        ph.ncols = pl[i].ncols;
        ph.base = base;
        base = (base + (ph.tiles < nc ? ph.tiles : 0)) % nc;   // a phase that fills the grid keeps the rotation
        ph.norm = s.ep.norm_w != nullptr;
        ph.x_src = pl[i].x_src;
        ph.r_src = pl[i].r_src;
        ph.std_out = pl[i].std_out;
        ph.ll_out = pl[i].ll_out;
        if (ph.ll_out) {
            ph.ll = scr.ll + ll_used;
            ll_used += (size_t)Mtok * ph.ncols;
        }
    }
    if (ll_used > scr.ll_words) return set_error(ctx, TB_ERR_ARG, "decode chain: scratch too small");
    for (int i = 0; i < n; i++) {
        PhaseInfo& ph = prm.ph[i].info;
        if (ph.x_src >= 0) ph.x_ll = prm.ph[ph.x_src].info.ll;
        if (ph.r_src >= 0) ph.r_ll = prm.ph[ph.r_src].info.ll;
    }
    prm.nph = n;
    prm.Mtok = Mtok;
    prm.cs = cs;
    prm.err = ctx->d_err;
    prm.sync = scr.sync;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((unsigned)(nc * cs), 1, 1);
    lc.blockDim = dim3(C::THREADS, 1, 1);
    lc.dynamicSmemBytes = C::SMEM;
    lc.stream = ctx->stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (ctx->pdl) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        lc.numAttrs = 2;
    }
    TB_CUDA_TRY(ctx, cudaLaunchKernelEx(&lc, kern, prm));
    return TB_OK;
}

}  // namespace

size_t chain_ll_words(int Mtok, int max_cols) { return (size_t)kChainMaxPhases * Mtok * max_cols; }

bool chain_step_ok(const ChainStep& s, int Mtok) {
    const Epi& e = s.ep;
    return Mtok >= 1 && Mtok <= 64 && s.Nw > 0 && s.Nw % 256 == 0 && s.Nw / 256 <= kChainMaxTiles && s.K > 0 &&
           s.K % 64 == 0 && s.x_ld >= s.K && s.x_ld % 8 == 0 && aligned16(s.x) && aligned16(s.w) && !e.out_f32 &&
           !e.scale && !e.bias && (!e.norm_w || aligned16(e.norm_w)) && (!e.rope_tab || e.rope_s_new == 1) &&
           (!e.resid || !e.swiglu);
}

int chain_launch(tb_ctx* ctx, const ChainStep* steps, int n, int Mtok, const ChainScratch& scr) {
    if (n < 1 || n > kChainMaxPhases || !scr.sync || !scr.ll)
        return set_error(ctx, TB_ERR_ARG, "decode chain: bad phase count or scratch");
    for (int i = 0; i < n; i++)
        if (!chain_step_ok(steps[i], Mtok)) return set_error(ctx, TB_ERR_UNSUPPORTED, "decode chain: step %d shape", i);
    if (Mtok <= 16) return launch_chain<16, 5, 2>(ctx, steps, n, Mtok, scr);
    if (Mtok <= 32) return launch_chain<32, 4, 2>(ctx, steps, n, Mtok, scr);
    return launch_chain<64, 3, 1>(ctx, steps, n, Mtok, scr);
}

}  // namespace tb

using namespace tb;

extern "C" int tb_linear_chain_fwd(tb_ctx* ctx, const tb_linear_step* steps, int n_steps, int64_t M) {
    if (!ctx || !steps) return TB_ERR_ARG;
    TB_REQUIRE(ctx, n_steps >= 1 && n_steps <= TB_LINEAR_CHAIN_MAX && n_steps <= kChainMaxPhases, TB_ERR_ARG,
               "linear chain: 1 to %d steps", TB_LINEAR_CHAIN_MAX);
    TB_REQUIRE(ctx, M >= 1 && M <= 64, TB_ERR_SHAPE, "linear chain: 1 <= M <= 64 tokens");
    ChainStep cs[kChainMaxPhases];
    int max_cols = 0;
    for (int i = 0; i < n_steps; i++) {
        const tb_linear_step& t = steps[i];
        TB_REQUIRE(ctx, t.x && t.w && t.y, TB_ERR_ARG, "linear chain: step %d: null x, w or y", i);
        TB_REQUIRE(ctx, t.N > 0 && t.N % 256 == 0 && t.N <= 256 * kChainMaxTiles && t.K > 0 && t.K % 64 == 0 &&
                            t.K < (1 << 30),
                   TB_ERR_SHAPE, "linear chain: step %d: N %% 256 (<= %d) and K %% 64 must be 0", i, 256 * kChainMaxTiles);
        const bool swiglu = (t.flags & TB_EPI_SWIGLU) != 0, resid = (t.flags & TB_EPI_RESIDUAL) != 0;
        TB_REQUIRE(ctx, !(t.flags & ~(TB_EPI_SWIGLU | TB_EPI_RESIDUAL)), TB_ERR_UNSUPPORTED,
                   "linear chain: step %d: only TB_EPI_RESIDUAL and TB_EPI_SWIGLU", i);
        TB_REQUIRE(ctx, !(swiglu && resid), TB_ERR_UNSUPPORTED, "linear chain: step %d: SwiGLU takes no residual", i);
        TB_REQUIRE(ctx, !resid || t.residual, TB_ERR_ARG, "linear chain: step %d: TB_EPI_RESIDUAL without residual", i);
        const int64_t ncol = swiglu ? t.N / 2 : t.N;
        TB_REQUIRE(ctx, t.ldx >= t.K && t.ldy >= ncol && t.ldx % 8 == 0 && t.ldy % 8 == 0, TB_ERR_ALIGN,
                   "linear chain: step %d: row strides (ldx >= K, ldy >= output columns, multiples of 8)", i);
        TB_REQUIRE(ctx, aligned16(t.x) && aligned16(t.w) && aligned16(t.y) && (!t.residual || aligned16(t.residual)) &&
                            (!t.norm_w || aligned16(t.norm_w)),
                   TB_ERR_ALIGN, "linear chain: step %d: pointers must be 16-byte aligned", i);
        ChainStep& c = cs[i];
        c = ChainStep{};
        c.x = t.x;
        c.x_ld = t.ldx;
        c.w = t.w;
        c.Nw = (int)t.N;
        c.K = (int)t.K;
        c.ep.out = t.y;
        c.ep.ldo = t.ldy;
        c.ep.resid = resid ? t.residual : nullptr;
        c.ep.ldr = t.ldy;
        c.ep.swiglu = swiglu ? 1 : 0;
        c.ep.norm_w = t.norm_w;
        c.ep.norm_eps = t.norm_eps;
        if (ncol > max_cols) max_cols = (int)ncol;
    }
    // scratch: grown (and zeroed) when a call needs more than the last one
    const size_t lw = chain_ll_words((int)M, max_cols);
    if (!ctx->chain_sync || lw > ctx->chain_ll_words) {
        TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
        if (!ctx->chain_sync) {
            unsigned* sw = nullptr;
            if (cudaMalloc(&sw, kChainSyncWords * sizeof(unsigned)) != cudaSuccess ||
                cudaMemset(sw, 0, kChainSyncWords * sizeof(unsigned)) != cudaSuccess) {
                cudaGetLastError();
                if (sw) cudaFree(sw);
                return set_error(ctx, TB_ERR_OOM, "linear chain: scratch allocation failed");
            }
            ctx->chain_sync = sw;
        }
        if (ctx->chain_ll) cudaFree(ctx->chain_ll);
        ctx->chain_ll = nullptr;
        ctx->chain_ll_words = 0;
        if (cudaMalloc(&ctx->chain_ll, lw * sizeof(uint64_t)) != cudaSuccess ||
            cudaMemset(ctx->chain_ll, 0, lw * sizeof(uint64_t)) != cudaSuccess) {
            cudaGetLastError();
            return set_error(ctx, TB_ERR_OOM, "linear chain: scratch allocation failed");
        }
        ctx->chain_ll_words = lw;
    }
    ChainScratch scr;
    scr.sync = ctx->chain_sync;
    scr.ll = ctx->chain_ll;
    scr.ll_words = ctx->chain_ll_words;
    int rc = chain_launch(ctx, cs, n_steps, (int)M, scr);
    if (rc) return rc;
    return check_launch(ctx, "linear chain");
}

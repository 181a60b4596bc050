// conv2d forward (NCHW, groups = 1) with the inference epilogue
// bias -> folded BatchNorm scale/shift -> activation.
//
//  * bf16: implicit GEMM on tcgen05.  The input is first transposed to NHWC
//    with channels padded to a multiple of 8 (caller workspace), the weights
//    reordered to [Cout][KH][KW][Cin_pad].  GEMM view: M = output pixels,
//    N = Cout, K = KH * KW * Cin_pad.  A persistent kernel computes tiles of
//    32 x 8 output pixels x 64 output channels (see conv_tc_kernel).  Unit
//    stride, OW % 8 == 0, filters up to 5 x 5 (see conv_tc_ok).
//  * CUDA cores: implicit GEMM with exact f32 FMA accumulation, for f32 I/O
//    (the reference's fp32 kernels, conv2d.rs:44-148 / :643-764, and its 1e-4
//    tolerance) and for the bf16 shapes the tensor-core path does not take.
#include <stdlib.h>

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
// One launch prepares both operands of the tensor-core conv:
//  * x [B][C][H][W] bf16 -> xn [B][H][W][Cp] bf16, channels >= C zero.  CTA
//    (image row, 64 columns, 64 channels) for blockIdx.z < B * H: thread
//    (channel pair p, 8 columns) reads the two channel rows (16-byte loads
//    when rows are 16-byte aligned), interleaves them into 32-bit (c, c + 1)
//    words with byte permutes and stores them to a [pair][column] tile whose
//    row stride of 66 words makes the read-back conflict-free; a thread then
//    gathers 4 pairs of one column and stores 8 channels of one pixel (16 B).
//    Only bits are moved: bf16 in, bf16 out.
//  * w [Co][C][KH][KW] -> wr [Co][KH][KW][Cp] bf16 (channels >= C zero), one
//    element per thread, by the first CTAs (blockIdx.z < rz), so they are
//    scheduled first and overlap the transpose instead of trailing it.
constexpr int PREP_TS = 66;   // tile row stride in 32-bit words (64 columns + 2)

__global__ void __launch_bounds__(256)
conv_prep_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ xn, int B, int C, int H, int W,
                 int Cp, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ wr, int Co, int KH, int KW,
                 int rz) {
    __shared__ __align__(16) uint32_t tile[32 * PREP_TS];
    pdl_trigger();
    pdl_wait();
    if ((int)blockIdx.z < rz) {
        const int64_t total = (int64_t)Co * KH * KW * Cp;
        const int64_t nrb = (int64_t)rz * gridDim.y * gridDim.x;
        const int64_t rb = ((int64_t)blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        for (int64_t i = rb * 256 + threadIdx.x; i < total; i += nrb * 256) {
            const int c = (int)(i % Cp);
            int64_t r = i / Cp;
            const int kw = (int)(r % KW);
            r /= KW;
            const int kh = (int)(r % KH);
            const int co = (int)(r / KH);
            wr[i] = c < C ? w[(((int64_t)co * C + c) * KH + kh) * KW + kw] : __float2bfloat16_rn(0.f);
        }
        return;
    }
    const int bh = blockIdx.z - rz;       // b * H + h
    const int b = bh / H, h = bh % H;
    const int w0 = blockIdx.x * 64, c0 = blockIdx.y * 64;
    const bool vec = (W % 8) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    {
        const int p = threadIdx.x >> 3, ch = threadIdx.x & 7;   // channel pair, 8-column chunk
        const int ca = c0 + 2 * p, gw = w0 + 8 * ch;
        uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};  // 8 bf16 of channel ca and ca + 1
        if (gw < W) {
            const __nv_bfloat16* ra = x + (((int64_t)b * C + ca) * H + h) * W + gw;
            const __nv_bfloat16* rb = ra + (int64_t)H * W;
            if (vec && gw + 8 <= W) {
                if (ca < C) {
                    const uint4 u = *reinterpret_cast<const uint4*>(ra);
                    lo[0] = u.x; lo[1] = u.y; lo[2] = u.z; lo[3] = u.w;
                }
                if (ca + 1 < C) {
                    const uint4 u = *reinterpret_cast<const uint4*>(rb);
                    hi[0] = u.x; hi[1] = u.y; hi[2] = u.z; hi[3] = u.w;
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; k++) {
                    const uint32_t va = (ca < C && gw + k < W) ? __bfloat16_as_ushort(ra[k]) : 0u;
                    const uint32_t vb = (ca + 1 < C && gw + k < W) ? __bfloat16_as_ushort(rb[k]) : 0u;
                    lo[k >> 1] |= va << (16 * (k & 1));
                    hi[k >> 1] |= vb << (16 * (k & 1));
                }
            }
        }
        // word for column 2j: (ca, ca + 1) = low halves; column 2j + 1: high halves
        uint32_t* trow = tile + p * PREP_TS + 8 * ch;
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<uint2*>(trow + 2 * j) =
                make_uint2(__byte_perm(lo[j], hi[j], 0x5410), __byte_perm(lo[j], hi[j], 0x7632));
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 2; k++) {
        const int i = threadIdx.x + 256 * k;
        const int oct = (i >> 3) & 7, col = (i & 7) + 8 * (i >> 6);   // 8-channel group, column
        const int gw = w0 + col, gc = c0 + 8 * oct;
        if (gw >= W || gc >= Cp) continue;
        const uint32_t* t = tile + (4 * oct) * PREP_TS + col;
        *reinterpret_cast<uint4*>(xn + (((int64_t)b * H + h) * W + gw) * Cp + gc) =
            make_uint4(t[0], t[PREP_TS], t[2 * PREP_TS], t[3 * PREP_TS]);
    }
}

// ---------------------------------------------------------- tcgen05 conv --
// Persistent implicit GEMM for Y^T: output channels are the MMA's rows (A =
// weights [64 couts][64 channels] of one tap and channel chunk), output
// pixels its columns (B = a tile of BH x 8 pixels, BH <= 32 chosen per shape
// so row tiles are not padded, conv_bh).  One thread issues an MMA per ~75 ns
// whatever its N, so every instruction carries up to N = 256 pixels; the M = 128 instruction also reads the 64 weight
// rows that follow (next slice), which land in TMEM lanes 64-127 and are
// never read.  Per tile and 64-channel chunk ONE TMA load brings the haloed
// NHWC patch [32 + KH - 1 rows][8 + KW - 1 columns][64 channels] (128-B
// swizzle; zero fill outside the image = the padding).  Tap (kh, kw) is the
// B operand read in place: start patch row kh * PW + kw, 8-pixel groups one
// patch row (PW * 128 B) apart; the swizzle is a function of the absolute
// shared-memory address, so shifted starts read what TMA wrote (descriptor
// base offset 0).  Weights stay resident when they fit, else stream through
// a ring.  TMEM holds two [128 x 256] f32 accumulators so the epilogue of one
// tile overlaps the MMAs of the next.  Epilogue: warps 4, 5, 8, 9 (TMEM lanes
// 0-63 = channels; 128 pixels each) apply bias -> BN -> activation and stage
// [row][channel][column] (16-byte rows, conflict-free) for a TMA store to NCHW
// (OS = 1 or 2 staging buffers, whichever fits beside the patch ring).
constexpr int CONV_BH_MAX = 32, CONV_BW = 8, CONV_BN = 64;   // tile: BH x 8 pixels x 64 output channels
constexpr int CONV_WS = 4;                                   // weight ring slices (streaming mode)
constexpr int CONV_W_BYTES = CONV_BN * 128;                  // [64 couts][64 channels] bf16
constexpr int CONV_ACC_COLS = 256;                           // TMEM columns per accumulator (N <= 256)
constexpr int CONV_TMEM = 2 * CONV_ACC_COLS;                 // two accumulators
constexpr int CONV_THREADS = 320;                            // warps 0 TMA, 1-2 MMA, 4-5 + 8-9 epilogue

// Tile height: the fewest row tiles of at most 32 rows, each of even height (the
// MMA's N = 8 * BH must be a multiple of 16), e.g. 56 output rows -> 2 x 28.
__host__ __device__ constexpr int conv_bh(int OH) {
    const int t = (OH + CONV_BH_MAX - 1) / CONV_BH_MAX;
    const int h = (OH + t - 1) / t;
    return (h + 1) / 2 * 2;
}
__host__ __device__ constexpr int conv_pw(int KW) { return CONV_BW + KW - 1; }
__host__ __device__ constexpr int conv_patch_bytes(int BH, int KH, int KW) { return (BH + KH - 1) * conv_pw(KW) * 128; }
__host__ __device__ constexpr int conv_out_bytes(int BH) { return BH * CONV_BW * CONV_BN * 2; }   // [BH rows][64 couts][8 columns]
// wslots: weight slices held in shared memory (all of them when resident, else the ring);
// OS: output staging buffers (2 lets a tile's staging overlap the previous tile's store)
__host__ __device__ constexpr int conv_smem_bytes(int BH, int KH, int KW, int AS, int wslots, int OS) {
    return AS * ((conv_patch_bytes(BH, KH, KW) + 1023) / 1024 * 1024) + wslots * CONV_W_BYTES + OS * conv_out_bytes(BH) +
           1024 + 256;
}

__device__ __forceinline__ void tma_store_4d_async(const CUtensorMap* m, uint32_t src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(m)),
                 "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Shapes the tensor-core path takes: unit stride, output rows of 16-byte
// multiples (the NCHW TMA store), KH <= 7, KW <= 9, and the shared-memory
// footprint within 227 KB (e.g. 5 x 5 fits, 7 x 7 does not).
struct ConvShape;
bool conv_tc_ok(const ConvShape& s, int stride, int KH, int KW);

__global__ void __launch_bounds__(CONV_THREADS, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
               const __grid_constant__ CUtensorMap tmY, ConvEpi ep, int B, int OH, int OW, int Cout, int KH, int KW,
               int Cp, int pad, int AS, int wres, int BH, int OS, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    const int PW = conv_pw(KW);
    const int a_bytes = (conv_patch_bytes(BH, KH, KW) + 1023) / 1024 * 1024;
    const int NPIX = BH * CONV_BW;            // MMA N
    const int out_bytes = conv_out_bytes(BH);
    const int nc = (Cp + 63) / 64;            // 64-channel chunks
    const int taps = KH * KW;
    const int wslots = wres ? taps * nc : CONV_WS;
    // Patch and (streaming) weight rings: one half per MMA issuer (slots i * PD ..,
    // i * WD ..).  The issuers take tiles in turn, and a slot shared between them
    // could be waited on two fills ahead of its barrier, which a parity wait
    // cannot tell from one fill behind.  One producer and one consumer per slot.
    const int PD = AS / 2, WD = CONV_WS / 2;
    uint8_t* sP = smem;                                        // [AS] patches
    uint8_t* sW = sP + AS * a_bytes;                           // weight slices
    uint8_t* sO = sW + wslots * CONV_W_BYTES;                  // [2] output staging (also the
                                                               // rows past the last weight slice)
    uint64_t* bars = reinterpret_cast<uint64_t*>(sO + OS * out_bytes);
    // p_full[4], p_empty[4], w_full[WS], w_empty[WS], acc_full[2], acc_empty[2]
    const uint32_t p_full0 = smem_u32(bars), p_empty0 = smem_u32(bars + 4);
    const uint32_t w_full0 = smem_u32(bars + 8), w_empty0 = smem_u32(bars + 8 + CONV_WS);
    const uint32_t acc_full0 = smem_u32(bars + 8 + 2 * CONV_WS), acc_empty0 = smem_u32(bars + 10 + 2 * CONV_WS);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12 + 2 * CONV_WS);

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int tiles_w = (OW + CONV_BW - 1) / CONV_BW, tiles_h = (OH + BH - 1) / BH;
    const int nN = (Cout + CONV_BN - 1) / CONV_BN;
    const int units = tiles_w * tiles_h * B * nN;
    auto tile_of = [&](int t, int& b, int& oh0, int& ow0, int& n0) {
        n0 = (t % nN) * CONV_BN;
        int p = t / nN;
        ow0 = (p % tiles_w) * CONV_BW;
        p /= tiles_w;
        oh0 = (p % tiles_h) * BH;
        b = p / tiles_h;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < AS; s++) {
            mbar_init(p_full0 + 8 * s, 1);
            mbar_init(p_empty0 + 8 * s, 1);
        }
        for (int s = 0; s < CONV_WS; s++) {
            mbar_init(w_full0 + 8 * s, 1);
            mbar_init(w_empty0 + 8 * s, 1);
        }
        for (int s = 0; s < 2; s++) {
            mbar_init(acc_full0 + 8 * s, 1);
            mbar_init(acc_empty0 + 8 * s, 4);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), CONV_TMEM);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();

    if (warp == 0) {
        // ---------------- producer: haloed input patch per (tile, chunk); weights
        if (lane == 0) {
            tma_prefetch_desc(&tmX);
            tma_prefetch_desc(&tmW);
            int jp[2] = {0, 0}, jw[2] = {0, 0};   // patches / weight slices handed to each issuer
            bool ok = true;
            if (wres && blockIdx.x < units) {
                // every weight slice of this CTA's output block (grid % nN == 0: fixed block)
                const int n0 = (blockIdx.x % nN) * CONV_BN;
                mbar_expect_tx(w_full0, (uint32_t)(wslots * CONV_W_BYTES));
                for (int k = 0; k < wslots; k++)
                    tma_load_2d(smem_u32(sW + k * CONV_W_BYTES), &tmW, w_full0, (k % taps) * Cp + (k / taps) * 64, n0);
            }
            for (int t = blockIdx.x, tl = 0; ok && t < units; t += gridDim.x, tl++) {
                int b, oh0, ow0, n0;
                tile_of(t, b, oh0, ow0, n0);
                const int i = tl & 1;   // the issuer of this tile
                for (int c = 0; ok && c < nc; c++) {
                    const int j = jp[i]++;
                    const int sp = i * PD + j % PD;
                    if (j >= PD && !mbar_wait(p_empty0 + 8 * sp, ((j / PD) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(p_full0 + 8 * sp, (uint32_t)conv_patch_bytes(BH, KH, KW));
                    tma_load_4d(smem_u32(sP + sp * a_bytes), &tmX, p_full0 + 8 * sp, c * 64, ow0 - pad, oh0 - pad, b);
                    for (int tap = 0; !wres && tap < taps; tap++) {
                        const int jj = jw[i]++;
                        const int sw = i * WD + jj % WD;
                        if (jj >= WD && !mbar_wait(w_empty0 + 8 * sw, ((jj / WD) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        mbar_expect_tx(w_full0 + 8 * sw, CONV_W_BYTES);
                        tma_load_2d(smem_u32(sW + sw * CONV_W_BYTES), &tmW, w_full0 + 8 * sw, tap * Cp + c * 64, n0);
                    }
                }
            }
            // every load issued has landed before the CTA can exit
            for (int i = 0; i < 2; i++) {
                for (int j = (jp[i] > PD ? jp[i] - PD : 0); j < jp[i]; j++)
                    mbar_wait(p_full0 + 8 * (i * PD + j % PD), (j / PD) & 1, err, DEV_ERR_TIMEOUT_FULL);
                for (int j = (jw[i] > WD ? jw[i] - WD : 0); j < jw[i]; j++)
                    mbar_wait(w_full0 + 8 * (i * WD + j % WD), (j / WD) & 1, err, DEV_ERR_TIMEOUT_FULL);
            }
            if (wres && blockIdx.x < units) mbar_wait(w_full0, 0, err, DEV_ERR_TIMEOUT_FULL);
        }
    } else if (warp == 1 || warp == 2) {
        // ---------------- MMA issuers: D^T[couts][pixels] += W_tap (A) x patch_tap (B).
        // Warp 1 issues the CTA's even tiles (accumulator 0), warp 2 the odd ones
        // (accumulator 1), so one tile's MMAs do not wait on the other's patch.
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, NPIX, false, false);
            // descriptors built once; an operand at byte offset o adds o >> 4 (start-address field)
            const uint64_t b_desc0 = sdesc_sw128(smem_u32(sP), 16, (uint32_t)PW * 128);
            const uint64_t a_desc0 = sdesc_sw128(smem_u32(sW), 16, 1024);
            const int par = warp - 1;   // tile parity of this issuer
            bool ok = !wres || blockIdx.x >= units || mbar_wait(w_full0, 0, err, DEV_ERR_TIMEOUT_FULL);
            for (int t = blockIdx.x + par * gridDim.x, tl = par; ok && t < units; t += 2 * gridDim.x, tl += 2) {
                const int ab = tl & 1;
                if (tl >= 2 && !mbar_wait(acc_empty0 + 8 * ab, ((tl >> 1) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + ab * CONV_ACC_COLS;
                for (int c = 0; ok && c < nc; c++) {
                    const int j = (tl >> 1) * nc + c;    // this issuer's patch number
                    const int sp = par * PD + j % PD;
                    if (!mbar_wait(p_full0 + 8 * sp, (j / PD) & 1, err, DEV_ERR_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    const uint64_t b_st = b_desc0 + (uint64_t)((sp * a_bytes) >> 4);
                    for (int tap = 0, kh = 0, kw = 0; tap < taps; tap++) {
                        const int wi = j * taps + tap;   // this issuer's weight slice number (streaming mode)
                        const int sw = wres ? c * taps + tap : par * WD + wi % WD;
                        if (!wres && !mbar_wait(w_full0 + 8 * sw, (wi / WD) & 1, err, DEV_ERR_TIMEOUT_FULL)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t b_tap = b_st + (uint64_t)((kh * PW + kw) * 8);   // rows of 128 B
                        const uint64_t a_tap = a_desc0 + (uint64_t)(sw * (CONV_W_BYTES >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_f16_ss(d_tmem, a_tap + 2 * kk, b_tap + 2 * kk, idesc, (c | tap | kk) != 0);
                        if (!wres) umma_commit(w_empty0 + 8 * sw);
                        if (++kw == KW) {
                            kw = 0;
                            kh++;
                        }
                    }
                    umma_commit(p_empty0 + 8 * sp);
                }
                umma_commit(acc_full0 + 8 * ab);
            }
        }
    } else if (warp == 4 || warp == 5 || warp == 8 || warp == 9) {
        // ---------------- epilogue: thread <-> output channel co = 32 * (warp % 4) + lane
        // (TMEM lane), pixel columns [128 * half, 128 * half + 128) of the tile
        const int q = warp & 3, half = warp >> 3;
        const int col = q * 32 + lane;            // channel within the block
        bool ok = true;
        int tl = 0, cur_n0 = -1;
        float eb = 0.f, es = 1.f, et = 0.f;
        for (int t = blockIdx.x; t < units; t += gridDim.x, tl++) {
            int b, oh0, ow0, n0;
            tile_of(t, b, oh0, ow0, n0);
            const int ab = tl & 1;
            const int co = n0 + col;
            if (n0 != cur_n0) {
                eb = 0.f;
                es = 1.f;
                et = 0.f;
                if (co < Cout) {
                    if (ep.bias && !ep.shift) eb = ep.bias[co];
                    if (ep.scale) es = ep.scale[co];
                    if (ep.shift) et = ep.shift[co];
                }
                cur_n0 = n0;
            }
            ok = mbar_wait(acc_full0 + 8 * ab, (tl >> 1) & 1, err, DEV_ERR_TIMEOUT_ACC) && ok;
            tc_fence_after();
            // TMEM -> registers 32 pixels at a time, the next chunk's load in flight
            // while the current one is processed; the accumulator is released as
            // soon as its last chunk has been read
            const int pbeg = half * 128;
            const int pend = pbeg + 128 < NPIX ? pbeg + 128 : NPIX;
            const uint32_t t_acc = tmem + ((uint32_t)(q * 32) << 16) + ab * CONV_ACC_COLS;
            float v[32];
            if (pbeg < pend) tmem_ld32(t_acc + pbeg, v);
            // the staging buffer was last read by the store issued OS tiles ago
            if (warp == 4 && lane == 0) {
                if (OS == 2) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
                else asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            }
            asm volatile("bar.sync 2, 128;" ::: "memory");
            uint8_t* so = sO + (OS == 2 ? ab : 0) * out_bytes;
            tmem_wait_ld32(v);
            if (pbeg >= pend) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(acc_empty0 + 8 * ab);
            }
#pragma unroll 1
            for (int p0 = pbeg; p0 < pend; p0 += 32) {
                float c[32];
#pragma unroll
                for (int j = 0; j < 32; j++) c[j] = v[j];
                const bool more = p0 + 32 < pend;
                if (more) {
                    tmem_ld32(t_acc + p0 + 32, v);
                } else {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(acc_empty0 + 8 * ab);
                }
                // c -> ((c + bias) * scale + shift) -> activation (as conv_epi)
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    float o = (c[j] + eb) * es + et;
                    if (ep.act == TB_ACT_RELU) o = o > 0.f ? o : 0.f;
                    else if (ep.act == TB_ACT_SILU) o = o / (1.0f + expf(-o));
                    c[j] = co < Cout ? o : 0.f;
                }
                // pixels p0 .. p0 + 31 = rows p0 / 8 .. + 3, 8 columns each: [row][channel][column]
                // (rows past BH, when NPIX is not a multiple of 32, are not staged)
#pragma unroll
                for (int r = 0; r < 4; r++) {
                    if (p0 / 8 + r >= BH) break;
                    uint4 u;
                    u.x = pack_bf16x2(c[8 * r + 0], c[8 * r + 1]);
                    u.y = pack_bf16x2(c[8 * r + 2], c[8 * r + 3]);
                    u.z = pack_bf16x2(c[8 * r + 4], c[8 * r + 5]);
                    u.w = pack_bf16x2(c[8 * r + 6], c[8 * r + 7]);
                    *reinterpret_cast<uint4*>(so + ((p0 / 8 + r) * CONV_BN + col) * 16) = u;
                }
                if (more) tmem_wait_ld32(v);
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (warp == 4 && lane == 0 && ok) tma_store_4d_async(&tmY, smem_u32(so), ow0, n0, oh0, b);
        }
        if (warp == 4 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, CONV_TMEM);
}

// ------------------------------------------- tcgen05 conv, pixels as rows --
// The same implicit GEMM with output PIXELS as the MMA's M = 128 rows (a tile of
// 16 output rows x 8 columns) and the 64 output channels of a block as N.
// Every MMA row is a real output (conv_tc_kernel's 64-channel M leaves half of
// each instruction's rows unused), and the accumulator spans all four TMEM
// lane quarters, so the epilogue runs on all four SM sub-partitions.
//   A = the haloed NHWC patch read in place per tap (8-pixel groups one patch
//       row apart, as conv_tc_kernel's B operand);  B = the tap's resident
//       weights [64 couts][64 channels].
// An N = 64 tcgen05.mma takes ~26 ns of the tensor pipe (10 TFLOP/s per SM).
// Four warps (1, 2, 3, 12) issue the tiles tl = i, i + 4, ... of this CTA,
// each into its own two of eight 64-column TMEM accumulators, so a tile whose
// patch or accumulator is late does not hold up the others' MMAs.  Two epilogue groups (warps 4-7 and 8-11,
// one warp per lane quarter) take alternate tiles: thread = pixel, 64 channels
// each, staged as [channel][row][column] for one TMA store into NCHW.
constexpr int PM_BH = 16;                          // tile rows (16 x 8 = 128 pixels = M)
constexpr int PM_THREADS = 416;                    // 13 warps
constexpr int PM_ACC = 8;                          // TMEM accumulators of 64 columns
constexpr int PM_ISSUERS = 4;
constexpr int PM_OUT_BYTES = CONV_BN * PM_BH * CONV_BW * 2;   // [64 couts][16 rows][8 columns] bf16

__host__ __device__ constexpr int pm_smem_bytes(int KH, int KW, int AS, int wslots) {
    return AS * ((conv_patch_bytes(PM_BH, KH, KW) + 1023) / 1024 * 1024) + wslots * CONV_W_BYTES + 2 * PM_OUT_BYTES +
           2 * CONV_BN * 4 + 1024 + 512;
}

__device__ __forceinline__ int pm_issuer(int warp) { return warp >= 1 && warp <= 3 ? warp - 1 : warp == 12 ? 3 : -1; }

__global__ void __launch_bounds__(PM_THREADS, 1)
conv_pm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
               const __grid_constant__ CUtensorMap tmY, ConvEpi ep, int B, int OH, int OW, int Cout, int KH, int KW,
               int Cp, int pad, int AS, int y_nhwc, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_align1024(smem_raw);
    const int PW = conv_pw(KW);
    const int a_bytes = (conv_patch_bytes(PM_BH, KH, KW) + 1023) / 1024 * 1024;
    const int nc = (Cp + 63) / 64;            // 64-channel chunks
    const int taps = KH * KW;
    const int wslots = taps * nc;             // resident weights of this CTA's output block
    // The patch ring is split into one sub-ring of PD slots per MMA issuer (slots
    // i * PD ..): the issuers take tiles in turn, and a slot shared between them
    // could be waited on two fills ahead of its barrier, which a parity wait
    // cannot tell from one fill behind.  One producer and one consumer per slot.
    const int PD = AS / PM_ISSUERS;
    uint8_t* sP = smem;                                        // [AS] patches
    uint8_t* sW = sP + AS * a_bytes;                           // weight slices
    uint8_t* sO = sW + wslots * CONV_W_BYTES;                  // [2 groups] output staging
    float2* sC = reinterpret_cast<float2*>(sO + 2 * PM_OUT_BYTES);   // [64] (scale, bias * scale + shift)
    uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(sC) + 2 * CONV_BN * 4);
    // p_full[8], p_empty[8], w_full, acc_full[8], acc_empty[8]
    const uint32_t p_full0 = smem_u32(bars), p_empty0 = smem_u32(bars + 8);
    const uint32_t w_full = smem_u32(bars + 16);
    const uint32_t acc_full0 = smem_u32(bars + 17), acc_empty0 = smem_u32(bars + 25);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 33);

    pdl_trigger();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int tiles_w = OW / CONV_BW, tiles_h = (OH + PM_BH - 1) / PM_BH;
    const int nN = (Cout + CONV_BN - 1) / CONV_BN;
    const int units = tiles_w * tiles_h * B * nN;
    const int n0c = (blockIdx.x % nN) * CONV_BN;   // grid % nN == 0: this CTA's output block
    auto tile_of = [&](int t, int& b, int& oh0, int& ow0) {
        int p = t / nN;
        ow0 = (p % tiles_w) * CONV_BW;
        p /= tiles_w;
        oh0 = (p % tiles_h) * PM_BH;
        b = p / tiles_h;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < 8; s++) {
            mbar_init(p_full0 + 8 * s, 1);
            mbar_init(p_empty0 + 8 * s, 1);
        }
        mbar_init(w_full, 1);
        for (int s = 0; s < PM_ACC; s++) {
            mbar_init(acc_full0 + 8 * s, 1);
            mbar_init(acc_empty0 + 8 * s, 4);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(tmem_slot), 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();
    // per-channel epilogue constants of the block: (c + bias) * scale + shift as one
    // FMA, c * scale + (bias * scale + shift)
    if (threadIdx.x < CONV_BN) {
        const int co = n0c + threadIdx.x;
        float eb = 0.f, es = 1.f, et = 0.f;
        if (co < Cout) {
            if (ep.bias && !ep.shift) eb = ep.bias[co];
            if (ep.scale) es = ep.scale[co];
            if (ep.shift) et = ep.shift[co];
        }
        sC[threadIdx.x] = make_float2(es, fmaf(eb, es, et));
    }
    __syncthreads();

    const int iss = pm_issuer(warp);
    if (warp == 0) {
        // ---------------- producer: the block's weights once, then one haloed patch per (tile, chunk)
        if (lane == 0) {
            tma_prefetch_desc(&tmX);
            tma_prefetch_desc(&tmW);
            int jc[PM_ISSUERS] = {0, 0, 0, 0};   // patches handed to each issuer so far
            bool ok = true;
            if (blockIdx.x < units) {
                mbar_expect_tx(w_full, (uint32_t)(wslots * CONV_W_BYTES));
                for (int k = 0; k < wslots; k++)
                    tma_load_2d(smem_u32(sW + k * CONV_W_BYTES), &tmW, w_full, (k % taps) * Cp + (k / taps) * 64, n0c);
            }
            for (int t = blockIdx.x, tl = 0; ok && t < units; t += gridDim.x, tl++) {
                int b, oh0, ow0;
                tile_of(t, b, oh0, ow0);
                const int i = tl % PM_ISSUERS;
                for (int c = 0; ok && c < nc; c++) {
                    const int j = jc[i]++;
                    const int sp = i * PD + j % PD;
                    if (j >= PD && !mbar_wait(p_empty0 + 8 * sp, ((j / PD) - 1) & 1, err, DEV_ERR_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(p_full0 + 8 * sp, (uint32_t)conv_patch_bytes(PM_BH, KH, KW));
                    tma_load_4d(smem_u32(sP + sp * a_bytes), &tmX, p_full0 + 8 * sp, c * 64, ow0 - pad, oh0 - pad, b);
                }
            }
            // every load issued has landed before the CTA can exit
            for (int i = 0; i < PM_ISSUERS; i++)
                for (int j = (jc[i] > PD ? jc[i] - PD : 0); j < jc[i]; j++)
                    mbar_wait(p_full0 + 8 * (i * PD + j % PD), (j / PD) & 1, err, DEV_ERR_TIMEOUT_FULL);
            if (blockIdx.x < units) mbar_wait(w_full, 0, err, DEV_ERR_TIMEOUT_FULL);
        }
    } else if (iss >= 0) {
        // ---------------- MMA issuer iss: tiles tl = iss, iss + 4, ... of this CTA into
        // accumulators tl % 8.  D[pixels][couts] += patch_tap (A) x W_tap (B).
        if (lane == 0) {
            const uint32_t idesc = idesc_bf16_f32(128, CONV_BN, false, false);
            const uint64_t a_desc0 = sdesc_sw128(smem_u32(sP), 16, (uint32_t)PW * 128);
            const uint64_t b_desc0 = sdesc_sw128(smem_u32(sW), 16, 1024);
            bool ok = blockIdx.x >= units || mbar_wait(w_full, 0, err, DEV_ERR_TIMEOUT_FULL);
            for (int t = blockIdx.x + iss * gridDim.x, tl = iss; ok && t < units; t += PM_ISSUERS * gridDim.x, tl += PM_ISSUERS) {
                const int ab = tl % PM_ACC;
                if (tl >= PM_ACC && !mbar_wait(acc_empty0 + 8 * ab, ((tl / PM_ACC) - 1) & 1, err, DEV_ERR_TIMEOUT_MISC)) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem + ab * CONV_BN;
                for (int c = 0; ok && c < nc; c++) {
                    const int j = (tl / PM_ISSUERS) * nc + c;   // this issuer's patch number
                    const int sp = iss * PD + j % PD;
                    if (!mbar_wait(p_full0 + 8 * sp, (j / PD) & 1, err, DEV_ERR_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t a_st = a_desc0 + (uint64_t)((sp * a_bytes) >> 4);
                    for (int tap = 0, kh = 0, kw = 0; tap < taps; tap++) {
                        const uint64_t a_tap = a_st + (uint64_t)((kh * PW + kw) * 8);   // rows of 128 B
                        const uint64_t b_tap = b_desc0 + (uint64_t)((c * taps + tap) * (CONV_W_BYTES >> 4));
#pragma unroll
                        for (int kk = 0; kk < 4; kk++)
                            umma_f16_ss(d_tmem, a_tap + 2 * kk, b_tap + 2 * kk, idesc, (c | tap | kk) != 0);
                        if (++kw == KW) {
                            kw = 0;
                            kh++;
                        }
                    }
                    umma_commit(p_empty0 + 8 * sp);
                }
                umma_commit(acc_full0 + 8 * ab);
            }
        }
    } else if (warp >= 4 && warp < 12) {
        // ---------------- epilogue group g (warps 4-7 or 8-11): tiles tl = g, g + 2, ...;
        // thread <-> pixel m = 32 * (warp % 4) + lane (TMEM lane) = row m / 8, column m % 8
        const int g = (warp - 4) >> 2, q = warp & 3;
        const int m = q * 32 + lane, pr = m >> 3, pc = m & 7;
        uint8_t* so = sO + g * PM_OUT_BYTES;
        const int bar_id = 2 + g;
        bool ok = true;
        for (int t = blockIdx.x + g * gridDim.x, tl = g; t < units; t += 2 * gridDim.x, tl += 2) {
            int b, oh0, ow0;
            tile_of(t, b, oh0, ow0);
            const int ab = tl % PM_ACC;
            ok = mbar_wait(acc_full0 + 8 * ab, (tl / PM_ACC) & 1, err, DEV_ERR_TIMEOUT_ACC) && ok;
            tc_fence_after();
            const uint32_t t_acc = tmem + ((uint32_t)(q * 32) << 16) + ab * CONV_BN;
            float v[64];
            tmem_ld32(t_acc, v);
            tmem_ld32(t_acc + 32, v + 32);
            // the staging buffer was last read by this group's previous store
            if (q == 0 && lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_empty0 + 8 * ab);
            asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
            // NCHW: channel j of pixel (pr, pc) -> staging [j][pr][pc]: a warp's 32 pixels
            // are 64 contiguous bytes of one channel plane (conflict-free).  NHWC: the
            // pixel's 64 channels -> staging row m of 128 B, 16-byte chunk k at k ^ (m % 8)
            // (the tensor map's 128-B swizzle; 8 consecutive pixels cover all banks).
            // The constants of 8 channels are loaded before their stores (the stores
            // could alias them, so a per-channel load would wait for the previous store).
            __nv_bfloat16* sob = reinterpret_cast<__nv_bfloat16*>(so) + pr * CONV_BW + pc;
            const int act = ep.act;
#pragma unroll
            for (int j0 = 0; j0 < 64; j0 += 8) {
                float4 kc[4];
#pragma unroll
                for (int i = 0; i < 4; i++) kc[i] = reinterpret_cast<const float4*>(sC + j0)[i];
                float o8[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float es = (i & 1) ? kc[i >> 1].z : kc[i >> 1].x, et = (i & 1) ? kc[i >> 1].w : kc[i >> 1].y;
                    float o = fmaf(v[j0 + i], es, et);
                    if (act == TB_ACT_RELU) o = o > 0.f ? o : 0.f;
                    else if (act == TB_ACT_SILU) o = o / (1.0f + expf(-o));
                    o8[i] = o;
                }
                if (y_nhwc) {
                    *reinterpret_cast<uint4*>(so + m * 128 + ((((j0 >> 3) ^ m) & 7) << 4)) =
                        make_uint4(pack_bf16x2(o8[0], o8[1]), pack_bf16x2(o8[2], o8[3]), pack_bf16x2(o8[4], o8[5]),
                                   pack_bf16x2(o8[6], o8[7]));
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) sob[(j0 + i) * PM_BH * CONV_BW] = __float2bfloat16_rn(o8[i]);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            asm volatile("bar.sync %0, 128;" ::"r"(bar_id) : "memory");
            if (q == 0 && lane == 0 && ok) {
                if (y_nhwc) tma_store_4d_async(&tmY, smem_u32(so), n0c, ow0, oh0, b);
                else tma_store_4d_async(&tmY, smem_u32(so), ow0, oh0, n0c, b);
            }
        }
        if (q == 0 && lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 512);
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

// ------------------------------------------------- f32 3 x 3 direct conv ---
// fp32, 3 x 3, stride 1, pad 1 (the fp32 C2 stage): a CTA computes two output
// rows of one image for 64 output channels; thread (cg, seg, row) the 8
// consecutive pixels [8 seg, 8 seg + 8) of its row x the 8 channels [8 cg, 8 cg + 8)
// of the block, 64 accumulators.  Per chunk of 8 input channels the four input
// rows the two output rows need ([8][4][W + 2], zero padded) and the chunk's weights, transposed to
// [8][9][64] so that a thread's 8 output channels are two 16-byte words, are
// staged in shared memory; per (channel, kh) a thread reads one 10-float input
// window, reused by the three kw taps, and 24 weights: 192 FMAs for 9 loads.
// Many small CTAs (row pairs x images, 4 resident per SM at W = 56) keep the SMs
// evenly loaded and cover each other's staging; a chunk's weights serve both rows.
// Accumulation order: channel, kh, kw.
constexpr int C3_CC = 8;                 // input channels per chunk
constexpr int C3_WS = 64 + 4;            // weight row stride (16-byte aligned rows)
constexpr int C3_TR = 2;                 // output rows per CTA (the chunk's weights serve both)

__global__ void __launch_bounds__(256, 2)
conv3x3_f32_kernel(const float* __restrict__ x, const float* __restrict__ w, ConvEpi ep, float* __restrict__ y, int C,
                   int Co, int H, int W) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float c3_smem[];
    constexpr int XR = C3_TR + 2;                    // input rows per channel
    const int XW = W + 4;                            // input row stride: columns -1 .. W, 16-byte aligned rows
    float* xs = c3_smem;                             // [C3_CC * XR][XW]
    float* ws = xs + C3_CC * XR * XW;                // [C3_CC * 9][C3_WS]
    const int oh0 = blockIdx.x * C3_TR, b = blockIdx.y, co0 = blockIdx.z * 64;
    const int t = threadIdx.x, nt = blockDim.x;
    const int SEG = W / 8;
    const int cg = t & 7, seg = (t >> 3) % SEG, rr = (t >> 3) / SEG;   // rr: this thread's output row
    const int oh = oh0 + rr;
    float acc[8][8];
#pragma unroll
    for (int j = 0; j < 8; j++)
#pragma unroll
        for (int i = 0; i < 8; i++) acc[j][i] = 0.f;
    const int K9 = C * 9;
    for (int c0 = 0; c0 < C; c0 += C3_CC) {
        // input rows oh0 - 1 .. oh0 + C3_TR of the chunk's channels, columns -1 .. W (zero
        // outside): row by row, the CTA's threads along each (unrolled, so a thread's
        // loads of several rows are in flight before their stores)
#pragma unroll 8
        for (int rc = 0; rc < C3_CC * XR; rc++) {
            const int r = rc % XR, cc = rc / XR;
            const int ih = oh0 - 1 + r;
            const bool row_in = ih >= 0 && ih < H;
            const float* xrow = x + (((int64_t)b * C + c0 + cc) * H + (row_in ? ih : 0)) * W;
            for (int col = t; col < W + 2; col += nt) {
                const int iw = col - 1;
                xs[rc * XW + col] = (row_in && iw >= 0 && iw < W) ? xrow[iw] : 0.f;
            }
        }
        // weights w[co][c][kh][kw] of the chunk (72 contiguous floats per output channel,
        // 16-byte aligned) -> ws[cc * 9 + tap][co]; consecutive threads take consecutive
        // output channels, so the transposing stores hit 32 different banks (the loads
        // are 2.3 KB apart, but each output channel's 288 bytes stay in L1 across q)
#pragma unroll 4
        for (int i = t; i < 64 * (C3_CC * 9 / 4); i += nt) {
            const int co = i & 63, q = i >> 6;
            const float4 v = *reinterpret_cast<const float4*>(w + (int64_t)(co0 + co) * K9 + c0 * 9 + q * 4);
            ws[(q * 4 + 0) * C3_WS + co] = v.x;
            ws[(q * 4 + 1) * C3_WS + co] = v.y;
            ws[(q * 4 + 2) * C3_WS + co] = v.z;
            ws[(q * 4 + 3) * C3_WS + co] = v.w;
        }
        __syncthreads();
#pragma unroll 1
        for (int cc = 0; cc < C3_CC; cc++) {
#pragma unroll
            for (int kh = 0; kh < 3; kh++) {
                const float* xr = xs + (cc * XR + rr + kh) * XW + seg * 8;
                float xin[10];
                const float4 x0 = *reinterpret_cast<const float4*>(xr);
                const float4 x1 = *reinterpret_cast<const float4*>(xr + 4);
                const float2 x2 = *reinterpret_cast<const float2*>(xr + 8);
                xin[0] = x0.x; xin[1] = x0.y; xin[2] = x0.z; xin[3] = x0.w;
                xin[4] = x1.x; xin[5] = x1.y; xin[6] = x1.z; xin[7] = x1.w;
                xin[8] = x2.x; xin[9] = x2.y;
#pragma unroll
                for (int kw = 0; kw < 3; kw++) {
                    const float* wr = ws + (cc * 9 + kh * 3 + kw) * C3_WS + cg * 8;
                    const float4 w0 = *reinterpret_cast<const float4*>(wr);
                    const float4 w1 = *reinterpret_cast<const float4*>(wr + 4);
                    const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int j = 0; j < 8; j++)
#pragma unroll
                        for (int i = 0; i < 8; i++) acc[j][i] = fmaf(xin[i + kw], wv[j], acc[j][i]);
                }
            }
        }
        __syncthreads();
    }
    if (oh >= H) return;   // the second row of the last CTA when H is odd
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int co = co0 + cg * 8 + j;
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; i++) o[i] = conv_epi(ep, co, acc[j][i]);
        float* dst = y + (((int64_t)b * Co + co) * H + oh) * W + seg * 8;
        *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(o[4], o[5], o[6], o[7]);
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

bool conv_tc_ok(const ConvShape& s, int stride, int KH, int KW) {
    // two patch stages + the weight ring + one output staging buffer within 227 KB of shared memory
    return stride == 1 && s.OW % 8 == 0 && KH <= 7 && KW <= 9 &&
           conv_smem_bytes(conv_bh(s.OH), KH, KW, 2, CONV_WS, 1) <= 227 * 1024;
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
    *bytes = (dtype == TB_BF16 && conv_tc_ok(s, stride, KH, KW)) ? conv_ws_bytes(s) : 0;
    return TB_OK;
}

int tb_conv2d_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias, const float* bn_scale,
                  const float* bn_shift, void* y, int B, int Cin, int Cout, int H, int W, int KH, int KW, int stride,
                  int pad, int act, void* workspace, size_t workspace_bytes) {
    return tb_conv2d_fwd_ex(ctx, dtype, x, w, bias, bn_scale, bn_shift, y, B, Cin, Cout, H, W, KH, KW, stride, pad, act,
                            0, workspace, workspace_bytes);
}

int tb_conv2d_pack_weights(tb_ctx* ctx, int dtype, const void* w, void* w_packed, int Cout, int Cin, int KH, int KW) {
    if (!ctx || !w || !w_packed) return TB_ERR_ARG;
    TB_REQUIRE(ctx, dtype == TB_BF16, TB_ERR_UNSUPPORTED, "conv2d_pack_weights: bf16 only");
    TB_REQUIRE(ctx, Cout > 0 && Cin > 0 && Cin % 8 == 0 && KH > 0 && KW > 0, TB_ERR_SHAPE,
               "conv2d_pack_weights: Cout, KH, KW > 0 and Cin a positive multiple of 8");
    const int64_t tot = (int64_t)Cout * KH * KW * Cin;
    const int rz = (int)std::min<int64_t>((tot + 255) / 256, 64);
    return launch(ctx, "conv_pack_weights", conv_prep_kernel, dim3(1, 1, rz), dim3(256), 0,
                  (const __nv_bfloat16*)nullptr, (__nv_bfloat16*)nullptr, 0, Cin, 1, 1, Cin,
                  (const __nv_bfloat16*)w, (__nv_bfloat16*)w_packed, Cout, KH, KW, rz);
}

int tb_conv2d_fwd_ex(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias, const float* bn_scale,
                     const float* bn_shift, void* y, int B, int Cin, int Cout, int H, int W, int KH, int KW, int stride,
                     int pad, int act, int flags, void* workspace, size_t workspace_bytes) {
    if (!ctx || !x || !w || !y) return TB_ERR_ARG;
    ConvShape s;
    TB_REQUIRE(ctx, conv_shape(B, Cin, Cout, H, W, KH, KW, stride, pad, &s), TB_ERR_SHAPE, "conv2d: bad shape");
    TB_REQUIRE(ctx, act == TB_ACT_NONE || act == TB_ACT_RELU || act == TB_ACT_SILU, TB_ERR_ARG, "conv2d: act %d", act);
    TB_REQUIRE(ctx, (flags & ~(TB_CONV_X_NHWC | TB_CONV_Y_NHWC | TB_CONV_W_PACKED)) == 0, TB_ERR_ARG,
               "conv2d: unknown flags %#x", flags);
    const bool x_nhwc = flags & TB_CONV_X_NHWC, y_nhwc = flags & TB_CONV_Y_NHWC, w_packed = flags & TB_CONV_W_PACKED;
    if (flags) {
        TB_REQUIRE(ctx, dtype == TB_BF16 && conv_tc_ok(s, stride, KH, KW), TB_ERR_UNSUPPORTED,
                   "conv2d: layout flags need bf16 and the tensor-core path (stride 1, OW %% 8 == 0)");
        TB_REQUIRE(ctx, !((x_nhwc || w_packed) && Cin % 8), TB_ERR_UNSUPPORTED,
                   "conv2d: NHWC x / packed w need Cin %% 8 == 0");
        TB_REQUIRE(ctx, !(y_nhwc && Cout % 8), TB_ERR_UNSUPPORTED, "conv2d: NHWC y needs Cout %% 8 == 0");
        TB_REQUIRE(ctx, !x_nhwc || aligned16(x), TB_ERR_ALIGN, "conv2d: NHWC x must be 16-byte aligned");
        TB_REQUIRE(ctx, !w_packed || aligned16(w), TB_ERR_ALIGN, "conv2d: packed w must be 16-byte aligned");
    }
    ConvEpi ep{bias, bn_scale, bn_shift, act};
    const int64_t P = (int64_t)B * s.OH * s.OW;
    const dim3 sgrid((unsigned)((P + 63) / 64), (unsigned)((Cout + 63) / 64));
    if (dtype == TB_F32 && stride == 1 && KH == 3 && KW == 3 && pad == 1 && Cin % C3_CC == 0 && Cout % 64 == 0 &&
        W % 8 == 0 && W <= 128 && B <= 65535 && aligned16(y) && aligned16(x) && aligned16(w)) {
        // fp32 3 x 3 direct conv: two output rows x 64 output channels per CTA (2W threads)
        const int smem = (C3_CC * (C3_TR + 2) * (W + 4) + C3_CC * 9 * C3_WS) * (int)sizeof(float);
        TB_CUDA_TRY(ctx, cudaFuncSetAttribute(conv3x3_f32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        return launch(ctx, "conv3x3_f32", conv3x3_f32_kernel,
                      dim3((unsigned)((H + C3_TR - 1) / C3_TR), (unsigned)B, (unsigned)(Cout / 64)),
                      dim3((unsigned)(C3_TR * W)), smem, (const float*)x, (const float*)w, ep, (float*)y, Cin, Cout, H, W);
    }
    if (dtype == TB_F32)
        return launch(ctx, "conv2d_f32", conv_simt_kernel<float>, sgrid, dim3(256), 0, (const float*)x, (const float*)w,
                      ep, (float*)y, B, Cin, Cout, H, W, KH, KW, stride, pad, s.OH, s.OW);
    if (dtype != TB_BF16) return set_error(ctx, TB_ERR_UNSUPPORTED, "conv2d: dtype %d", dtype);
    if (!conv_tc_ok(s, stride, KH, KW))   // tensor-core path: see conv_tc_ok
        return launch(ctx, "conv2d_simt_bf16", conv_simt_kernel<__nv_bfloat16>, sgrid, dim3(256), 0,
                      (const __nv_bfloat16*)x, (const __nv_bfloat16*)w, ep, (__nv_bfloat16*)y, B, Cin, Cout, H, W, KH,
                      KW, stride, pad, s.OH, s.OW);
    TB_REQUIRE(ctx, aligned16(y), TB_ERR_ALIGN, "conv2d bf16: y must be 16-byte aligned");
    // workspace: the NHWC copy of x, then the reordered weights (each only when the
    // caller does not already hold that layout)
    const size_t xn_bytes = x_nhwc ? 0 : (((size_t)B * H * W * s.Cp * 2 + 255) / 256) * 256;
    const size_t need = xn_bytes + (w_packed ? 0 : (((size_t)Cout * KH * KW * s.Cp * 2 + 255) / 256) * 256);
    TB_REQUIRE(ctx, need == 0 || (workspace && workspace_bytes >= need && aligned16(workspace)), TB_ERR_ARG,
               "conv2d bf16: workspace of %zu bytes required (tb_conv2d_workspace_size)", need);
    __nv_bfloat16* xn = x_nhwc ? (__nv_bfloat16*)x : reinterpret_cast<__nv_bfloat16*>(workspace);
    __nv_bfloat16* wr = w_packed ? (__nv_bfloat16*)w
                                 : reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(workspace) + xn_bytes);
    if (!x_nhwc || !w_packed) {
        // CTAs for the weight reorder (one element per thread, at most 64 z-slices), then
        // transpose CTAs for every (image row, 64 columns, 64 channels)
        const int64_t tot = w_packed ? 0 : (int64_t)Cout * KH * KW * s.Cp;
        const int gx = (W + 63) / 64, gy = (s.Cp + 63) / 64;
        const int64_t per_z = (int64_t)gx * gy * 256;
        const int rz = (int)std::min<int64_t>((tot + per_z - 1) / per_z, 64);
        dim3 grid(gx, gy, rz + (x_nhwc ? 0 : B * H));
        int rc = launch(ctx, "conv_prep", conv_prep_kernel, grid, dim3(256), 0, (const __nv_bfloat16*)x, xn, B, Cin, H, W,
                        s.Cp, (const __nv_bfloat16*)w, wr, Cout, KH, KW, rz);
        if (rc) return rc;
    }
    constexpr int kSmemMax = 227 * 1024;
    const int nN = (Cout + CONV_BN - 1) / CONV_BN;
    const int wall = KH * KW * ((s.Cp + 63) / 64);
    {
        // pixels-as-rows kernel: resident weights and at least four patch stages
        // (one per MMA issuer) must fit; TB_CONV_PM=0 keeps conv_tc_kernel
        static const bool pm_off = getenv("TB_CONV_PM") && getenv("TB_CONV_PM")[0] == '0';
        int AS = 0;   // patch slots: a sub-ring of AS / 4 per MMA issuer
        for (int a = 8; a >= 4 && !AS; a -= 4)
            if (pm_smem_bytes(KH, KW, a, wall) <= kSmemMax) AS = a;
        if (!pm_off && AS && nN <= ctx->num_sms && PM_BH + KH - 1 <= 256) {
            CUtensorMap mx, mw, my;
            uint64_t dims[4] = {(uint64_t)s.Cp, (uint64_t)W, (uint64_t)H, (uint64_t)B};
            uint64_t strides[3] = {(uint64_t)s.Cp * 2, (uint64_t)W * s.Cp * 2, (uint64_t)H * W * s.Cp * 2};
            uint32_t box[4] = {64, (uint32_t)conv_pw(KW), (uint32_t)(PM_BH + KH - 1), 1};
            cuuint32_t es[4] = {1, 1, 1, 1};
            int rc = make_tmap_strided(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, xn, dims, strides, box, es,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
            if (rc) return rc;
            rc = make_tmap_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wr, Cout, (uint64_t)KH * KW * s.Cp,
                              (uint64_t)KH * KW * s.Cp, 64, CONV_BN);
            if (rc) return rc;
            if (y_nhwc) {
                // NHWC output as (channel, w, h, image): the staged tile is [h][w][64 channels],
                // 128-B swizzled
                uint64_t ydims[4] = {(uint64_t)Cout, (uint64_t)s.OW, (uint64_t)s.OH, (uint64_t)B};
                uint64_t ystr[3] = {(uint64_t)Cout * 2, (uint64_t)s.OW * Cout * 2, (uint64_t)s.OH * s.OW * Cout * 2};
                uint32_t ybox[4] = {CONV_BN, CONV_BW, PM_BH, 1};
                rc = make_tmap(ctx, &my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, y, ydims, ystr, ybox,
                               CU_TENSOR_MAP_SWIZZLE_128B);
            } else {
                // NCHW output as (w, h, channel, image): the staged tile is [channel][h][w]
                uint64_t ydims[4] = {(uint64_t)s.OW, (uint64_t)s.OH, (uint64_t)Cout, (uint64_t)B};
                uint64_t ystr[3] = {(uint64_t)s.OW * 2, (uint64_t)s.OH * s.OW * 2, (uint64_t)Cout * s.OH * s.OW * 2};
                uint32_t ybox[4] = {CONV_BW, PM_BH, CONV_BN, 1};
                rc = make_tmap(ctx, &my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, y, ydims, ystr, ybox,
                               CU_TENSOR_MAP_SWIZZLE_NONE);
            }
            if (rc) return rc;
            const int smem = pm_smem_bytes(KH, KW, AS, wall);
            TB_CUDA_TRY(ctx, cudaFuncSetAttribute(conv_pm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
            const int64_t units = (int64_t)(s.OW / CONV_BW) * ((s.OH + PM_BH - 1) / PM_BH) * B * nN;
            int grid = (ctx->num_sms / nN) * nN;   // a multiple of nN: each CTA keeps one output block
            if (units < grid) grid = (int)units;
            const bool pdl_saved = ctx->pdl;
            ctx->pdl = true;
            rc = launch(ctx, "conv_pm", conv_pm_kernel, dim3(grid), dim3(PM_THREADS), smem, mx, mw, my, ep, B, s.OH, s.OW,
                        Cout, KH, KW, s.Cp, pad, AS, y_nhwc ? 1 : 0, ctx->d_err);
            ctx->pdl = pdl_saved;
            return rc;
        }
    }
    TB_REQUIRE(ctx, !y_nhwc, TB_ERR_UNSUPPORTED,
               "conv2d: NHWC y needs resident block weights (conv_pm_kernel); this shape takes conv_tc_kernel");
    const int BH = conv_bh(s.OH);
    CUtensorMap mx, mw, my;
    {
        uint64_t dims[4] = {(uint64_t)s.Cp, (uint64_t)W, (uint64_t)H, (uint64_t)B};
        uint64_t strides[3] = {(uint64_t)s.Cp * 2, (uint64_t)W * s.Cp * 2, (uint64_t)H * W * s.Cp * 2};
        uint32_t box[4] = {64, (uint32_t)conv_pw(KW), (uint32_t)(BH + KH - 1), 1};
        cuuint32_t es[4] = {1, 1, 1, 1};
        int rc = make_tmap_strided(ctx, &mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, xn, dims, strides, box, es,
                                   CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc) return rc;
        rc = make_tmap_2d(ctx, &mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, wr, Cout, (uint64_t)KH * KW * s.Cp,
                          (uint64_t)KH * KW * s.Cp, 64, CONV_BN);
        if (rc) return rc;
        // NCHW output viewed as (w, channel, h, image): the staged tile is [h][channel][w]
        uint64_t ydims[4] = {(uint64_t)s.OW, (uint64_t)Cout, (uint64_t)s.OH, (uint64_t)B};
        uint64_t ystr[3] = {(uint64_t)s.OH * s.OW * 2, (uint64_t)s.OW * 2, (uint64_t)Cout * s.OH * s.OW * 2};
        uint32_t ybox[4] = {CONV_BW, CONV_BN, (uint32_t)BH, 1};
        rc = make_tmap(ctx, &my, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, y, ydims, ystr, ybox, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (rc) return rc;
    }
    // Resident weights (all taps x chunks of one 64-channel output block) when
    // they fit beside two patch stages; otherwise a 4-slice weight ring.  Then
    // two output staging buffers (a tile's staging overlaps the previous
    // tile's store) with the deepest patch ring that fits beside them.
    const int wres = conv_smem_bytes(BH, KH, KW, 2, wall, 1) <= kSmemMax && nN <= ctx->num_sms ? 1 : 0;
    const int wslots = wres ? wall : CONV_WS;
    int AS = 2, OS = 1;   // patch slots: a half per MMA issuer, so an even count
    if (conv_smem_bytes(BH, KH, KW, 4, wslots, 2) <= kSmemMax) AS = 4, OS = 2;
    else if (conv_smem_bytes(BH, KH, KW, 2, wslots, 2) <= kSmemMax) AS = 2, OS = 2;
    const int smem = conv_smem_bytes(BH, KH, KW, AS, wslots, OS);
    TB_CUDA_TRY(ctx, cudaFuncSetAttribute(conv_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int64_t units = (int64_t)((s.OW + CONV_BW - 1) / CONV_BW) * ((s.OH + BH - 1) / BH) * B * nN;
    // resident weights: a grid that is a multiple of nN keeps each CTA on one output block
    int grid = wres ? (ctx->num_sms / nN) * nN : ctx->num_sms;
    if (units < grid) grid = (int)units;
    // The conv reads the prep kernel's outputs only after griddepcontrol.wait, so this one
    // edge may be programmatic: its CTAs start their prologue while the prep drains.
    const bool pdl_saved = ctx->pdl;
    ctx->pdl = true;
    const int rc_conv = launch(ctx, "conv_tc", conv_tc_kernel, dim3(grid), dim3(CONV_THREADS), smem, mx, mw, my, ep, B, s.OH, s.OW, Cout,
                  KH, KW, s.Cp, pad, AS, wres, BH, OS, ctx->d_err);
    ctx->pdl = pdl_saved;
    return rc_conv;
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

// Epilogue of one decode-GEMV row pair, shared by the persistent decode chain.
//
// A 256-row weight tile's outputs are handled as row pairs (p, p + 128): the
// gate / up rows of a SwiGLU tile, or dims (i, i + hd/2) of one head of a
// permuted QKV tile (qkv_perm_row).  epi_pair() loads a pair's constants once
// (scales, bias, RoPE slot and angle); epi_finish() applies the epilogue to
// one token of the pair and stores it.
#pragma once

#include "common.cuh"
#include "gemm.h"

namespace tb {

struct EpiPair {
    int p, n0, n1;
    bool in0, in1;
    float sc0, sc1, bi0, bi1;
    int kind, hd, hh, H, ri, posb;   // RoPE: kind 0 q, 1 k, 2 v, 3 no head
    float2 cs;
};

// posb: the RoPE position base (*ep.pos_ptr or ep.pos_host), read once by the
// caller.  The RoPE angle is not loaded here (epi_rope_cs).
__device__ __forceinline__ EpiPair epi_pair(const Epi& ep, int tile, int Nw, int p, int posb) {
    EpiPair k{};
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
        k.posb = posb;
        k.cs = make_float2(1.f, 0.f);
    }
    return k;
}

// The pair's RoPE (cos, sin) for a one-token-per-sequence call.
__device__ __forceinline__ float2 epi_rope_cs(const Epi& ep, const EpiPair& k) {
    if (ep.rope_tab && ep.rope_s_new == 1 && k.kind <= 1 && k.posb >= 0 && k.posb < ep.max_seq)
        return __ldg(ep.rope_tab + (int64_t)k.posb * k.hh + k.ri);
    return make_float2(1.f, 0.f);
}

__device__ __forceinline__ int epi_posb(const Epi& ep) {
    return ep.rope_tab ? (ep.pos_ptr ? __ldcg(ep.pos_ptr) : ep.pos_host) : 0;
}

// Residual of token m for the pair (bf16 output), read through L2: it may have
// been written by another CTA earlier in the same grid.
__device__ __forceinline__ void epi_resid_bf16(const Epi& ep, const EpiPair& k, int m, int Mtok, float& r0,
                                               float& r1) {
    r0 = r1 = 0.f;
    if (!ep.resid || ep.swiglu || ep.rope_tab || m >= Mtok) return;
    const unsigned short* r = reinterpret_cast<const unsigned short*>(ep.resid) + (int64_t)m * ep.ldr;
    if (k.in0) r0 = __uint_as_float((uint32_t)__ldcg(r + k.n0) << 16);
    if (k.in1) r1 = __uint_as_float((uint32_t)__ldcg(r + k.n1) << 16);
}

// (a0, a1): the pair's accumulated dot products for token m, already scaled
// by the token's 1/rms when the norm is fused.  bf16 output only.
__device__ __forceinline__ void epi_finish_bf16(const Epi& ep, const EpiPair& k, int tile, int m, float a0, float a1,
                                                float r0, float r1, int* err) {
    if (ep.rope_tab) {
        // (a0, a1) = dims (i, i + hd/2) of head slot H; rounded to bf16 first (as
        // the unfused path stores the projection), then rotated (rotate-half)
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
        if (k.kind <= 1) {
            const float2 cs = ep.rope_s_new == 1 ? k.cs : ep.rope_tab[(int64_t)pos * k.hh + k.ri];
            const float y0 = x0 * cs.x - x1 * cs.y, y1 = x1 * cs.x + x0 * cs.y;
            x0 = y0;
            x1 = y1;
        }
        __nv_bfloat16* dst;
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
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(ep.out) + (int64_t)m * ep.ldo;
    if (ep.swiglu) {
        if (k.in1) out[tile * 128 + k.p] = __float2bfloat16_rn(silu_f(a0 * k.sc0) * (a1 * k.sc1));
        return;
    }
    // acc * scale + bias, then + residual (added only when present, so -0 stays -0)
    float o0 = a0 * k.sc0 + k.bi0, o1 = a1 * k.sc1 + k.bi1;
    if (ep.resid) {
        o0 += r0;
        o1 += r1;
    }
    if (k.in0) out[k.n0] = __float2bfloat16_rn(o0);
    if (k.in1) out[k.n1] = __float2bfloat16_rn(o1);
}

}  // namespace tb

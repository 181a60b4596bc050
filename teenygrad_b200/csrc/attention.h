// Internal attention launch interface shared with the decoder executor.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "tb_internal.h"

namespace tb {

// Output addressing: element (b, h, s, d) of O lives at b*o_sb + h*o_sh + s*o_ss + d.
struct AttnOut {
    void* o;
    int64_t o_sh, o_ss, o_sb;
    float* lse;   // [B, Hq, Sq] or null
};

// Strides in elements; d is always contiguous.
struct AttnTensors {
    const void* q;
    int64_t q_sh, q_ss, q_sb;
    const void* k;
    const void* v;
    int64_t kv_sh, kv_ss, kv_sb;
    int kv_len_alloc;   // rows addressable along s (the cache capacity)
    void* o;
    int64_t o_sh, o_ss, o_sb;
    float* lse;
};

struct DecodeArgs {
    const __nv_bfloat16* q;
    int64_t q_sb, q_sh;
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    int64_t kv_sb, kv_sh, kv_ss;
    int kv_rows;           // positions allocated per (batch, kv head): [B][Hkv][kv_rows][D]
    __nv_bfloat16* o;
    int64_t o_sb, o_sh;
    float* lse;
    int Hq, Hkv;
    int len;               // context length if len_ptr is null, else added to *len_ptr
    const int* len_ptr;    // device-resident context length (CUDA-graph replay)
    float scale_log2;
    int chunk;             // keys per split (set by attn_decode_launch)
};

// f32 CUDA-core attention over strided q / k / v / o (lse [B, Hq, Sq], may be null).
int attn_f32_launch(tb_ctx* ctx, const AttnTensors& t, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale,
                    int causal);
int attn_tc_launch(tb_ctx* ctx, const AttnTensors& t, int B, int Hq, int Hkv, int Sq, int Sk, int D,
                   float scale, int causal);
// Decode attention over a KV cache of capacity >= max_len; no global scratch.
int attn_decode_launch(tb_ctx* ctx, DecodeArgs a, int B, int D, int max_len);

}  // namespace tb

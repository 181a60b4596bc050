// Persistent decode chain: several decode GEMVs of a layer in one launch
// (internal interface used by the decoder executor).
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "gemm.h"

namespace tb {

constexpr int kChainMaxPhases = 4;
constexpr int kChainMaxTiles = 128;   // 256-row weight tiles per phase
constexpr int kChainSyncWords = 4;    // [0] CTAs finished, [1] launch epoch

// One GEMV of the chain: y = epilogue(x[Mtok, K] w[Nw, K]^T), bf16 weights
// (256-row tiles, K in 64-wide blocks), bf16 output.  The epilogue is the
// decode GEMV's (residual, SwiGLU, fused RMSNorm of x, RoPE + KV write).
struct ChainStep {
    const void* x;
    int64_t x_ld;      // row stride of x (elements)
    const void* w;
    int Nw, K;
    Epi ep;
};

// Device scratch of the chain, zeroed when allocated; one chain at a time may
// use it (launches in stream order).
struct ChainScratch {
    unsigned* sync = nullptr;   // kChainSyncWords
    uint64_t* ll = nullptr;     // outputs read by later phases (flagged words)
    size_t ll_words = 0;
};

// Words of flagged-output storage for up to Mtok tokens and outputs of up to
// max_cols columns.
size_t chain_ll_words(int Mtok, int max_cols);

// Whether the chain runs this step (shape limits), without launching.
bool chain_step_ok(const ChainStep& s, int Mtok);

// Launches the chain over steps[0..n): step i + 1 reads what step i wrote.
// The first step's x comes from the previous kernel on the stream.
int chain_launch(tb_ctx* ctx, const ChainStep* steps, int n, int Mtok, const ChainScratch& scr);

}  // namespace tb

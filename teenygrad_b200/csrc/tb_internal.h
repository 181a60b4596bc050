// Host-side internals shared by the library's translation units.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>
#include <utility>

#include "../../include/teeny_b200.h"

struct tb_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;
    int* d_err = nullptr;           // device error word (bounded-wait timeouts)
    std::string last_error;
    void* comm = nullptr;           // NCCL communicator state (comm.cu)
    bool pdl = false;               // launch with programmatic stream serialization
    unsigned* chain_sync = nullptr; // tb_linear_chain_fwd scratch (allocated on first use)
    uint64_t* chain_ll = nullptr;
    size_t chain_ll_words = 0;
};

namespace tb {

int set_error(tb_ctx* ctx, int status, const char* fmt, ...);

// Records cudaGetLastError() (launch-configuration errors) into ctx.
int check_launch(tb_ctx* ctx, const char* what);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// dims/strides in elements / bytes as the driver API defines them
// (strides[0] is the stride of dim 1).  Returns 0 on success.
int make_tmap(tb_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dt, int rank, const void* base,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swz);

// As make_tmap, with per-dimension element (traversal) strides.
int make_tmap_strided(tb_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dt, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      const cuuint32_t* elem_strides, CUtensorMapSwizzle swz);

// 2-D K-major bf16/int8 operand: rows x cols (cols contiguous), box = box_cols x box_rows.
int make_tmap_2d(tb_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dt, int elem_bytes,
                 const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                 uint32_t box_cols, uint32_t box_rows);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace tb

// Workspace of the backward ops (backward.cu); tb_workspace_bytes forwards to it.
extern "C" int tb_backward_workspace_bytes(int op, int dtype, const int64_t* shape, int n_shape, size_t* bytes);

namespace tb {

// cudaLaunchKernelEx on ctx->stream; adds the programmatic-serialization
// attribute when ctx->pdl is set (the kernel must call pdl_wait()).
template <typename... KArgs, typename... Args>
int launch(tb_ctx* ctx, const char* what, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
           Args&&... args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    lc.attrs = attr;
    lc.numAttrs = 0;
    if (ctx->pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        lc.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&lc, kern, std::forward<Args>(args)...);
    if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace tb

#define TB_CUDA_TRY(ctx, call)                                                              \
    do {                                                                                    \
        cudaError_t e_ = (call);                                                            \
        if (e_ != cudaSuccess)                                                              \
            return tb::set_error((ctx), TB_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

#define TB_REQUIRE(ctx, cond, status, ...)                \
    do {                                                  \
        if (!(cond)) return tb::set_error((ctx), (status), __VA_ARGS__); \
    } while (0)

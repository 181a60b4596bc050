// Context, error reporting, workspace and TMA descriptor helpers.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>

#include "tb_internal.h"

namespace tb {

int set_error(tb_ctx* ctx, int status, const char* fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return status;
}

int check_launch(tb_ctx* ctx, const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(ctx, TB_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
    return TB_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

int make_tmap(tb_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dt, int rank, const void* base,
              const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
              CUtensorMapSwizzle swz) {
    const cuuint32_t ones[5] = {1, 1, 1, 1, 1};
    return make_tmap_strided(ctx, out, dt, rank, base, dims, strides_bytes, box, ones, swz);
}

int make_tmap_strided(tb_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dt, int rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      const cuuint32_t* elem_strides, CUtensorMapSwizzle swz) {
    EncodeTiledFn fn = get_encode_fn();
    if (!fn) return set_error(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint64_t d[5];
    cuuint64_t s[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; i++) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = elem_strides[i];
        if (i + 1 < rank) s[i] = strides_bytes[i];
    }
    CUresult r = fn(out, dt, (cuuint32_t)rank, const_cast<void*>(base), d, s, b, e,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(ctx, TB_ERR_ALIGN, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TB_OK;
}

int make_tmap_2d(tb_ctx* ctx, CUtensorMap* out, CUtensorMapDataType dt, int elem_bytes,
                 const void* base, uint64_t rows, uint64_t cols, uint64_t row_stride_elems,
                 uint32_t box_cols, uint32_t box_rows) {
    uint64_t dims[2] = {cols, rows};
    uint64_t strides[1] = {row_stride_elems * (uint64_t)elem_bytes};
    uint32_t box[2] = {box_cols, box_rows};
    return make_tmap(ctx, out, dt, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace tb

extern "C" {

int tb_abi_version(void) { return TB_ABI_VERSION; }

const char* tb_strerror(int status) {
    switch (status) {
        case TB_OK: return "ok";
        case TB_ERR_ARG: return "invalid argument";
        case TB_ERR_SHAPE: return "unsupported or inconsistent shape";
        case TB_ERR_ALIGN: return "misaligned pointer or stride";
        case TB_ERR_CUDA: return "CUDA error";
        case TB_ERR_UNSUPPORTED: return "unsupported dtype/option";
        case TB_ERR_DEVICE: return "device-side bounded wait timed out";
        case TB_ERR_NCCL: return "NCCL error";
        case TB_ERR_OOM: return "out of device memory";
        default: return "unknown status";
    }
}

const char* tb_last_error(tb_ctx* ctx) { return ctx ? ctx->last_error.c_str() : ""; }

int tb_init(tb_ctx** out, int device) {
    if (!out) return TB_ERR_ARG;
    *out = nullptr;
    tb_ctx* ctx = new tb_ctx();
    ctx->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) {
        delete ctx;
        return TB_ERR_CUDA;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
    if (major != 10 || minor != 0) {
        delete ctx;
        return TB_ERR_UNSUPPORTED;  // sm_100a binaries only
    }
    cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
    if (cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess || cudaMemset(ctx->d_err, 0, sizeof(int)) != cudaSuccess) {
        delete ctx;
        return TB_ERR_OOM;
    }
    *out = ctx;
    return TB_OK;
}

int tb_destroy(tb_ctx* ctx) {
    if (!ctx) return TB_OK;
    cudaSetDevice(ctx->device);
    if (ctx->d_err) cudaFree(ctx->d_err);
    if (ctx->chain_sync) cudaFree(ctx->chain_sync);
    if (ctx->chain_ll) cudaFree(ctx->chain_ll);
    delete ctx;
    return TB_OK;
}

int tb_set_stream(tb_ctx* ctx, void* stream) {
    if (!ctx) return TB_ERR_ARG;
    ctx->stream = reinterpret_cast<cudaStream_t>(stream);
    return TB_OK;
}

int tb_output_row_stride(int op, int dtype, int64_t row_elems, int64_t* stride) {
    if (!stride || row_elems < 0) return TB_ERR_ARG;
    const int64_t esz = dtype == TB_F32 || dtype == TB_I32 ? 4 : dtype == TB_BF16 ? 2 : dtype == TB_I8 ? 1 : 0;
    if (!esz) return TB_ERR_UNSUPPORTED;
    switch (op) {
        case TB_OP_LINEAR:
        case TB_OP_INT8_LINEAR: {
            // rows padded to 16 bytes (LinearForward::forward_output_row_stride)
            const int64_t align = 16 / esz;
            *stride = (row_elems + align - 1) / align * align;
            return TB_OK;
        }
        case TB_OP_MATMUL:
        case TB_OP_RMSNORM:
        case TB_OP_LAYERNORM:
        case TB_OP_ACT:
        case TB_OP_ATTN:
        case TB_OP_CONV2D:
        case TB_OP_QUANTIZE_INT8:
        case TB_OP_RMSNORM_BWD:
        case TB_OP_LINEAR_BWD:
        case TB_OP_ATTN_BWD:
        case TB_OP_CONV2D_BWD:
            *stride = row_elems;   // dense rows
            return TB_OK;
        default: return TB_ERR_ARG;
    }
}

int tb_workspace_bytes(int op, int dtype, const int64_t* shape, int n_shape, size_t* bytes) {
    if (!bytes) return TB_ERR_ARG;
    *bytes = 0;
    switch (op) {
        case TB_OP_CONV2D:
            // shape = {B, Cin, Cout, H, W, KH, KW, stride, pad}
            if (!shape || n_shape != 9) return TB_ERR_ARG;
            return tb_conv2d_workspace_size(dtype, (int)shape[0], (int)shape[1], (int)shape[2], (int)shape[3],
                                            (int)shape[4], (int)shape[5], (int)shape[6], (int)shape[7], (int)shape[8],
                                            bytes);
        case TB_OP_LINEAR:
        case TB_OP_INT8_LINEAR:
        case TB_OP_MATMUL:
        case TB_OP_RMSNORM:
        case TB_OP_LAYERNORM:
        case TB_OP_ACT:
        case TB_OP_ATTN:
        case TB_OP_QUANTIZE_INT8:
            return TB_OK;   // no workspace: split-K and attention splits reduce on chip
        case TB_OP_RMSNORM_BWD:
        case TB_OP_LINEAR_BWD:
        case TB_OP_ATTN_BWD:
        case TB_OP_CONV2D_BWD:
            return tb_backward_workspace_bytes(op, dtype, shape, n_shape, bytes);
        default: return TB_ERR_ARG;
    }
}

int tb_device_error(tb_ctx* ctx, int* code, int clear) {
    if (!ctx || !code) return TB_ERR_ARG;
    TB_CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream));
    TB_CUDA_TRY(ctx, cudaMemcpy(code, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (clear) TB_CUDA_TRY(ctx, cudaMemset(ctx->d_err, 0, sizeof(int)));
    return TB_OK;
}

}  // extern "C"

/*
 * teeny_b200.h -- C ABI of the B200 (sm_100a) kernels behind teenygrad's
 * operator surface.
 *
 * Every entry point takes device pointers and plain sizes, enqueues work on the
 * context's stream (no implicit synchronisation) and returns a tb_status.  The
 * reference executes one RuntimeOp per graph node: it packs kernel arguments
 * (RuntimeOp::pack_args, core/teeny-core/src/model/mod.rs:145), computes a grid
 * (RuntimeOp::grid, model/mod.rs:156) and launches teenyc-compiled PTX through
 * CudaDevice::launch (drivers/teeny-cuda/src/device/mod.rs:315-385), then
 * synchronises.  A RuntimeOp implementation in drivers/teeny-cuda calls the
 * matching tb_* function instead of pack_args + cuLaunchKernel; each function
 * below names the reference kernel whose RuntimeOp it replaces.
 *
 * Layouts are the reference's: row-major, contiguous, PyTorch weight layout
 * ([out, in]) for linear layers, NCHW for convolutions.
 */
#ifndef TEENY_B200_H
#define TEENY_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_ABI_VERSION 1

#if defined(__GNUC__)
#define TB_API __attribute__((visibility("default")))
#else
#define TB_API
#endif

typedef struct tb_ctx tb_ctx;

typedef enum tb_status {
    TB_OK = 0,
    TB_ERR_ARG = 1,         /* null pointer / bad enum */
    TB_ERR_SHAPE = 2,       /* unsupported or inconsistent sizes */
    TB_ERR_ALIGN = 3,       /* pointer or row stride not 16-byte aligned */
    TB_ERR_CUDA = 4,        /* CUDA runtime error (tb_last_error has the text) */
    TB_ERR_UNSUPPORTED = 5, /* dtype / option combination not implemented */
    TB_ERR_DEVICE = 6,      /* a kernel reported a bounded-wait timeout */
    TB_ERR_NCCL = 7,        /* NCCL failure or timeout */
    TB_ERR_OOM = 8          /* device allocation failed */
} tb_status;

typedef enum tb_dtype { TB_F32 = 0, TB_BF16 = 1, TB_I8 = 2, TB_I32 = 3 } tb_dtype;

typedef enum tb_act {
    TB_ACT_NONE = -1,
    TB_ACT_SILU = 0,      /* silu_forward, nn/activation/sigmoid.rs:120-156 */
    TB_ACT_GELU_TANH = 1, /* gelu_forward, nn/activation/gelu.rs:32-75 */
    TB_ACT_RELU = 2,      /* relu_forward, nn/activation/relu.rs:28 */
    TB_ACT_SIGMOID = 3    /* sigmoid_forward, nn/activation/sigmoid.rs */
} tb_act;

/* Epilogue flags for the linear layers. */
#define TB_EPI_BIAS 1     /* + bias[N] (f32) */
#define TB_EPI_RESIDUAL 2 /* + residual[M,N] (same dtype as y) */
#define TB_EPI_SWIGLU 4   /* y[:, j] = silu(acc[:, gate j]) * acc[:, up j]; W rows interleaved
                             in blocks of 128 (gate block, up block), y has N/2 columns */
#define TB_EPI_OUT_F32 8  /* write y as f32 instead of the input dtype */

/* ------------------------------------------------------------ context --- */
TB_API int tb_init(tb_ctx** out, int device);
TB_API int tb_destroy(tb_ctx* ctx);
/* stream is a cudaStream_t (NULL = legacy default stream). */
TB_API int tb_set_stream(tb_ctx* ctx, void* stream);
TB_API const char* tb_strerror(int status);
TB_API const char* tb_last_error(tb_ctx* ctx);
/* Synchronises the stream and reads the device error word that bounded waits
 * set (0 = none); clears it when `clear` is non-zero. */
TB_API int tb_device_error(tb_ctx* ctx, int* code, int clear);
TB_API int tb_abi_version(void);
/* Failure-path self-test (no counterpart in the reference, which has no
 * device-side waits).  Launches two CTAs that wait on an mbarrier nothing
 * arrives on: CTA 0 with a limit of limit_us, CTA 1 with the kernels' normal
 * limit (seconds).  CTA 0 gives up and flags the device error word; CTA 1
 * must then return early.  elapsed_ns: device memory for 2 values, each CTA's
 * time until it gave up.  Afterwards tb_device_error reports the timeout bit
 * and the context stays usable. */
TB_API int tb_selftest_bounded_wait(tb_ctx* ctx, int limit_us, unsigned long long* elapsed_ns);

/* -------------------------------------------------------------- norms --- */
/* rms_norm_forward (kernels/teeny-kernels/src/nn/norm/rmsnorm.rs:40-122):
 * y = x * rsqrt(mean(x^2) + eps) * w, rrms[M] optional (may be NULL).
 * dtype TB_F32 or TB_BF16 for x, w, y; math in f32. */
TB_API int tb_rmsnorm_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, void* y, float* rrms,
                   int64_t M, int64_t N, float eps);

/* layer_norm_forward_inference (nn/norm/layernorm.rs:43-157). */
TB_API int tb_layernorm_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const void* b, void* y,
                     int64_t M, int64_t N, float eps);

/* -------------------------------------------------------- elementwise --- */
/* silu / gelu(tanh) / relu / sigmoid forward over n elements. */
TB_API int tb_act_fwd(tb_ctx* ctx, int act, int dtype, const void* x, void* y, int64_t n);
/* SwiGLU: y = silu(gate) * up (silu_forward + elemwise_mul_forward,
 * nn/tensor/elemwise_binary.rs:189, fused). */
TB_API int tb_swiglu_fwd(tb_ctx* ctx, int dtype, const void* gate, const void* up, void* y, int64_t n);
/* elemwise_add_forward (nn/tensor/elemwise_add.rs:29). */
TB_API int tb_add_fwd(tb_ctx* ctx, int dtype, const void* a, const void* b, void* y, int64_t n);

/* --------------------------------------------------- allocation queries --- */
/* Operator ids for the queries below. */
typedef enum tb_op {
    TB_OP_LINEAR = 0, TB_OP_MATMUL = 1, TB_OP_INT8_LINEAR = 2, TB_OP_RMSNORM = 3, TB_OP_LAYERNORM = 4,
    TB_OP_ACT = 5, TB_OP_ATTN = 6, TB_OP_CONV2D = 7, TB_OP_QUANTIZE_INT8 = 8,
    TB_OP_RMSNORM_BWD = 9, TB_OP_LINEAR_BWD = 10, TB_OP_ATTN_BWD = 11, TB_OP_CONV2D_BWD = 12
} tb_op;
/* Row stride (elements) an executor should allocate for an op's output rows
 * of row_elems elements: RuntimeOp::forward_output_row_stride
 * (core/teeny-core/src/model/mod.rs:100-115); for linear layers the
 * reference pads rows to 16 bytes (LinearForward, nn/mlp/linear.rs:267-272),
 * every other op writes dense rows.  Needs no GPU. */
TB_API int tb_output_row_stride(int op, int dtype, int64_t row_elems, int64_t* stride);
/* Device workspace an op needs, in bytes.  shape: TB_OP_CONV2D {B, Cin,
 * Cout, H, W, KH, KW, stride, pad} (bf16 tensor-core path only);
 * TB_OP_RMSNORM_BWD {M, N}; TB_OP_LINEAR_BWD {M, N, K}; TB_OP_ATTN_BWD
 * {B, Hq, Sq}; ignored for the others (no workspace).  Needs no GPU. */
TB_API int tb_workspace_bytes(int op, int dtype, const int64_t* shape, int n_shape, size_t* bytes);

/* ------------------------------------------------------------- linear --- */
/* linear_forward (nn/mlp/linear.rs:22-117; LinearForward RuntimeOp :251-388):
 * y[M, N] = x[M, K] * w[N, K]^T (+ bias) (+ residual), epilogue per `flags`.
 * TB_BF16: tcgen05 tensor cores, f32 accumulate (K % 8 == 0, N % 8 == 0).
 * TB_F32: f32 CUDA-core path (exact f32 accumulate). */
TB_API int tb_linear_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias,
                  const void* residual, void* y, int64_t M, int64_t N, int64_t K, int flags);
/* The same with row strides, as LinearForward's pack_args passes them
 * (nn/mlp/linear.rs:274-300: stride_xm, and stride_ym = the padded
 * output_row_stride): x rows ldx >= K elements apart, y rows (and the
 * residual's) ldy >= N (N / 2 with SwiGLU) apart.  TB_BF16 needs ldx and ldy
 * multiples of 8; columns of y past N are not written. */
TB_API int tb_linear_fwd_strided(tb_ctx* ctx, int dtype, const void* x, int64_t ldx, const void* w,
                                 const float* bias, const void* residual, void* y, int64_t ldy, int64_t M,
                                 int64_t N, int64_t K, int flags);

/* A chain of dependent decode linear layers in one persistent launch: step
 * i + 1 may read what step i wrote (e.g. a layer's output projection with its
 * residual, gate/up with the RMSNorm fused and SwiGLU, then down with its
 * residual).  No counterpart in the reference, whose executor launches one
 * kernel per op (drivers/teeny-cuda/src/model/mod.rs:524-700); each step has
 * linear_forward's semantics (nn/mlp/linear.rs:22-117), plus an optional
 * RMSNorm of x (rmsnorm.rs:19-134, gains norm_w) fused in front.
 * bf16 only; M <= 64 tokens; N % 256 == 0 (N <= 32768) and K % 64 == 0;
 * ldx, ldy multiples of 8 elements; at most TB_LINEAR_CHAIN_MAX steps.
 * flags: TB_EPI_RESIDUAL (residual rows ldy apart; may alias y) and / or
 * TB_EPI_SWIGLU (w rows interleaved as for tb_linear_fwd; y has N / 2 columns).
 * Its split-K reduction uses ctx scratch memory allocated on the first call. */
#define TB_LINEAR_CHAIN_MAX 4
typedef struct tb_linear_step {
    const void* x;      /* bf16 [M, K], rows ldx apart */
    int64_t ldx;
    const void* w;      /* bf16 [N, K] */
    const void* norm_w; /* bf16 [K] RMSNorm gains, or NULL: no norm */
    float norm_eps;
    const void* residual;
    void* y;            /* bf16 [M, N] (N / 2 with SwiGLU), rows ldy apart */
    int64_t ldy;
    int64_t N, K;
    int flags;
} tb_linear_step;
TB_API int tb_linear_chain_fwd(tb_ctx* ctx, const tb_linear_step* steps, int n_steps, int64_t M);

/* matmul_forward (math/gemm.rs:44-105; MatMulRuntimeOp gemm.rs:232):
 * c[M, N] = a[M, K] * b[K, N]. */
TB_API int tb_matmul_fwd(tb_ctx* ctx, int dtype, const void* a, const void* b, void* c, int64_t M,
                  int64_t N, int64_t K);

/* --------------------------------------------------------------- int8 --- */
/* quantize_affine, symmetric per output channel, 8 bits
 * (utilities/teeny-quant/src/quant/affine.rs:55-148): bit-exact.
 * w f32 [N, K] -> q int8 [N, K], scale f32 [N]. */
TB_API int tb_quantize_int8(tb_ctx* ctx, const float* w, int8_t* q, float* scale, int64_t N, int64_t K);
/* Same, reading bf16 weights (upcast exactly, as teeny-quant's read_f32). */
TB_API int tb_quantize_int8_bf16(tb_ctx* ctx, const void* w_bf16, int8_t* q, float* scale, int64_t N,
                          int64_t K);
/* dequantize_affine (affine.rs:151-159): w = q * scale[n]. */
TB_API int tb_dequantize_int8(tb_ctx* ctx, const int8_t* q, const float* scale, float* w, int64_t N,
                       int64_t K);
/* int8 weight-only linear (the op graph/mod.rs:2595-2600 leaves as TODO):
 * y[M, N] = scale[n] * x[M, K](bf16) * q[N, K]^T (+ residual), bf16 out unless
 * TB_EPI_OUT_F32.  Tensor cores: the int8 weights are converted exactly to
 * bf16 straight into tensor memory, which the MMA reads as its A operand. */
TB_API int tb_int8_linear_fwd(tb_ctx* ctx, const void* x, const int8_t* q, const float* scale,
                       const void* residual, void* y, int64_t M, int64_t N, int64_t K, int flags);

/* ---------------------------------------------------------- attention --- */
/* flash_attention2_forward (nn/attention/flash_attn2.rs:53-158) extended with
 * causal masking and GQA.  q [B, Hq, Sq, D], k/v [B, Hkv, Sk, D],
 * o [B, Hq, Sq, D], lse [B, Hq, Sq] f32 (natural log of the scaled scores'
 * sum of exps; may be NULL).  Causal: query i sees key j iff
 * j <= i + (Sk - Sq).  TB_BF16 runs on tcgen05 (D = 64 or 128);
 * TB_F32 on CUDA cores (D <= 128). */
TB_API int tb_attn_fwd(tb_ctx* ctx, int dtype, const void* q, const void* k, const void* v, void* o,
                float* lse, int B, int Hq, int Hkv, int Sq, int Sk, int D, float scale, int causal);

/* --------------------------------------------------------------- conv --- */
/* conv2d_bias_forward (nn/conv/conv2d.rs:643-764; Conv2dBiasForward RuntimeOp
 * :766-820; the inference fusion of graph/mod.rs:845-918) with the folded-BN
 * epilogue of nn/fused/conv2d_bn_silu.rs:141-170:
 *   y = act(scale[co] * (conv(x, w) [+ bias[co] if shift is NULL]) + shift[co])
 * NCHW x [B, Cin, H, W], w [Cout, Cin, KH, KW], y [B, Cout, OH, OW], groups = 1,
 * zero padding.  bias / bn_scale / bn_shift are f32 [Cout] and may be NULL
 * (scale 1, shift 0).  act: TB_ACT_NONE, TB_ACT_RELU or TB_ACT_SILU.
 * TB_BF16 with stride 1 and OW % 8 == 0 runs as a tcgen05 implicit GEMM and
 * needs a workspace of tb_conv2d_workspace_size() bytes (NHWC copy of x,
 * reordered weights); other bf16 shapes and TB_F32 run on CUDA cores with f32
 * accumulation and need none. */
TB_API int tb_conv2d_workspace_size(int dtype, int B, int Cin, int Cout, int H, int W, int KH, int KW, int stride,
                                    int pad, size_t* bytes);
TB_API int tb_conv2d_fwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias,
                         const float* bn_scale, const float* bn_shift, void* y, int B, int Cin, int Cout, int H,
                         int W, int KH, int KW, int stride, int pad, int act, void* workspace,
                         size_t workspace_bytes);
/* Layout options of tb_conv2d_fwd_ex for an executor that chains convolutions
 * (the reference's NCHW API is flags = 0, i.e. tb_conv2d_fwd).  The NCHW ->
 * NHWC copy of x and the weight reorder that the tensor-core path otherwise
 * makes in its workspace, in a launch of their own, are skipped when the
 * caller already holds those layouts:
 *   TB_CONV_X_NHWC   x is [B, H, W, Cin]
 *   TB_CONV_W_PACKED w is [Cout, KH, KW, Cin] (tb_conv2d_pack_weights)
 *   TB_CONV_Y_NHWC   y is written [B, OH, OW, Cout]
 * The options need TB_BF16, Cin % 8 == 0 and the tensor-core path (stride 1,
 * OW % 8 == 0); TB_CONV_Y_NHWC also needs Cout % 8 == 0 and a shape whose block
 * weights stay resident (3 x 3 and 1 x 1 filters at <= 64 input channels, as the
 * C2 stage).  Other shapes return TB_ERR_UNSUPPORTED.  The workspace may be NULL
 * when both TB_CONV_X_NHWC and TB_CONV_W_PACKED are given. */
#define TB_CONV_X_NHWC 1
#define TB_CONV_Y_NHWC 2
#define TB_CONV_W_PACKED 4
TB_API int tb_conv2d_fwd_ex(tb_ctx* ctx, int dtype, const void* x, const void* w, const float* bias,
                            const float* bn_scale, const float* bn_shift, void* y, int B, int Cin, int Cout, int H,
                            int W, int KH, int KW, int stride, int pad, int act, int flags, void* workspace,
                            size_t workspace_bytes);
/* w [Cout, Cin, KH, KW] -> w_packed [Cout, KH, KW, Cin] (bf16, Cin % 8 == 0), the
 * weight layout TB_CONV_W_PACKED takes; done once per weight tensor. */
TB_API int tb_conv2d_pack_weights(tb_ctx* ctx, int dtype, const void* w, void* w_packed, int Cout, int Cin, int KH,
                                  int KW);
/* BN folding (nn/fused/conv2d_bn_silu.rs:33-35): scale = gamma / sqrt(var + eps),
 * shift = beta - scale * mean (+ scale * bias when bias is given).  f32 [C]. */
TB_API int tb_bn_fold(tb_ctx* ctx, const float* gamma, const float* beta, const float* mean, const float* var,
                      const float* bias, float eps, float* scale, float* shift, int C);
/* batch_norm_2d_nchw_forward_inference (nn/norm/batchnorm.rs:574-686):
 * y = (x - mean[c]) * rsqrt(var[c] + eps) * gamma[c] + beta[c], x [B, C, HW]. */
TB_API int tb_batchnorm_fwd(tb_ctx* ctx, int dtype, const void* x, const float* gamma, const float* beta,
                            const float* mean, const float* var, void* y, int64_t B, int64_t C, int64_t HW,
                            float eps);

/* ----------------------------------------------------------- backward --- */
/* Gradients for the reference's training executor (LoadedModel::backward,
 * drivers/teeny-cuda/src/model/mod.rs:963).  dtype TB_F32 or TB_BF16 for the
 * tensors; f32 math; deterministic (fixed-order reductions, no atomics). */

/* rms_norm_backward (nn/norm/rmsnorm.rs:125-277): dx[m,n] = rrms[m] *
 * (w[n] dy[m,n] - x[m,n] rrms[m]^2 sum_n(dy w x) / N); dw (f32 [N], may be
 * NULL) accumulates sum_m dy x rrms, as the reference's dweight does.  rrms
 * is the forward's f32 [M] output.  Workspace: tb_workspace_bytes
 * (TB_OP_RMSNORM_BWD, {M, N}) when dw is given. */
TB_API int tb_rmsnorm_bwd(tb_ctx* ctx, int dtype, const void* dy, const void* x, const void* w, const float* rrms,
                          void* dx, float* dw, int64_t M, int64_t N, void* workspace, size_t workspace_bytes);
/* linear_backward (nn/mlp/linear.rs:119-249) of y = x w^T + b: dx = dy w
 * [M, K], dw = dy^T x [N, K] (dtype; either may be NULL), db = sum_m dy
 * (f32 [N], may be NULL).  TB_BF16 on the tensor cores (M, N, K multiples of
 * 8); TB_F32 exact.  Workspace: TB_OP_LINEAR_BWD {M, N, K}. */
TB_API int tb_linear_bwd(tb_ctx* ctx, int dtype, const void* x, const void* w, const void* dy, void* dx, void* dw,
                         float* db, int64_t M, int64_t N, int64_t K, void* workspace, size_t workspace_bytes);
/* flash_attention2_backward_dq / _dkv (nn/attention/flash_attn2.rs:160-447)
 * with the forward's causal mask and GQA: dq [B, Hq, Sq, D], dk / dv
 * [B, Hkv, Sk, D] (summed over each kv head's query heads).  o and lse are
 * the forward's outputs (lse f32 [B, Hq, Sq]).  D <= 128.  Workspace:
 * TB_OP_ATTN_BWD {B, Hq, Sq}. */
TB_API int tb_attn_bwd(tb_ctx* ctx, int dtype, const void* q, const void* k, const void* v, const void* o,
                       const void* dout, const float* lse, void* dq, void* dk, void* dv, int B, int Hq, int Hkv, int Sq,
                       int Sk, int D, float scale, int causal, void* workspace, size_t workspace_bytes);
/* conv2d_backward (nn/conv/conv2d.rs:395-521), groups = 1, zero padding:
 * dx [B, Cin, H, W] and dw [Cout, Cin, KH, KW] (either may be NULL), both
 * written (not accumulated).  KH * KW <= 49.  No workspace. */
TB_API int tb_conv2d_bwd(tb_ctx* ctx, int dtype, const void* dy, const void* x, const void* w, void* dx, void* dw,
                         int B, int Cin, int Cout, int H, int W, int KH, int KW, int stride, int pad);

/* ------------------------------------------------------------ decoder --- */
/* RoPE, rotate-half pairing (d, d + D/2), inv_freq = theta^(-2i/D).
 * x, y [T, H, D] (may alias), pos [T] int32. */
TB_API int tb_rope_fwd(tb_ctx* ctx, int dtype, const void* x, const int32_t* pos, void* y, int64_t T,
                int H, int D, float theta);
/* Embedding gather: y[t, :] = table[ids[t], :]. */
TB_API int tb_embedding_fwd(tb_ctx* ctx, int dtype, const void* table, const int32_t* ids, void* y,
                     int64_t T, int64_t D, int64_t vocab);
/* Row argmax; the lowest index wins ties, NaN never wins. x [M, N]. */
TB_API int tb_argmax_fwd(tb_ctx* ctx, int dtype, const void* x, int32_t* out, int64_t M, int64_t N);

/* Row argmax that allocates nothing.  No counterpart in the reference.
 * Same result as tb_argmax_fwd (lowest index on ties, NaN never wins), from a
 * split-row kernel whose cross-block reduction state lives in a static device
 * array, so the call needs no workspace from the caller and never calls
 * cudaMalloc/cudaFree: for callers that cannot allocate device memory, such as
 * a serving loop whose device memory belongs to an external pool.  At most
 * TB_ARGMAX_NOALLOC_MAX_ROWS rows per call (larger M returns TB_ERR_SHAPE).
 * The array (64 KiB) stays resident on every GPU that loads the library until
 * the process exits.  The first call on a device looks up the array's device
 * address and caches it for the life of the process.  All calls share
 * the array: calls that overlap on the GPU (two streams or two host threads
 * at once) race.  dtype TB_F32 or TB_BF16. */
#define TB_ARGMAX_NOALLOC_MAX_ROWS 4096
TB_API int tb_argmax_noalloc_fwd(tb_ctx* ctx, int dtype, const void* x, int32_t* out, int64_t M, int64_t N);

/* ------------------------------------------------------ decoder model --- */
/* A Llama-style decoder assembled from the ops above (the reference's
 * teeny-llm is a placeholder, apps/teeny-llm/src/server/main.rs:6-8, and its
 * graph lowering lacks attention/RoPE/gather, kernels/teeny-kernels/src/graph/
 * mod.rs:2472-2530).  It plays the role of LoadedModel (drivers/teeny-cuda/
 * src/model/mod.rs:231-700): it owns the parameters, a KV cache and every
 * activation buffer (allocated once at create, not per forward), runs prefill
 * stream-ordered without per-op synchronisation, and replays decode steps as
 * captured CUDA graphs (capture_graph, model/mod.rs:1245): one step per
 * tb_decoder_decode_step, eight steps per replay inside tb_decoder_generate.
 * Pre-norm blocks: x += Wo attn(rope(Wqkv rmsnorm(x))); x += Wdown swiglu(
 * Wgate/up rmsnorm(x)); logits = lm_head rmsnorm(x_last); greedy argmax. */
typedef struct tb_decoder tb_decoder;

typedef struct tb_decoder_config {
    int n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn_hidden, vocab;
    float rope_theta, norm_eps;
    int max_batch;          /* sequences per call */
    int max_seq;            /* KV-cache capacity per sequence (prompt + generated) */
    int max_prefill_tokens; /* activation rows for prefill (0: max_batch * max_seq) */
    int weights_int8;       /* 1: linear layers use int8 weight-only GEMV (tokens per call <= 64) */
} tb_decoder_config;

enum tb_param_kind {
    TB_P_EMBED = 0,      /* [vocab, d] */
    TB_P_ATTN_NORM = 1,  /* [d] per layer */
    TB_P_WQ = 2,         /* [Hq*hd, d] */
    TB_P_WK = 3,         /* [Hkv*hd, d] */
    TB_P_WV = 4,         /* [Hkv*hd, d] */
    TB_P_WO = 5,         /* [d, Hq*hd] */
    TB_P_MLP_NORM = 6,   /* [d] */
    TB_P_W_GATE = 7,     /* [F, d] */
    TB_P_W_UP = 8,       /* [F, d] */
    TB_P_W_DOWN = 9,     /* [d, F] */
    TB_P_FINAL_NORM = 10,/* [d] */
    TB_P_LM_HEAD = 11    /* [vocab, d] */
};

TB_API int tb_decoder_create(tb_ctx* ctx, const tb_decoder_config* cfg, tb_decoder** out);
TB_API int tb_decoder_destroy(tb_decoder* dec);
/* Copies one parameter (f32 or bf16, host or device memory, row-major in the
 * PyTorch layout listed above) into the decoder's own layout. */
TB_API int tb_decoder_set_param(tb_decoder* dec, int layer, int kind, const void* src, int src_dtype,
                                int src_on_host);
/* Copies one int8 weight with its per-output-channel f32 scales, as
 * teeny-quant stores them (I8 [rows, cols] + F32 `_scale` [rows],
 * utilities/teeny-quant/src/format.rs:145-182), into the int8 GEMV layout
 * without re-quantising.  Linear kinds need a weights_int8 decoder;
 * TB_P_EMBED is dequantised (q * scale) into the bf16 gather table. */
TB_API int tb_decoder_set_param_int8(tb_decoder* dec, int layer, int kind, const int8_t* q, const float* scale,
                                     int src_on_host);
/* Fills every parameter from a counter-based N(0, std) generator (norm
 * weights = 1).  Deterministic in seed. */
TB_API int tb_decoder_init_random(tb_decoder* dec, uint64_t seed, float std);
/* Call after the parameters are set: quantises the linear layers when
 * weights_int8 is set (tb_quantize_int8 semantics, bit-exact). */
TB_API int tb_decoder_prepare(tb_decoder* dec);
/* Prefill B prompts of S tokens (ids: device int32 [B, S]).  Resets the KV
 * cache, writes the first greedy token.  logits (device f32 [B, vocab]) and
 * next_ids (device int32 [B]) may be NULL. */
TB_API int tb_decoder_prefill(tb_decoder* dec, const int32_t* ids, int B, int S, float* logits,
                              int32_t* next_ids);
/* One decode step for the B sequences of the last prefill: consumes ids
 * (device int32 [B], NULL = the previous step's greedy tokens), appends to the
 * KV cache, writes logits / next_ids (either may be NULL). */
TB_API int tb_decoder_decode_step(tb_decoder* dec, const int32_t* ids, float* logits, int32_t* next_ids);
/* Prefill + (n_new - 1) graph-replayed greedy decode steps; out_ids is device
 * int32 [B, n_new]. */
TB_API int tb_decoder_generate(tb_decoder* dec, const int32_t* prompt_ids, int B, int S, int n_new,
                               int32_t* out_ids);
/* Decode-only workloads: fill the KV cache of B sequences with len positions
 * of N(0, 1) keys/values and set the current tokens (device int32 [B]). */
TB_API int tb_decoder_fill_kv_random(tb_decoder* dec, int B, int len, uint64_t seed, const int32_t* ids);
/* Copies cache positions [0, len) of the first B sequences of one layer into
 * device bf16 buffers k_out / v_out [B, n_kv_heads, len, head_dim]
 * (stream-ordered).  Inspection / session save; the reference has no KV cache. */
TB_API int tb_decoder_read_kv(tb_decoder* dec, int layer, int B, int len, void* k_out, void* v_out);
/* Tokens currently in the KV cache per sequence. */
TB_API int tb_decoder_seq_len(tb_decoder* dec, int* len);

/* --------------------------------------------------------- checkpoints --- */
/* safetensors files (memory-mapped, read in place), as the reference's
 * loader reads them (utilities/teeny-data/src/safetensors/mod.rs:22-45).
 * Host code only: needs no GPU. */
typedef struct tb_st tb_st;
TB_API int tb_st_open(const char* path, tb_st** out);
TB_API int tb_st_close(tb_st* st);
/* Number of tensors, and the i-th name in header order. */
TB_API int tb_st_count(tb_st* st);
TB_API const char* tb_st_name(tb_st* st, int i);
/* dtype: TB_F32 / TB_BF16 / TB_I8 / TB_I32, or -1 for other safetensors
 * dtypes; *rank in: capacity of shape, out: the tensor's rank; data points
 * into the mapping (valid until tb_st_close).  Any output may be NULL. */
TB_API int tb_st_tensor(tb_st* st, const char* name, int* dtype, int64_t* shape, int* rank, const void** data,
                        size_t* bytes);
/* A "__metadata__" value (e.g. teeny-quant's "quantization_config" JSON), or NULL. */
TB_API const char* tb_st_metadata(tb_st* st, const char* key);
/* Loads a Llama-layout checkpoint (model.embed_tokens.weight,
 * model.layers.N.{input_layernorm, self_attn.{q,k,v,o}_proj,
 * post_attention_layernorm, mlp.{gate,up,down}_proj}.weight, model.norm.weight,
 * lm_head.weight, tied to the embedding when absent) into the decoder, then
 * prepares it.  F32 / BF16 tensors go through tb_decoder_set_param; I8 tensors
 * with a `<name>_scale` (teeny-quant symmetric per-channel int8) through
 * tb_decoder_set_param_int8. */
TB_API int tb_decoder_load_safetensors(tb_decoder* dec, tb_st* st);

/* ------------------------------------------------------ graph executor --- */
/* The counterpart of LoadedModel::forward (drivers/teeny-cuda/src/model/
 * mod.rs:524-700) for a whole lowered DAG: nodes named after the reference's
 * graph ops (kernels/teeny-kernels/src/graph/mod.rs), shapes inferred as
 * nodes are added, every input and intermediate planned once into one
 * device arena by liveness (tb_graph_plan allocates it; runs allocate
 * nothing), node launches stream-ordered on the context's stream with no
 * synchronisation, optionally captured once into a CUDA graph and replayed.
 * Parameters stay in the caller's device memory. */
typedef struct tb_graph tb_graph;

typedef enum tb_graph_op {
    TB_G_LINEAR = 0,    /* x [.., K], w [N, K] (+ f32 bias [N], + residual [.., N]; pass -1 to skip) */
    TB_G_MATMUL = 1,    /* a [.., K], b [K, N] */
    TB_G_RMSNORM = 2,   /* x [.., N], w [N]; eps   (the reference's RuntimeOp is a stub, graph/mod.rs:454) */
    TB_G_LAYERNORM = 3, /* x [.., N], w [N], b [N]; eps */
    TB_G_ACT = 4,       /* x; act (tb_act) */
    TB_G_ADD = 5,       /* a, b */
    TB_G_SWIGLU = 6,    /* gate, up: silu(gate) * up (Silu + Mul fused) */
    TB_G_ATTENTION = 7, /* q [B, S, heads * D], k / v [B, S, kv_heads * D], or one fused qkv
                           [B, S, (heads + 2 kv_heads) * D] -> [B, S, heads * D], read in place;
                           heads, kv_heads, causal, scale (0: 1/sqrt(D)) (TODO in the reference, :2477) */
    TB_G_ROPE = 8,      /* x [T, H, D], positions int32 [T]; theta (0: 10000) (TODO :2472) */
    TB_G_GATHER = 9,    /* table [V, D], ids int32 [..] -> [.., D] (TODO :2527) */
    TB_G_ARGMAX = 10,   /* x [.., N] -> int32 [..] (TODO :2250) */
    TB_G_CONV2D = 11,   /* x [B, C, H, W], w [Co, C, KH, KW] (+ f32 bias, bn scale, bn shift [Co]; -1 skips);
                           stride, pad, act (TB_ACT_NONE = -1 for none) */
    TB_G_BATCHNORM = 12 /* x [B, C, ..], gamma, beta, mean, var f32 [C]; eps */
} tb_graph_op;

typedef struct tb_node_attr {
    float eps;        /* norms */
    int act;          /* TB_G_ACT, TB_G_CONV2D: a tb_act */
    int heads, kv_heads, causal;
    float scale;      /* attention softmax scale, 0: 1 / sqrt(head dim) */
    float theta;      /* RoPE base, 0: 10000 */
    int stride, pad;  /* conv2d */
} tb_node_attr;

TB_API int tb_graph_create(tb_ctx* ctx, tb_graph** out);
TB_API int tb_graph_destroy(tb_graph* g);
/* A graph input (written before each run into its planned buffer, whose
 * pointer tb_graph_tensor_ptr returns after tb_graph_plan). */
TB_API int tb_graph_input(tb_graph* g, int dtype, int rank, const int64_t* shape, int* id);
/* A parameter in the caller's device memory (not copied). */
TB_API int tb_graph_param(tb_graph* g, int dtype, int rank, const int64_t* shape, const void* dev_ptr, int* id);
/* Appends a node; inputs are tensor ids (-1 for skipped optional inputs);
 * attr may be NULL; *out_id is the node's output tensor. */
TB_API int tb_graph_node(tb_graph* g, int op, const int* inputs, int n_inputs, const tb_node_attr* attr, int* out_id);
/* Keeps a tensor's buffer for reading after the run (tensors nothing consumes are kept anyway). */
TB_API int tb_graph_mark_output(tb_graph* g, int id);
/* Plans the arena and allocates it (the only allocation); capture = 1
 * records the node launches into a CUDA graph at the first run and replays it. */
TB_API int tb_graph_plan(tb_graph* g, int capture);
TB_API int tb_graph_arena_bytes(tb_graph* g, size_t* bytes);
/* Device pointer of a tensor (inputs, outputs, intermediates: in the arena). */
TB_API int tb_graph_tensor_ptr(tb_graph* g, int id, void** ptr);
/* Stream-ordered copies into / out of a planned tensor's buffer (host or
 * device memory on the other side; bytes must be the tensor's size). */
TB_API int tb_graph_write(tb_graph* g, int id, const void* src, size_t bytes);
TB_API int tb_graph_read(tb_graph* g, int id, void* dst, size_t bytes);
/* Enqueues every node on the context's stream (no synchronisation). */
TB_API int tb_graph_run(tb_graph* g);

/* ---------------------------------------------------------- multi-GPU --- */
/* Batch-sharded runs: one process per GPU, each on its own shard; the only
 * exchange is an all-gather of the final outputs (the reference has no
 * distributed code at all).  NCCL is loaded at run time (libnccl.so.2).  The
 * communicator is non-blocking and every host-side wait on it is bounded by
 * timeout_ms, after which it is aborted and TB_ERR_NCCL returned. */
TB_API int tb_comm_unique_id_bytes(void);
/* Rank 0 creates the id and shares its bytes with the other ranks. */
TB_API int tb_comm_get_unique_id(void* out);
TB_API int tb_comm_init(tb_ctx* ctx, const void* unique_id, int nranks, int rank, int timeout_ms);
/* recv[r * bytes_per_rank ...] = rank r's send buffer, on ctx's stream. */
TB_API int tb_comm_allgather(tb_ctx* ctx, const void* send, void* recv, size_t bytes_per_rank);
TB_API int tb_comm_abort(tb_ctx* ctx);
TB_API int tb_comm_destroy(tb_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* TEENY_B200_H */

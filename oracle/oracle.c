/*
 * CPU oracle for the teenygrad hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic of the teenygrad kernels that
 * the B200 library replaces.  It is the checker the parity tests compare the
 * CUDA path against, and the timed CPU baseline of bench.py.  Nothing in the
 * product library (teenygrad_b200/) links, loads or calls it.
 *
 * Parity pinning: the reference's own golden vectors (its PyTorch-generated
 * fixtures, copied under tests/golden/) pin rmsnorm, layernorm, silu, gelu,
 * relu, sigmoid, linear, conv2d, batchnorm and non-causal attention.  The int8
 * quantiser has no golden bytes in the reference; it is pinned by formula and
 * by an independent numpy restatement.  bf16 rounding, causal masking, GQA,
 * RoPE and the decoder composition have no reference test at all ("parity
 * unpinned" for those rows; the oracle defines them and torch CPU cross-checks).
 *
 * Conventions: row-major, contiguous.  All accumulation is done in double and
 * rounded to float once, so the oracle is at least as accurate as any fp32
 * kernel it checks.  "bf16" arrays are passed as uint16_t bit patterns.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- bf16 --- */

/* Round-to-nearest-even f32 -> bf16, as half::bf16::from_f32 (half 2.7.1). */
uint16_t or_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

float or_bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

void or_f32_to_bf16_array(const float* x, uint16_t* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = or_f32_to_bf16(x[i]);
}

void or_bf16_to_f32_array(const uint16_t* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = or_bf16_to_f32(x[i]);
}

int or_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void or_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ------------------------------------------------------------- norms ----- */

/* rms_norm_forward, kernels/teeny-kernels/src/nn/norm/rmsnorm.rs:40-122:
 * pass 1 sum of x^2; rrms = rsqrt(sum * (1/N) + eps); pass 2 y = x * rrms * w.
 * rrms[M] is stored (rmsnorm.rs:84). */
void or_rmsnorm(const float* x, const float* w, float* y, float* rrms,
                int64_t M, int64_t N, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) {
        const float* xr = x + m * N;
        double ss = 0.0;
        for (int64_t n = 0; n < N; n++) ss += (double)xr[n] * (double)xr[n];
        double r = 1.0 / sqrt(ss / (double)N + (double)eps);
        if (rrms) rrms[m] = (float)r;
        for (int64_t n = 0; n < N; n++) y[m * N + n] = (float)((double)xr[n] * r * (double)w[n]);
    }
}

/* layer_norm_forward_inference, nn/norm/layernorm.rs:43-157: mean, masked
 * variance (:101), rstd = rsqrt(var/N + eps) (:106), y = (x-mean)*rstd*w + b. */
void or_layernorm(const float* x, const float* w, const float* b, float* y,
                  int64_t M, int64_t N, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) {
        const float* xr = x + m * N;
        double s = 0.0;
        for (int64_t n = 0; n < N; n++) s += xr[n];
        double mean = s / (double)N;
        double v = 0.0;
        for (int64_t n = 0; n < N; n++) {
            double d = xr[n] - mean;
            v += d * d;
        }
        double rstd = 1.0 / sqrt(v / (double)N + (double)eps);
        for (int64_t n = 0; n < N; n++)
            y[m * N + n] = (float)((xr[n] - mean) * rstd * (double)w[n] + (double)b[n]);
    }
}

/* ------------------------------------------------------- activations ----- */

/* kinds: 0 silu (nn/activation/sigmoid.rs:144-147: y = x * 1/(1+exp(-x)))
 *        1 gelu tanh form (nn/activation/gelu.rs:56-64:
 *          y = x / (1 + exp(-2c(x + 0.044715 x^3))), c = sqrt(2/pi))
 *        2 relu (nn/activation/relu.rs:28)
 *        3 sigmoid (nn/activation/sigmoid.rs, 1/(1+exp(-x))) */
static double act1(int kind, double x) {
    switch (kind) {
        case 0: return x / (1.0 + exp(-x));
        case 1: return x / (1.0 + exp(-2.0 * 0.7978845608028654 * (x + 0.044715 * x * x * x)));
        case 2: return x > 0.0 ? x : 0.0;
        case 3: return 1.0 / (1.0 + exp(-x));
        default: return x;
    }
}

void or_act(int kind, const float* x, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = (float)act1(kind, x[i]);
}

/* SwiGLU: silu_forward followed by elemwise_mul_forward
 * (nn/tensor/elemwise_binary.rs:189); fused, one rounding. */
void or_swiglu(const float* g, const float* u, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = (float)(act1(0, g[i]) * (double)u[i]);
}

/* elemwise_add_forward, nn/tensor/elemwise_add.rs:29. */
void or_add(const float* a, const float* b, float* y, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) y[i] = a[i] + b[i];
}

/* ------------------------------------------------------------- GEMMs ----- */

/* linear_forward, nn/mlp/linear.rs:22-117: y[m,n] = sum_k x[m,k] w[n,k] (+ b[n]).
 * W is [N,K] (PyTorch layout).  Optional residual r[m,n] is added after the
 * bias (the fused residual epilogue of the decoder). */
void or_linear(const float* x, const float* w, const float* bias, const float* resid,
               float* y, int64_t M, int64_t N, int64_t K) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            const float* xr = x + m * K;
            const float* wr = w + n * K;
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)xr[k] * (double)wr[k];
            if (bias) acc += bias[n];
            if (resid) acc += resid[m * N + n];
            y[m * N + n] = (float)acc;
        }
    }
}

/* matmul_forward, math/gemm.rs:44-105: C[m,n] = sum_k A[m,k] B[k,n]. */
void or_matmul(const float* a, const float* b, float* c, int64_t M, int64_t N, int64_t K) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) {
        double* acc = (double*)calloc((size_t)N, sizeof(double));
        for (int64_t k = 0; k < K; k++) {
            double av = a[m * K + k];
            const float* br = b + k * N;
            for (int64_t n = 0; n < N; n++) acc[n] += av * (double)br[n];
        }
        for (int64_t n = 0; n < N; n++) c[m * N + n] = (float)acc[n];
        free(acc);
    }
}

/* --------------------------------------------------------- attention ----- */

/* flash_attention2_forward, nn/attention/flash_attn2.rs:53-158, restated as
 * exact softmax: O = softmax(scale * Q K^T) V and L = logsumexp(scale * Q K^T)
 * (natural log, on scaled scores, :136-140 and fixtures/generate.py:719-721).
 * Extensions the reference lacks (documented, unpinned):
 *   - GQA: query head h reads kv head h / (Hq / Hkv);
 *   - causal: query i (0-based within Sq) sees key j iff j <= i + (Sk - Sq)
 *     (bottom-right aligned, so decode with Sq=1 sees the whole cache).
 * Layouts: q [B, Hq, Sq, D], k/v [B, Hkv, Sk, D], o [B, Hq, Sq, D], lse [B, Hq, Sq]. */
void or_attention(const float* q, const float* k, const float* v, float* o, float* lse,
                  int64_t B, int64_t Hq, int64_t Hkv, int64_t Sq, int64_t Sk, int64_t D,
                  float scale, int causal) {
    int64_t group = Hq / Hkv;
#pragma omp parallel for collapse(3) schedule(dynamic, 4)
    for (int64_t b = 0; b < B; b++) {
        for (int64_t h = 0; h < Hq; h++) {
            for (int64_t i = 0; i < Sq; i++) {
                int64_t hk = h / group;
                const float* qr = q + ((b * Hq + h) * Sq + i) * D;
                const float* kb = k + (b * Hkv + hk) * Sk * D;
                const float* vb = v + (b * Hkv + hk) * Sk * D;
                int64_t jmax = causal ? i + (Sk - Sq) : Sk - 1;
                if (jmax > Sk - 1) jmax = Sk - 1;
                double* s = (double*)malloc(sizeof(double) * (size_t)(Sk > 0 ? Sk : 1));
                double mx = -INFINITY;
                for (int64_t j = 0; j <= jmax; j++) {
                    double acc = 0.0;
                    for (int64_t d = 0; d < D; d++) acc += (double)qr[d] * (double)kb[j * D + d];
                    s[j] = acc * (double)scale;
                    if (s[j] > mx) mx = s[j];
                }
                double l = 0.0;
                for (int64_t j = 0; j <= jmax; j++) {
                    s[j] = exp(s[j] - mx);
                    l += s[j];
                }
                float* orow = o + ((b * Hq + h) * Sq + i) * D;
                for (int64_t d = 0; d < D; d++) {
                    double acc = 0.0;
                    for (int64_t j = 0; j <= jmax; j++) acc += s[j] * (double)vb[j * D + d];
                    orow[d] = (jmax >= 0) ? (float)(acc / l) : 0.0f;
                }
                if (lse) lse[(b * Hq + h) * Sq + i] = (jmax >= 0) ? (float)(mx + log(l)) : -INFINITY;
                free(s);
            }
        }
    }
}

/* -------------------------------------------------------------- conv ----- */

/* BN fold of the fused conv spec, nn/fused/conv2d_bn_silu.rs:33-35:
 *   scale = gamma / sqrt(var + eps); shift = beta - scale * mean.
 * The conv bias is folded in as well: shift' = shift + scale * bias. */
void or_bn_fold(const float* gamma, const float* beta, const float* mean, const float* var,
                const float* bias, float eps, float* scale, float* shift, int64_t C) {
    for (int64_t c = 0; c < C; c++) {
        double sc = (double)gamma[c] / sqrt((double)var[c] + (double)eps);
        double sh = (double)beta[c] - sc * (double)mean[c];
        if (bias) sh += sc * (double)bias[c];
        scale[c] = (float)sc;
        shift[c] = (float)sh;
    }
}

/* conv2d_bias_forward, nn/conv/conv2d.rs:643-764 (direct NCHW conv, zero
 * padding, groups = 1), with the inference epilogue of
 * nn/fused/conv2d_bn_silu.rs:141-170: acc -> scale[c]*acc + shift[c] -> act.
 * scale == NULL means 1, shift == NULL means 0 (then `bias` is added as in
 * conv2d.rs:738-754).  act: -1 none, 0 silu, 2 relu. */
void or_conv2d(const float* x, const float* w, const float* bias, const float* scale,
               const float* shift, float* y, int64_t B, int64_t Cin, int64_t Cout, int64_t H,
               int64_t W, int64_t KH, int64_t KW, int64_t stride, int64_t pad, int act) {
    int64_t OH = (H + 2 * pad - KH) / stride + 1;
    int64_t OW = (W + 2 * pad - KW) / stride + 1;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; b++) {
        for (int64_t co = 0; co < Cout; co++) {
            for (int64_t oh = 0; oh < OH; oh++) {
                for (int64_t ow = 0; ow < OW; ow++) {
                    double acc = 0.0;
                    for (int64_t ci = 0; ci < Cin; ci++) {
                        for (int64_t kh = 0; kh < KH; kh++) {
                            int64_t ih = oh * stride + kh - pad;
                            if (ih < 0 || ih >= H) continue;
                            for (int64_t kw = 0; kw < KW; kw++) {
                                int64_t iw = ow * stride + kw - pad;
                                if (iw < 0 || iw >= W) continue;
                                acc += (double)x[((b * Cin + ci) * H + ih) * W + iw] *
                                       (double)w[((co * Cin + ci) * KH + kh) * KW + kw];
                            }
                        }
                    }
                    if (bias && !shift) acc += bias[co];
                    if (scale) acc *= (double)scale[co];
                    if (shift) acc += (double)shift[co];
                    if (act >= 0) acc = act1(act, acc);
                    y[((b * Cout + co) * OH + oh) * OW + ow] = (float)acc;
                }
            }
        }
    }
}

/* batch_norm_2d_nchw_forward_inference, nn/norm/batchnorm.rs:574-686:
 * y = (x - mean[c]) * rsqrt(var[c] + eps) * gamma[c] + beta[c].  x is [B, C, HW]. */
void or_batchnorm_inference(const float* x, const float* gamma, const float* beta,
                            const float* mean, const float* var, float* y, int64_t B,
                            int64_t C, int64_t HW, float eps) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t b = 0; b < B; b++) {
        for (int64_t c = 0; c < C; c++) {
            double r = 1.0 / sqrt((double)var[c] + (double)eps);
            for (int64_t i = 0; i < HW; i++) {
                int64_t idx = (b * C + c) * HW + i;
                y[idx] = (float)(((double)x[idx] - mean[c]) * r * gamma[c] + beta[c]);
            }
        }
    }
}

/* -------------------------------------------------------------- int8 ----- */

/* quantize_affine, utilities/teeny-quant/src/quant/affine.rs:55-148, with
 * Granularity::PerChannel{axis 0} (quant/groups.rs:78-100), symmetric, 8 bits:
 *   qrange = [-127, 127] (:47-51)
 *   lo = min(min(row), 0), hi = max(max(row), 0); amax = max(|lo|, |hi|)
 *   scale = amax == 0 ? 1 : amax / 127            (f32 arithmetic, :112)
 *   q = clamp(round(x / scale) as i32, -127, 127) (:138-139)
 * Rust f32::round rounds half away from zero; C roundf does the same.
 * Non-finite weights follow Rust: NaN is skipped by the min/max pass (its
 * comparisons are false), a row holding -Inf has a non-finite minimum and
 * gets scale 1, a row holding +Inf gets scale Inf; NaN / scale -> 0. */
void or_quantize_int8(const float* w, int8_t* q, float* scale, int64_t N, int64_t K) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++) {
        const float* wr = w + n * K;
        float vmin = INFINITY, vmax = -INFINITY;
        for (int64_t k = 0; k < K; k++) {
            if (wr[k] < vmin) vmin = wr[k];
            if (wr[k] > vmax) vmax = wr[k];
        }
        float lo = 0.0f, hi = 0.0f;
        if (isfinite(vmin)) {
            lo = vmin < 0.0f ? vmin : 0.0f;
            hi = vmax > 0.0f ? vmax : 0.0f;
        }
        float amax = fabsf(lo) > fabsf(hi) ? fabsf(lo) : fabsf(hi);
        float s = (amax == 0.0f) ? 1.0f : amax / 127.0f;
        scale[n] = s;
        for (int64_t k = 0; k < K; k++) {
            /* `(t.round()) as i32` saturates in Rust: NaN -> 0, beyond the
             * i32 range -> i32::MIN / MAX; clamp(-127, 127) follows (:138-139) */
            float t = wr[k] / s;
            int v;
            if (t != t) v = 0;
            else {
                float r = roundf(t);
                v = r <= -127.0f ? -127 : (r >= 127.0f ? 127 : (int)r);
            }
            q[n * K + k] = (int8_t)v;
        }
    }
}

/* dequantize_affine, quant/affine.rs:151-159: (q - 0) as f32 * scale. */
void or_dequantize_int8(const int8_t* q, const float* scale, float* w, int64_t N, int64_t K) {
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++)
        for (int64_t k = 0; k < K; k++) w[n * K + k] = (float)q[n * K + k] * scale[n];
}

/* int8 weight-only linear (absent in the reference: graph/mod.rs:2595-2600):
 * y[m,n] = scale[n] * sum_k x[m,k] * q[n,k] (+ residual). */
void or_int8_linear(const float* x, const int8_t* q, const float* scale, const float* resid,
                    float* y, int64_t M, int64_t N, int64_t K) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            const float* xr = x + m * K;
            const int8_t* qr = q + n * K;
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) acc += (double)xr[k] * (double)qr[k];
            acc *= (double)scale[n];
            if (resid) acc += resid[m * N + n];
            y[m * N + n] = (float)acc;
        }
    }
}

/* ------------------------------------------------- decoder pieces -------- */

/* RoPE (absent in the reference: graph/mod.rs:2472-2475).  Convention of the
 * build: rotate-half pairing (d, d + D/2), inv_freq[i] = theta^(-2i/D),
 * angle = pos * inv_freq[i]; out_d = x_d cos - x_{d+D/2} sin,
 * out_{d+D/2} = x_{d+D/2} cos + x_d sin.  x is [T, H, D], pos [T]. */
void or_rope(const float* x, const int32_t* pos, float* y, int64_t T, int64_t H, int64_t D,
             float theta) {
    int64_t half = D / 2;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t t = 0; t < T; t++) {
        for (int64_t h = 0; h < H; h++) {
            const float* xr = x + (t * H + h) * D;
            float* yr = y + (t * H + h) * D;
            for (int64_t i = 0; i < half; i++) {
                double inv = pow((double)theta, -2.0 * (double)i / (double)D);
                double ang = (double)pos[t] * inv;
                double c = cos(ang), s = sin(ang);
                double a = xr[i], bb = xr[i + half];
                yr[i] = (float)(a * c - bb * s);
                yr[i + half] = (float)(bb * c + a * s);
            }
        }
    }
}

/* Embedding gather (absent: graph/mod.rs:2527-2530): y[t,:] = table[ids[t],:]. */
void or_embedding(const float* table, const int32_t* ids, float* y, int64_t T, int64_t D) {
    for (int64_t t = 0; t < T; t++) memcpy(y + t * D, table + (int64_t)ids[t] * D, sizeof(float) * D);
}

/* ArgMax over rows (absent: graph/mod.rs:2250-2253).  Convention: the lowest
 * index wins ties; NaN is never selected unless the row is all NaN (then 0). */
void or_argmax(const float* x, int32_t* out, int64_t M, int64_t N) {
    for (int64_t m = 0; m < M; m++) {
        const float* r = x + m * N;
        int64_t best = 0;
        float bv = -INFINITY;
        int found = 0;
        for (int64_t n = 0; n < N; n++) {
            if (isnan(r[n])) continue;
            if (!found || r[n] > bv) {
                bv = r[n];
                best = n;
                found = 1;
            }
        }
        out[m] = (int32_t)best;
    }
}

/* ========================================================== backward ===== */

/* rms_norm_backward, kernels/teeny-kernels/src/nn/norm/rmsnorm.rs:125-277:
 *   dot    = sum_n dy[m,n] * w[n] * x[m,n]
 *   dx[m,n] = rrms[m] * (w[n] * dy[m,n] - x[m,n] * rrms[m]^2 * dot / N)
 *   dw[n] += sum_m dy[m,n] * x[m,n] * rrms[m]       (accumulated into dw)
 * rrms[m] is the forward's 1 / sqrt(mean(x^2) + eps).  dx is the gradient of
 * y = x * rrms * w; the reference's dx line (rmsnorm.rs:232) also multiplies
 * the correction term by w[n], which agrees with it only where w[n] == 1. */
void or_rmsnorm_bwd(const float* dy, const float* x, const float* w, const float* rrms, float* dx, float* dw,
                    int64_t M, int64_t N) {
#pragma omp parallel for schedule(static)
    for (int64_t m = 0; m < M; m++) {
        const float* xr = x + m * N;
        const float* dr = dy + m * N;
        double dot = 0.0;
        for (int64_t n = 0; n < N; n++) dot += (double)dr[n] * (double)w[n] * (double)xr[n];
        const double r = (double)rrms[m], sc = dot / (double)N;
        for (int64_t n = 0; n < N; n++)
            dx[m * N + n] = (float)(r * ((double)w[n] * (double)dr[n] - (double)xr[n] * r * r * sc));
    }
    if (dw) {
#pragma omp parallel for schedule(static)
        for (int64_t n = 0; n < N; n++) {
            double acc = 0.0;
            for (int64_t m = 0; m < M; m++) acc += (double)dy[m * N + n] * (double)x[m * N + n] * (double)rrms[m];
            dw[n] = (float)((double)dw[n] + acc);
        }
    }
}

/* linear_backward, nn/mlp/linear.rs:119-249 (y = x w^T + b):
 *   dx = dy w   [M, K];   dw = dy^T x   [N, K];   db = sum_m dy   [N]. */
void or_linear_bwd(const float* x, const float* w, const float* dy, float* dx, float* dw, float* db, int64_t M,
                   int64_t N, int64_t K) {
    if (dx) {
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t m = 0; m < M; m++)
            for (int64_t k = 0; k < K; k++) {
                double acc = 0.0;
                for (int64_t n = 0; n < N; n++) acc += (double)dy[m * N + n] * (double)w[n * K + k];
                dx[m * K + k] = (float)acc;
            }
    }
    if (dw) {
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t n = 0; n < N; n++)
            for (int64_t k = 0; k < K; k++) {
                double acc = 0.0;
                for (int64_t m = 0; m < M; m++) acc += (double)dy[m * N + n] * (double)x[m * K + k];
                dw[n * K + k] = (float)acc;
            }
    }
    if (db) {
        for (int64_t n = 0; n < N; n++) {
            double acc = 0.0;
            for (int64_t m = 0; m < M; m++) acc += (double)dy[m * N + n];
            db[n] = (float)acc;
        }
    }
}

/* flash_attention2_backward_dq / _dkv, nn/attention/flash_attn2.rs:160-447,
 * extended (as the forward) with the causal mask and GQA:
 *   p_ij  = exp(q_i . k_j * scale - L_i)          (L: the forward's LSE)
 *   D_i   = sum_d O_i[d] dO_i[d]
 *   dS_ij = p_ij (dO_i . v_j - D_i)
 *   dQ_i  = scale * sum_j dS_ij k_j;  dK_j = scale * sum_i dS_ij q_i;  dV_j = sum_i p_ij dO_i
 * with dK / dV of a kv head summed over the query heads of its group. */
void or_attention_bwd(const float* q, const float* k, const float* v, const float* o, const float* dout,
                      const float* lse, float* dq, float* dk, float* dv, int64_t B, int64_t Hq, int64_t Hkv,
                      int64_t Sq, int64_t Sk, int64_t D, float scale, int causal) {
    const int64_t group = Hq / Hkv;
    double* acc_k = (double*)calloc((size_t)(B * Hkv * Sk * D), sizeof(double));
    double* acc_v = (double*)calloc((size_t)(B * Hkv * Sk * D), sizeof(double));
    for (int64_t b = 0; b < B; b++) {
#pragma omp parallel for schedule(static)
        for (int64_t hk = 0; hk < Hkv; hk++) {
            for (int64_t h = hk * group; h < (hk + 1) * group; h++) {
                for (int64_t i = 0; i < Sq; i++) {
                    const float* qr = q + ((b * Hq + h) * Sq + i) * D;
                    const float* orow = o + ((b * Hq + h) * Sq + i) * D;
                    const float* dor = dout + ((b * Hq + h) * Sq + i) * D;
                    const float* kb = k + (b * Hkv + hk) * Sk * D;
                    const float* vb = v + (b * Hkv + hk) * Sk * D;
                    double* akb = acc_k + (b * Hkv + hk) * Sk * D;
                    double* avb = acc_v + (b * Hkv + hk) * Sk * D;
                    int64_t jmax = causal ? i + (Sk - Sq) : Sk - 1;
                    if (jmax > Sk - 1) jmax = Sk - 1;
                    const double L = (double)lse[(b * Hq + h) * Sq + i];
                    double Di = 0.0;
                    for (int64_t d = 0; d < D; d++) Di += (double)orow[d] * (double)dor[d];
                    double* dqa = (double*)calloc((size_t)D, sizeof(double));
                    for (int64_t j = 0; j <= jmax; j++) {
                        double s = 0.0, dp = 0.0;
                        for (int64_t d = 0; d < D; d++) {
                            s += (double)qr[d] * (double)kb[j * D + d];
                            dp += (double)dor[d] * (double)vb[j * D + d];
                        }
                        const double p = exp(s * (double)scale - L);
                        const double ds = p * (dp - Di);
                        for (int64_t d = 0; d < D; d++) {
                            dqa[d] += ds * (double)kb[j * D + d];
                            akb[j * D + d] += ds * (double)qr[d];
                            avb[j * D + d] += p * (double)dor[d];
                        }
                    }
                    float* dqr = dq + ((b * Hq + h) * Sq + i) * D;
                    for (int64_t d = 0; d < D; d++) dqr[d] = (float)(dqa[d] * (double)scale);
                    free(dqa);
                }
            }
        }
    }
    for (int64_t e = 0; e < B * Hkv * Sk * D; e++) {
        dk[e] = (float)(acc_k[e] * (double)scale);
        dv[e] = (float)acc_v[e];
    }
    free(acc_k);
    free(acc_v);
}

/* conv2d_backward, nn/conv/conv2d.rs:395-521 (groups = 1, zero padding):
 *   dx[b,ci,ih,iw] = sum_{co,kh,kw} dy[b,co,oh,ow] w[co,ci,kh,kw]
 *                    over oh*stride + kh - pad = ih, ow*stride + kw - pad = iw
 *   dw[co,ci,kh,kw] = sum_{b,oh,ow} dy[b,co,oh,ow] x[b,ci,oh*stride+kh-pad,ow*stride+kw-pad]
 * The reference scatters both with atomic adds; this restatement gathers. */
void or_conv2d_bwd(const float* dy, const float* x, const float* w, float* dx, float* dw, int64_t B, int64_t Cin,
                   int64_t Cout, int64_t H, int64_t W, int64_t KH, int64_t KW, int64_t stride, int64_t pad) {
    const int64_t OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
    if (dx) {
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t b = 0; b < B; b++)
            for (int64_t ci = 0; ci < Cin; ci++)
                for (int64_t ih = 0; ih < H; ih++)
                    for (int64_t iw = 0; iw < W; iw++) {
                        double acc = 0.0;
                        for (int64_t co = 0; co < Cout; co++)
                            for (int64_t kh = 0; kh < KH; kh++) {
                                const int64_t th = ih + pad - kh;
                                if (th < 0 || th % stride) continue;
                                const int64_t oh = th / stride;
                                if (oh >= OH) continue;
                                for (int64_t kw = 0; kw < KW; kw++) {
                                    const int64_t tw = iw + pad - kw;
                                    if (tw < 0 || tw % stride) continue;
                                    const int64_t ow = tw / stride;
                                    if (ow >= OW) continue;
                                    acc += (double)dy[((b * Cout + co) * OH + oh) * OW + ow] *
                                           (double)w[((co * Cin + ci) * KH + kh) * KW + kw];
                                }
                            }
                        dx[((b * Cin + ci) * H + ih) * W + iw] = (float)acc;
                    }
    }
    if (dw) {
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t co = 0; co < Cout; co++)
            for (int64_t ci = 0; ci < Cin; ci++)
                for (int64_t kh = 0; kh < KH; kh++)
                    for (int64_t kw = 0; kw < KW; kw++) {
                        double acc = 0.0;
                        for (int64_t b = 0; b < B; b++)
                            for (int64_t oh = 0; oh < OH; oh++) {
                                const int64_t ih = oh * stride + kh - pad;
                                if (ih < 0 || ih >= H) continue;
                                for (int64_t ow = 0; ow < OW; ow++) {
                                    const int64_t iw = ow * stride + kw - pad;
                                    if (iw < 0 || iw >= W) continue;
                                    acc += (double)dy[((b * Cout + co) * OH + oh) * OW + ow] *
                                           (double)x[((b * Cin + ci) * H + ih) * W + iw];
                                }
                            }
                        dw[((co * Cin + ci) * KH + kh) * KW + kw] = (float)acc;
                    }
    }
}

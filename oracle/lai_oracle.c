/*
 * lai_oracle.c - CPU restatement of local-ai-server's per-layer kernels.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA kernels and the timed CPU
 * baseline. The product library never links or calls it.
 *
 * Provenance. The reference's own C for qwen_rms_norm, qwen_rms_norm_per_head,
 * qwen_apply_rope_neox, qwen_compute_rope_neox, qwen_swiglu_multiply,
 * qwen_add_inplace and qwen_silu lives in the un-vendored git submodule
 * `qwen-asr` (https://github.com/rmtew/qwen-asr.git, .gitmodules:1-3, pinned
 * commit unknown), which is empty in the mounted reference. Those functions are
 * restated here from
 *   - their call sites (argument order, in-place conventions):
 *       src/tts_native.c:553-592, 634-669, 711-748; src/tts_vocoder_xfmr.c:150-211
 *   - the repo's own numpy specification of the same math:
 *       tools/verify_xfmr.py:32-35 (RMSNorm), :37-55 (NeoX RoPE), :79-80 (SiLU)
 *   - the C that is present for the neighbouring code:
 *       src/tts_native.c:377-417 (RoPE table), :149-161 (gate/up row interleave),
 *       :35-40 (BF16 -> F32), src/tts_vocoder_xfmr.c:73-80 (SiLU * up).
 * The parity of these restatements is pinned to the reference's numpy
 * functions (tests/golden/make_golden.py extracts them from tools/verify_*.py),
 * not to the absent C. SnakeBeta (src/tts_vocoder_ops.c:279-305) is present and
 * oracle/Makefile compiles the reference's own function into oracle/_ref/; the
 * restatement below is checked against it.
 *
 * LAI_ACC selects the accumulator of sums of squares: double in the checker
 * build (so that the oracle's own rounding stays far below the 1e-5 tolerance),
 * float in the timed baseline build (what a C implementation would do).
 */
#include "lai_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#ifndef LAI_ACC
#define LAI_ACC double
#endif

typedef LAI_ACC acc_t;

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Thread count of the timed build's parallel loops (launchers such as torchrun
 * export OMP_NUM_THREADS=1; the CPU baseline is meant to use every host core). */
void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---------------------------------------------------------------------------
 * BF16 <-> F32. Widening is the bit shift of src/tts_native.c:35-40 (exact).
 * Narrowing is round-to-nearest-even, the rounding of every BF16 store
 * (NaN becomes the canonical 0x7fff, as the GPU's cvt.rn.bf16.f32 makes it).
 * ------------------------------------------------------------------------- */
float oracle_bf16_to_f32(uint16_t h) {
    uint32_t bits = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &bits, sizeof(f));
    return f;
}

uint16_t oracle_f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, sizeof(u));
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fffu; /* canonical NaN, as cvt.rn.bf16 */
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* ---------------------------------------------------------------------------
 * RMSNorm: out[s,:] = (x[s,:] / sqrt(mean(x[s,:]^2) + eps)) * w
 * Spec: tools/verify_xfmr.py:32-35. Call sites: src/tts_native.c:556, 584, 637,
 * 661, 674 (out == x), src/tts_vocoder_xfmr.c:163, 189, 211. Row-wise, so
 * out == x is safe.
 * ------------------------------------------------------------------------- */
static void rms_norm_row(float *out, const float *x, const float *w, int dim, float eps) {
    acc_t ss = 0;
    for (int i = 0; i < dim; i++) ss += (acc_t)x[i] * (acc_t)x[i];
    float rms = sqrtf((float)(ss / (acc_t)dim) + eps);
    for (int i = 0; i < dim; i++) out[i] = (x[i] / rms) * w[i];
}

void oracle_rms_norm(float *out, const float *x, const float *w, int seq, int dim, float eps) {
#pragma omp parallel for schedule(static)
    for (int s = 0; s < seq; s++)
        rms_norm_row(out + (size_t)s * dim, x + (size_t)s * dim, w, dim, eps);
}

/* Per-head RMSNorm in place; w [head_dim] shared by all heads (q_norm / k_norm,
 * src/tts_native.c:125-128). Call sites src/tts_native.c:562-563, 644-645. */
void oracle_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim,
                              float eps) {
#pragma omp parallel for schedule(static)
    for (int s = 0; s < seq; s++)
        for (int h = 0; h < n_heads; h++) {
            float *xh = x + ((size_t)s * n_heads + h) * head_dim;
            rms_norm_row(xh, xh, w, head_dim, eps);
        }
}

/* ---------------------------------------------------------------------------
 * NeoX RoPE (rotate-half) in place. Row s uses row s of the cos/sin table;
 * decode call sites offset the table pointer to row `pos`
 * (src/tts_native.c:565-568, 647-648). Table rows are [head_dim] with
 * duplicated halves (src/tts_native.c:402-412), and the formula follows
 * tools/verify_xfmr.py:49-53: (x1*c - x2*s, x1*s + x2*c).
 * ------------------------------------------------------------------------- */
static void rope_head(float *xh, const float *c, const float *sn, int head_dim) {
    int half = head_dim / 2;
    for (int d = 0; d < half; d++) {
        float x1 = xh[d], x2 = xh[d + half];
        xh[d] = x1 * c[d] - x2 * sn[d];
        xh[d + half] = x1 * sn[d + half] + x2 * c[d + half];
    }
}

void oracle_apply_rope_neox(float *x, const float *cos_t, const float *sin_t, int seq,
                            int n_heads, int head_dim) {
#pragma omp parallel for schedule(static)
    for (int s = 0; s < seq; s++)
        for (int h = 0; h < n_heads; h++)
            rope_head(x + ((size_t)s * n_heads + h) * head_dim, cos_t + (size_t)s * head_dim,
                      sin_t + (size_t)s * head_dim, head_dim);
}

void oracle_apply_rope_neox_pos(float *x, const float *cos_t, const float *sin_t,
                                const int32_t *pos, int seq, int n_heads, int head_dim) {
    for (int s = 0; s < seq; s++) {
        size_t p = pos ? (size_t)pos[s] : (size_t)s;
        for (int h = 0; h < n_heads; h++)
            rope_head(x + ((size_t)s * n_heads + h) * head_dim, cos_t + p * head_dim,
                      sin_t + p * head_dim, head_dim);
    }
}

/* inv_freq[d] = 1 / theta^(2d/hd), exactly as ensure_rope_cache computes it
 * (src/tts_native.c:383-388). */
void oracle_rope_inv_freq(float *inv_freq, int head_dim, float theta) {
    for (int d = 0; d < head_dim / 2; d++)
        inv_freq[d] = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
}

/* cos/sin rows for arbitrary positions: qwen_compute_rope_neox's contract
 * (src/tts_vocoder_xfmr.c:150-156), row layout of src/tts_native.c:402-412. */
void oracle_compute_rope_neox(float *cos_t, float *sin_t, const int *pos, int n, int head_dim,
                              float theta) {
    int half = head_dim / 2;
    float inv_freq[1024];
    if (half > 1024) return;
    oracle_rope_inv_freq(inv_freq, head_dim, theta);
    for (int i = 0; i < n; i++) {
        float *cr = cos_t + (size_t)i * head_dim, *sr = sin_t + (size_t)i * head_dim;
        for (int d = 0; d < half; d++) {
            float angle = (float)pos[i] * inv_freq[d];
            float c = cosf(angle), s = sinf(angle);
            cr[d] = c;
            cr[half + d] = c;
            sr[d] = s;
            sr[half + d] = s;
        }
    }
}

/* ---------------------------------------------------------------------------
 * SwiGLU over the interleaved GEMM output. The gate/up weight rows are
 * interleaved [g0,u0,g1,u1,...] (src/tts_native.c:149-161), so row s of
 * gate_up is [g(s,0), u(s,0), g(s,1), u(s,1), ...] and, flattened,
 * out[k] = silu(in[2k]) * in[2k+1] for k < seq*inter. The call sites pass
 * out == gate_up (src/tts_native.c:588, 665, 744); increasing k is safe in place
 * because write k only clobbers inputs already consumed by k/2.
 * SiLU*up is written as src/tts_vocoder_xfmr.c:76-78 writes it.
 * ------------------------------------------------------------------------- */
static inline float silu_mul(float g, float u) {
    float sig = 1.0f / (1.0f + expf(-g));
    return (g * sig) * u;
}

void oracle_swiglu_multiply(float *out, const float *gate_up, int seq, int inter) {
    size_t n = (size_t)seq * (size_t)inter;
    for (size_t k = 0; k < n; k++) out[k] = silu_mul(gate_up[2 * k], gate_up[2 * k + 1]);
}

/* swiglu_separate (src/tts_vocoder_xfmr.c:73-80). */
void oracle_swiglu_separate(float *out, const float *gate, const float *up, int n) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) out[i] = silu_mul(gate[i], up[i]);
}

/* qwen_silu(x, n) in place (src/tts_native.c:504); spec tools/verify_xfmr.py:79-80. */
void oracle_silu(float *x, int n) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        float g = x[i];
        float sig = 1.0f / (1.0f + expf(-g));
        x[i] = g * sig;
    }
}

/* qwen_add_inplace(x, y, n): x += y (src/tts_native.c:582, 591, 1142). */
void oracle_add_inplace(float *x, const float *y, int n) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) x[i] += y[i];
}

/* ---------------------------------------------------------------------------
 * SnakeBeta, scalar branch of voc_snake_beta (src/tts_vocoder_ops.c:298-303):
 * x[c,t] += ieb[c] * sin(ea[c]*x[c,t])^2, params pre-exponentiated
 * (src/tts_vocoder.c:221-227).
 * ------------------------------------------------------------------------- */
void oracle_snake_beta(float *x, const float *exp_alpha, const float *inv_exp_beta,
                       int channels, int T) {
#pragma omp parallel for schedule(static)
    for (int ch = 0; ch < channels; ch++) {
        float *row = x + (size_t)ch * T;
        float ea = exp_alpha[ch], ieb = inv_exp_beta[ch];
        for (int t = 0; t < T; t++) {
            float s = sinf(ea * row[t]);
            row[t] += ieb * s * s;
        }
    }
}

/* ---------------------------------------------------------------------------
 * BF16 embedding gather (src/tts_native.c:35-40, 473-476): row id of a
 * [vocab, dim] BF16 table, widened to F32 by the bit shift, or copied as BF16.
 * ------------------------------------------------------------------------- */
void oracle_embed_gather_bf16_to_f32(float *out, const uint16_t *table, const int32_t *ids,
                                     int n, int dim) {
    for (int r = 0; r < n; r++) {
        const uint16_t *src = table + (size_t)ids[r] * dim;
        float *dst = out + (size_t)r * dim;
        for (int i = 0; i < dim; i++) {
            uint32_t bits = ((uint32_t)src[i]) << 16;
            memcpy(&dst[i], &bits, sizeof(float));
        }
    }
}

void oracle_embed_gather_bf16(uint16_t *out, const uint16_t *table, const int32_t *ids, int n,
                              int dim) {
    for (int r = 0; r < n; r++)
        memcpy(out + (size_t)r * dim, table + (size_t)ids[r] * dim, (size_t)dim * 2);
}

/* ---------------------------------------------------------------------------
 * Fused compositions. Each is the reference's own call sequence on one row
 * (src/tts_native.c:582-584: qwen_add_inplace then qwen_rms_norm;
 * :562-568: per-head norms then RoPE), which is what the fused kernels must
 * reproduce. BF16 variants round to BF16 wherever the kernel stores BF16: the
 * updated residual x' is rounded before it is normalised, so the fused kernel
 * equals the unfused BF16 add followed by the BF16 RMSNorm.
 * ------------------------------------------------------------------------- */
void oracle_add_rms_norm_f32(float *x, const float *delta, const float *w, float *y, int seq,
                             int dim, float eps) {
    for (int s = 0; s < seq; s++) {
        float *xr = x + (size_t)s * dim;
        const float *dr = delta + (size_t)s * dim;
        for (int i = 0; i < dim; i++) xr[i] += dr[i];
        rms_norm_row(y + (size_t)s * dim, xr, w, dim, eps);
    }
}

void oracle_add_bf16(uint16_t *x, const uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; i++)
        x[i] = oracle_f32_to_bf16(oracle_bf16_to_f32(x[i]) + oracle_bf16_to_f32(y[i]));
}

void oracle_rms_norm_bf16(uint16_t *out, const uint16_t *x, const float *w, int seq, int dim,
                          float eps) {
    float row[16384], o[16384];
    if (dim > 16384) return;
    for (int s = 0; s < seq; s++) {
        for (int i = 0; i < dim; i++) row[i] = oracle_bf16_to_f32(x[(size_t)s * dim + i]);
        rms_norm_row(o, row, w, dim, eps);
        for (int i = 0; i < dim; i++) out[(size_t)s * dim + i] = oracle_f32_to_bf16(o[i]);
    }
}

void oracle_add_rms_norm_bf16(uint16_t *x, const uint16_t *delta, const float *w, uint16_t *y,
                              int seq, int dim, float eps) {
    oracle_add_bf16(x, delta, (int64_t)seq * dim);
    oracle_rms_norm_bf16(y, x, w, seq, dim, eps);
}

void oracle_qk_norm_rope_f32(float *q, float *k, const float *wq, const float *wk,
                             const float *cos_t, const float *sin_t, const int32_t *pos,
                             int seq, int n_q_heads, int n_kv_heads, int head_dim, float eps) {
    if (wq) oracle_rms_norm_per_head(q, wq, seq, n_q_heads, head_dim, eps);
    if (wk && k) oracle_rms_norm_per_head(k, wk, seq, n_kv_heads, head_dim, eps);
    if (cos_t) {
        oracle_apply_rope_neox_pos(q, cos_t, sin_t, pos, seq, n_q_heads, head_dim);
        if (k) oracle_apply_rope_neox_pos(k, cos_t, sin_t, pos, seq, n_kv_heads, head_dim);
    }
}

static void qk_bf16_one(uint16_t *t, const float *w, const float *cos_t, const float *sin_t,
                        const int32_t *pos, int seq, int heads, int head_dim, float eps) {
    size_t n = (size_t)seq * heads * head_dim;
    for (size_t base = 0; base < n; base += (size_t)heads * head_dim) {
        int s = (int)(base / ((size_t)heads * head_dim));
        float buf[8192];
        int row = heads * head_dim;
        if (row > 8192) return;
        for (int i = 0; i < row; i++) buf[i] = oracle_bf16_to_f32(t[base + i]);
        if (w) oracle_rms_norm_per_head(buf, w, 1, heads, head_dim, eps);
        if (cos_t) {
            int32_t p = pos ? pos[s] : s;
            oracle_apply_rope_neox_pos(buf, cos_t, sin_t, &p, 1, heads, head_dim);
        }
        for (int i = 0; i < row; i++) t[base + i] = oracle_f32_to_bf16(buf[i]);
    }
}

void oracle_qk_norm_rope_bf16(uint16_t *q, uint16_t *k, const float *wq, const float *wk,
                              const float *cos_t, const float *sin_t, const int32_t *pos,
                              int seq, int n_q_heads, int n_kv_heads, int head_dim, float eps) {
    qk_bf16_one(q, wq, cos_t, sin_t, pos, seq, n_q_heads, head_dim, eps);
    if (k) qk_bf16_one(k, wk, cos_t, sin_t, pos, seq, n_kv_heads, head_dim, eps);
}

void oracle_swiglu_bf16(uint16_t *out, const uint16_t *gate_up, int seq, int inter) {
    size_t n = (size_t)seq * (size_t)inter;
    for (size_t k = 0; k < n; k++)
        out[k] = oracle_f32_to_bf16(
            silu_mul(oracle_bf16_to_f32(gate_up[2 * k]), oracle_bf16_to_f32(gate_up[2 * k + 1])));
}

/* ---------------------------------------------------------------------------
 * linear_bf16 / qwen_linear_nobias_bf16 (src/tts_native.c:66-79; the CPU body is in
 * the absent qwen-asr submodule): out[m,n] = sum_k in[m,k] * W[n,k], W row-major
 * [N, K] BF16 widened exactly to F32 (bits << 16).
 * ------------------------------------------------------------------------- */
void oracle_linear_bf16(float *out, const float *in, const uint16_t *W, int M, int K, int N) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const uint16_t *wr = W + (size_t)n * K;
        for (int m = 0; m < M; m++) {
            const float *xr = in + (size_t)m * K;
            acc_t s = 0;
            for (int k = 0; k < K; k++) s += (acc_t)oracle_bf16_to_f32(wr[k]) * (acc_t)xr[k];
            out[(size_t)m * N + n] = (float)s;
        }
    }
}

/* ---------------------------------------------------------------------------
 * Causal self-attention over a sequence: qwen_causal_attention(out, q, k, v, T, T, heads,
 * kv_heads, hd, scale, 0) as the vocoder's pre-transformer calls it
 * (src/tts_vocoder_xfmr.c:172-180); the math of tools/verify_xfmr.py:57-77: scores
 * q.k * scale over keys 0..t, max-subtracted softmax, weighted sum of v. The function body is
 * in the un-vendored qwen-asr sources, so this follows the spec, in acc_t.
 * ------------------------------------------------------------------------- */
void oracle_causal_attention(float *out, const float *q, const float *k, const float *v, int T,
                             int n_heads, int n_kv_heads, int head_dim, float scale) {
    const int group = n_heads / n_kv_heads;
    const int ldq = n_heads * head_dim, ldk = n_kv_heads * head_dim;
#pragma omp parallel for schedule(dynamic)
    for (int th = 0; th < T * n_heads; th++) {
        const int t = th / n_heads, h = th % n_heads, kvh = h / group;
        const float *qr = q + (size_t)t * ldq + (size_t)h * head_dim;
        acc_t *sc = (acc_t *)malloc(sizeof(acc_t) * (size_t)(t + 1));
        acc_t mx = -1e300;
        for (int j = 0; j <= t; j++) {
            const float *kr = k + (size_t)j * ldk + (size_t)kvh * head_dim;
            acc_t s = 0;
            for (int d = 0; d < head_dim; d++) s += (acc_t)qr[d] * (acc_t)kr[d];
            sc[j] = s * (acc_t)scale;
            if (sc[j] > mx) mx = sc[j];
        }
        acc_t den = 0;
        for (int j = 0; j <= t; j++) {
            sc[j] = (acc_t)exp((double)(sc[j] - mx));
            den += sc[j];
        }
        float *o = out + (size_t)t * ldq + (size_t)h * head_dim;
        for (int d = 0; d < head_dim; d++) {
            acc_t a = 0;
            for (int j = 0; j <= t; j++) a += sc[j] * (acc_t)v[(size_t)j * ldk + (size_t)kvh * head_dim + d];
            o[d] = (float)(a / den);
        }
        free(sc);
    }
}

/* ---------------------------------------------------------------------------
 * The reference's other GPU weight formats for the same linears: FP16 (its fp16 mode),
 * INT8 with a per-row scale (its int8 mode) and F32 (src/tts_pipeline.h:37-40,
 * src/tts_native.c:1185-1240). The INT8 recipe is tools/asr_benchmarks.md:342-352:
 * scale = max(abs(row)) / 127, int8[j] = round(row[j] / scale), the scale applied after
 * the row's reduction. The conversion code sits in the un-vendored qwen-asr GPU sources,
 * so "round" is taken as C roundf (halves away from zero) on the F32 quotient.
 * ------------------------------------------------------------------------- */
float oracle_f16_to_f32(uint16_t h) {
    /* binary16: sign, 5-bit exponent (bias 15), 10-bit fraction; exponent 0 is
     * subnormal (f * 2^-24), 31 is inf / NaN; normal = (1024 + f) * 2^(e - 25) */
    const int s = h >> 15, e = (h >> 10) & 31, f = h & 1023;
    float v;
    if (e == 0)
        v = ldexpf((float)f, -24);
    else if (e == 31)
        v = f ? NAN : INFINITY;
    else
        v = ldexpf((float)(f | 1024), e - 25);
    return s ? -v : v;
}

uint16_t oracle_f32_to_f16(float x) {
    const uint16_t sign = signbit(x) ? 0x8000 : 0;
    const float a = fabsf(x);
    if (isnan(x)) return sign | 0x7e00;
    if (isinf(x)) return sign | 0x7c00;
    if (a < 0x1p-14f) /* subnormal range: k * 2^-24 with k rounded to nearest even */
        return sign | (uint16_t)nearbyintf(a * 0x1p24f); /* k = 1024 is the least normal */
    int e;
    frexpf(a, &e); /* a in [2^(e-1), 2^e) */
    float q = nearbyintf(ldexpf(a, 11 - e)); /* 11 significant bits, in [1024, 2048] */
    int E = e - 1 + 15;
    if (q >= 2048.0f) {
        q = 1024.0f;
        E++;
    }
    if (E >= 31) return sign | 0x7c00;
    return sign | (uint16_t)(E << 10) | (uint16_t)((int)q - 1024);
}

void oracle_f32_to_f16_array(uint16_t *dst, const float *src, int64_t n) {
    for (int64_t i = 0; i < n; i++) dst[i] = oracle_f32_to_f16(src[i]);
}

void oracle_linear_f16(float *out, const float *in, const uint16_t *W, int M, int K, int N) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const uint16_t *wr = W + (size_t)n * K;
        for (int m = 0; m < M; m++) {
            const float *xr = in + (size_t)m * K;
            acc_t s = 0;
            for (int k = 0; k < K; k++) s += (acc_t)oracle_f16_to_f32(wr[k]) * (acc_t)xr[k];
            out[(size_t)m * N + n] = (float)s;
        }
    }
}

void oracle_linear_i8(float *out, const float *in, const int8_t *W, const float *scales, int M,
                      int K, int N) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const int8_t *wr = W + (size_t)n * K;
        for (int m = 0; m < M; m++) {
            const float *xr = in + (size_t)m * K;
            acc_t s = 0;
            for (int k = 0; k < K; k++) s += (acc_t)wr[k] * (acc_t)xr[k];
            out[(size_t)m * N + n] = (float)(s * (acc_t)scales[n]);
        }
    }
}

void oracle_linear_f32(float *out, const float *in, const float *W, int M, int K, int N) {
#pragma omp parallel for schedule(static)
    for (int n = 0; n < N; n++) {
        const float *wr = W + (size_t)n * K;
        for (int m = 0; m < M; m++) {
            const float *xr = in + (size_t)m * K;
            acc_t s = 0;
            for (int k = 0; k < K; k++) s += (acc_t)wr[k] * (acc_t)xr[k];
            out[(size_t)m * N + n] = (float)s;
        }
    }
}

void oracle_quantize_rows_i8_bf16(int8_t *q, float *scales, const uint16_t *W, int N, int K) {
    for (int n = 0; n < N; n++) {
        const uint16_t *wr = W + (size_t)n * K;
        float amax = 0.0f;
        for (int k = 0; k < K; k++) {
            const float a = fabsf(oracle_bf16_to_f32(wr[k]));
            if (a > amax) amax = a;
        }
        const float scale = amax / 127.0f;
        scales[n] = scale;
        for (int k = 0; k < K; k++) {
            float v = scale > 0.0f ? roundf(oracle_bf16_to_f32(wr[k]) / scale) : 0.0f;
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            q[(size_t)n * K + k] = (int8_t)(int)v;
        }
    }
}

/* ---------------------------------------------------------------------------
 * Causal dilated conv1d, channels-first, groups == 1 (voc_conv1d_causal,
 * src/tts_vocoder_ops.c:44-147): the input is left-padded with
 * dilation * (kernel - 1) zeros, so tap k of output t reads
 * in[c, t - (kernel - 1 - k) * dilation] (zero before t = 0); weight
 * [c_out, c_in, kernel] row-major; bias may be NULL. The reference sums through
 * im2col and SGEMM in float; this restatement sums each output in acc_t.
 * ------------------------------------------------------------------------- */
void oracle_voc_conv1d_causal(float *out, const float *in, const float *w, const float *bias,
                              int c_in, int c_out, int T, int kernel, int dilation) {
#pragma omp parallel for schedule(static)
    for (int o = 0; o < c_out; o++) {
        const float *wo = w + (size_t)o * c_in * kernel;
        for (int t = 0; t < T; t++) {
            acc_t s = 0;
            for (int c = 0; c < c_in; c++) {
                const float *row = in + (size_t)c * T;
                for (int k = 0; k < kernel; k++) {
                    int src = t - (kernel - 1 - k) * dilation;
                    if (src >= 0) s += (acc_t)wo[(size_t)c * kernel + k] * (acc_t)row[src];
                }
            }
            out[(size_t)o * T + t] = (float)s + (bias ? bias[o] : 0.0f);
        }
    }
}

/* ---------------------------------------------------------------------------
 * BigVGAN ResUnit (run_resunit, src/tts_vocoder.c:540-583), in place on x [C, T]:
 *   r = x ; x = snake1(x) ; h = conv1(x) (k = 7, dilation d) + b1 ; h = snake2(h)
 *   x = conv2(h) (k = 1) + b2 + r
 * Snake parameters are pre-exponentiated (src/tts_vocoder.c:221-227).
 * scratch: 2 * C * T floats (the residual copy and h).
 * ------------------------------------------------------------------------- */
void oracle_voc_resunit(float *x, const float *ea1, const float *ieb1, const float *w1,
                        const float *b1, const float *ea2, const float *ieb2, const float *w2,
                        const float *b2, int C, int T, int dilation, float *scratch) {
    size_t cT = (size_t)C * T;
    float *res = scratch, *h = scratch + cT;
    memcpy(res, x, cT * sizeof(float));
    oracle_snake_beta(x, ea1, ieb1, C, T);
    oracle_voc_conv1d_causal(h, x, w1, b1, C, C, T, 7, dilation);
    oracle_snake_beta(h, ea2, ieb2, C, T);
    oracle_voc_conv1d_causal(x, h, w2, b2, C, C, T, 1, 1);
    for (size_t i = 0; i < cT; i++) x[i] += res[i];
}

/* ---------------------------------------------------------------------------
 * Transposed conv1d (voc_conv_transpose1d, src/tts_vocoder_ops.c:153-221, its scatter
 * formulation): out[oc, t*stride + ki - trim] += x[ic, t] * w[ic, oc, ki] over all ic, t,
 * ki with 0 <= index < T_out, trim = kernel - stride, T_out = (T + 1) * stride - kernel;
 * then + bias. Summed per output in acc_t (gathered instead of scattered).
 * ------------------------------------------------------------------------- */
void oracle_voc_conv_transpose1d(float *out, const float *in, const float *w, const float *bias,
                                 int c_in, int c_out, int T, int kernel, int stride) {
    const int trim = kernel - stride, T_out = (T + 1) * stride - kernel;
#pragma omp parallel for schedule(static)
    for (int oc = 0; oc < c_out; oc++)
        for (int oi = 0; oi < T_out; oi++) {
            acc_t s = 0;
            for (int ki = 0; ki < kernel; ki++) {
                const int num = oi + trim - ki;  /* = t * stride */
                if (num < 0 || num % stride) continue;
                const int t = num / stride;
                if (t >= T) continue;
                for (int ic = 0; ic < c_in; ic++)
                    s += (acc_t)in[(size_t)ic * T + t] * w[((size_t)ic * c_out + oc) * kernel + ki];
            }
            out[(size_t)oc * T_out + oi] = (float)s + (bias ? bias[oc] : 0.0f);
        }
}

/* ---------------------------------------------------------------------------
 * ConvNeXt pieces. Depthwise causal conv: voc_conv1d_causal with groups == c_in ==
 * c_out (src/tts_vocoder_ops.c:52-73), out[c,t] = b[c] + sum_k w[c,k] x[c, t-(K-1)+k]
 * (zero before t = 0), summed in acc_t in tap order. out may equal in (the reference
 * pads into scratch first); here a row copy keeps that safe.
 * ------------------------------------------------------------------------- */
void oracle_voc_conv1d_depthwise(float *out, const float *in, const float *w, const float *bias,
                                 int channels, int T, int kernel) {
#pragma omp parallel for schedule(static)
    for (int c = 0; c < channels; c++) {
        float *row = (float *)malloc((size_t)T * sizeof(float));
        if (!row) continue;
        memcpy(row, in + (size_t)c * T, (size_t)T * sizeof(float));
        for (int t = 0; t < T; t++) {
            acc_t s = 0;
            for (int k = 0; k < kernel; k++) {
                const int src = t - (kernel - 1) + k;
                if (src >= 0) s += (acc_t)w[(size_t)c * kernel + k] * row[src];
            }
            out[(size_t)c * T + t] = (float)s + (bias ? bias[c] : 0.0f);
        }
        free(row);
    }
}

/* LayerNorm over channels at each time step of x [C, T] (voc_layer_norm_channels,
 * src/tts_vocoder_ops.c:311-336): mean, then the mean of squared deviations, then
 * (x - mean) / sqrt(var + eps) * w + b; sums in acc_t. */
void oracle_voc_layer_norm_channels(float *x, const float *w, const float *b, int channels, int T,
                                    float eps) {
#pragma omp parallel for schedule(static)
    for (int t = 0; t < T; t++) {
        acc_t mean = 0, var = 0;
        for (int c = 0; c < channels; c++) mean += x[(size_t)c * T + t];
        mean /= channels;
        for (int c = 0; c < channels; c++) {
            const acc_t d = x[(size_t)c * T + t] - mean;
            var += d * d;
        }
        var /= channels;
        const float inv_std = 1.0f / sqrtf((float)var + eps);
        for (int c = 0; c < channels; c++) {
            const float v = (x[(size_t)c * T + t] - (float)mean) * inv_std;
            x[(size_t)c * T + t] = v * w[c] + b[c];
        }
    }
}

/* Exact GELU: 0.5 x (1 + erf(x / sqrt 2)) (voc_gelu, src/tts_vocoder_ops.c:344-349). */
void oracle_voc_gelu(float *x, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) x[i] = 0.5f * x[i] * (1.0f + erff(x[i] * 0.7071067811865475f));
}

/* run_convnext (src/tts_vocoder.c:463-533) in place on x [C, T]:
 *   r = x; x = dwconv(x) + dw_b; x = LN_c(x); h = gelu(W1 x + b1) (W1 [4C, C]);
 *   x = W2 h + b2 (W2 [C, 4C]); x = x * gamma; x = x + r
 * scratch: 5 * C * T floats (the residual copy and h). */
void oracle_voc_convnext(float *x, const float *dw_w, const float *dw_b, const float *norm_w,
                         const float *norm_b, const float *pw1_w, const float *pw1_b,
                         const float *pw2_w, const float *pw2_b, const float *gamma, int C, int T,
                         float *scratch) {
    const size_t cT = (size_t)C * T;
    float *res = scratch, *h = scratch + cT;
    memcpy(res, x, cT * sizeof(float));
    oracle_voc_conv1d_depthwise(x, x, dw_w, dw_b, C, T, 7);
    oracle_voc_layer_norm_channels(x, norm_w, norm_b, C, T, 1e-6f);
    oracle_voc_conv1d_causal(h, x, pw1_w, pw1_b, C, 4 * C, T, 1, 1);
    oracle_voc_gelu(h, (int64_t)4 * cT);
    oracle_voc_conv1d_causal(x, h, pw2_w, pw2_b, 4 * C, C, T, 1, 1);
    for (int c = 0; c < C; c++)
        for (int t = 0; t < T; t++) x[(size_t)c * T + t] *= gamma[c];
    for (size_t i = 0; i < cT; i++) x[i] += res[i];
}

/* ---------------------------------------------------------------------------
 * Decode attention: one query token per sequence (qwen_causal_attention with
 * seq_q = 1 and q_offset = pos, src/tts_native.c:650-656; the math is the repo's numpy
 * specification tools/verify_xfmr.py:57-77: scores = q.k * scale, max-subtracted
 * softmax over keys 0..pos, weighted sum of v). GQA: query head h reads kv head
 * h / (n_heads / n_kv_heads). In the checker build scores, the softmax and the
 * weighted sum are accumulated in double.
 * ------------------------------------------------------------------------- */
void oracle_decode_attention(float *out, const float *q, const float *k_cache,
                             const float *v_cache, const int32_t *pos, int n_seqs, int n_heads,
                             int n_kv_heads, int head_dim, int max_seq, float scale) {
    const int kv_dim = n_kv_heads * head_dim, group = n_heads / n_kv_heads;
#pragma omp parallel for schedule(dynamic)
    for (int sh = 0; sh < n_seqs * n_heads; sh++) {
        const int s = sh / n_heads, h = sh % n_heads, kvh = h / group;
        const int L = pos[s] + 1;
        const float *qh = q + (size_t)s * n_heads * head_dim + (size_t)h * head_dim;
        const float *kc = k_cache + (size_t)s * max_seq * kv_dim + (size_t)kvh * head_dim;
        const float *vc = v_cache + (size_t)s * max_seq * kv_dim + (size_t)kvh * head_dim;
        float *o = out + (size_t)s * n_heads * head_dim + (size_t)h * head_dim;
        acc_t mx = -1e300;
        for (int j = 0; j < L; j++) {
            acc_t d = 0;
            for (int e = 0; e < head_dim; e++) d += (acc_t)qh[e] * kc[(size_t)j * kv_dim + e];
            d *= scale;
            if (d > mx) mx = d;
        }
        acc_t sum = 0;
        for (int e = 0; e < head_dim; e++) o[e] = 0.0f;
        acc_t accv[512];
        for (int e = 0; e < head_dim; e++) accv[e] = 0;
        for (int j = 0; j < L; j++) {
            acc_t d = 0;
            for (int e = 0; e < head_dim; e++) d += (acc_t)qh[e] * kc[(size_t)j * kv_dim + e];
            const acc_t p = exp((double)(d * scale - mx));
            sum += p;
            for (int e = 0; e < head_dim; e++) accv[e] += p * vc[(size_t)j * kv_dim + e];
        }
        for (int e = 0; e < head_dim; e++) o[e] = (float)(accv[e] / sum);
    }
}

/* ---------------------------------------------------------------------------
 * Repetition penalty (tts_apply_repetition_penalty, src/tts_sampling.c:19-36): every
 * distinct history token in [0, vocab) is penalised once.
 * ------------------------------------------------------------------------- */
void oracle_repetition_penalty(float *logits, int vocab, const int32_t *history, int history_len,
                               float penalty) {
    if (penalty <= 1.0f) return;
    for (int i = 0; i < history_len; i++) {
        const int tok = history[i];
        if (tok < 0 || tok >= vocab) continue;
        int dup = 0;
        for (int j = 0; j < i && !dup; j++) dup = history[j] == tok;
        if (dup) continue;
        logits[tok] = logits[tok] > 0.0f ? logits[tok] / penalty : logits[tok] * penalty;
    }
}

/* ---------------------------------------------------------------------------
 * Top-k sampling (tts_sample_topk, src/tts_sampling.c:40-109). The candidate list is
 * built in the reference's order: the first top_k tokens fill slots 0..k-1, then each
 * later token strictly above the current minimum replaces the slot holding it (the
 * first such slot), after which the minimum is searched again over the slots. The
 * softmax at the temperature and the cumulative walk run over the slots in that order
 * with float sums, and the first slot whose running sum reaches r = u * sum is taken
 * (slot 0 when none does). The order matters: it decides which token a given u picks.
 * ------------------------------------------------------------------------- */
int oracle_sample_topk(const float *logits, int vocab, float temperature, int top_k, float u,
                       float *margin, float *sum_out) {
    if (top_k <= 0 || top_k > vocab) top_k = vocab;
    float *val = (float *)malloc((size_t)top_k * sizeof(float));
    int *idx = (int *)malloc((size_t)top_k * sizeof(int));
    if (!val || !idx) {
        free(val);
        free(idx);
        return -1;
    }
    int slot_min = 0;
    for (int i = 0; i < top_k; i++) {
        val[i] = logits[i];
        idx[i] = i;
        if (logits[i] < val[slot_min]) slot_min = i;
    }
    for (int i = top_k; i < vocab; i++) {
        if (!(logits[i] > val[slot_min])) continue;
        val[slot_min] = logits[i];
        idx[slot_min] = i;
        slot_min = 0;
        for (int j = 1; j < top_k; j++)
            if (val[j] < val[slot_min]) slot_min = j;
    }
    float mx = val[0];
    for (int i = 1; i < top_k; i++)
        if (val[i] > mx) mx = val[i];
    float sum = 0.0f;
    for (int i = 0; i < top_k; i++) {
        val[i] = expf((val[i] - mx) / temperature);
        sum += val[i];
    }
    const float r = u * sum;
    float cum = 0.0f, best = INFINITY;
    int sel = idx[0], found = 0;
    for (int i = 0; i < top_k; i++) {
        cum += val[i];
        const float d = fabsf(cum - r);
        if (d < best) best = d;
        if (!found && cum >= r) {
            sel = idx[i];
            found = 1;
        }
    }
    if (margin) *margin = best;
    if (sum_out) *sum_out = sum;
    free(val);
    free(idx);
    return sel;
}

/* ---------------------------------------------------------------------------
 * Timed CPU reference: the elementwise ops of one decoder layer, FP32, in the
 * order talker_prefill calls them (src/tts_native.c:553-592), with the GEMM and
 * attention outputs supplied as inputs:
 *   add(x, ffn residual) ; rms_norm ; per-head q, k ; rope q, k ;
 *   add(x, attn residual) ; rms_norm ; swiglu
 * The reference compacts SwiGLU in place; in place is only safe serially, so
 * the multi-threaded timing writes it to gate_up's first half row by row
 * within each thread's rows (same bytes moved as in place).
 * ------------------------------------------------------------------------- */
void oracle_layer_chain_f32(float *x, const float *delta_attn, const float *delta_ffn,
                            float *x_norm, float *q, float *k, float *gate_up,
                            const float *w_in, const float *w_post, const float *wq,
                            const float *wk, const float *cos_t, const float *sin_t, int seq,
                            int dim, int n_q_heads, int n_kv_heads, int head_dim, int inter,
                            float eps) {
    oracle_add_inplace(x, delta_ffn, seq * dim);
    oracle_rms_norm(x_norm, x, w_in, seq, dim, eps);
    oracle_rms_norm_per_head(q, wq, seq, n_q_heads, head_dim, eps);
    oracle_rms_norm_per_head(k, wk, seq, n_kv_heads, head_dim, eps);
    oracle_apply_rope_neox(q, cos_t, sin_t, seq, n_q_heads, head_dim);
    oracle_apply_rope_neox(k, cos_t, sin_t, seq, n_kv_heads, head_dim);
    oracle_add_inplace(x, delta_attn, seq * dim);
    oracle_rms_norm(x_norm, x, w_post, seq, dim, eps);
#pragma omp parallel for schedule(static)
    for (int s = 0; s < seq; s++) {
        float *row = gate_up + (size_t)s * 2 * inter;
        for (int j = 0; j < inter; j++) row[j] = silu_mul(row[2 * j], row[2 * j + 1]);
    }
}

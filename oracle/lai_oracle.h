/*
 * lai_oracle.h - CPU restatement of local-ai-server's per-layer kernels.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg do, as the checker or as the timed CPU reference.
 *
 * The same source (lai_oracle.c) is compiled twice:
 *   liblai_oracle.so  - the parity checker: -O2 -ffp-contract=off, double
 *                       accumulation of sums of squares, single thread.
 *   liblai_cpuref.so  - the timed CPU baseline: the reference's optimisation
 *                       tier (Makefile:7, -O2 -march=native -ffast-math, here
 *                       -mavx2 -mfma so it runs on any x86-64 GPU host),
 *                       float accumulation, OpenMP over rows.
 *
 * Function names keep the reference's names with an "oracle_" prefix; argument
 * order and meaning follow the call sites cited in lai_oracle.c.
 */
#ifndef LAI_ORACLE_H
#define LAI_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference signatures (FP32, host memory) ---- */
void oracle_rms_norm(float *out, const float *x, const float *w, int seq, int dim, float eps);
void oracle_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim,
                              float eps);
void oracle_apply_rope_neox(float *x, const float *cos_t, const float *sin_t, int seq,
                            int n_heads, int head_dim);
void oracle_compute_rope_neox(float *cos_t, float *sin_t, const int *pos, int n, int head_dim,
                              float theta);
void oracle_rope_inv_freq(float *inv_freq, int head_dim, float theta);
void oracle_swiglu_multiply(float *out, const float *gate_up, int seq, int inter);
void oracle_swiglu_separate(float *out, const float *gate, const float *up, int n);
void oracle_add_inplace(float *x, const float *y, int n);
void oracle_silu(float *x, int n);
void oracle_snake_beta(float *x, const float *exp_alpha, const float *inv_exp_beta,
                       int channels, int T);
void oracle_embed_gather_bf16_to_f32(float *out, const uint16_t *table, const int32_t *ids,
                                     int n, int dim);
void oracle_embed_gather_bf16(uint16_t *out, const uint16_t *table, const int32_t *ids, int n,
                              int dim);

/* ---- position-indexed RoPE (device API semantics: row r uses table row pos[r]) ---- */
void oracle_apply_rope_neox_pos(float *x, const float *cos_t, const float *sin_t,
                                const int32_t *pos, int seq, int n_heads, int head_dim);

/* ---- BF16 storage variants: BF16 in/out, FP32 arithmetic, RNE rounding on store ---- */
uint16_t oracle_f32_to_bf16(float f);
float oracle_bf16_to_f32(uint16_t h);
void oracle_rms_norm_bf16(uint16_t *out, const uint16_t *x, const float *w, int seq, int dim,
                          float eps);
void oracle_add_rms_norm_bf16(uint16_t *x, const uint16_t *delta, const float *w, uint16_t *y,
                              int seq, int dim, float eps);
void oracle_add_rms_norm_f32(float *x, const float *delta, const float *w, float *y, int seq,
                             int dim, float eps);
void oracle_qk_norm_rope_bf16(uint16_t *q, uint16_t *k, const float *wq, const float *wk,
                              const float *cos_t, const float *sin_t, const int32_t *pos,
                              int seq, int n_q_heads, int n_kv_heads, int head_dim, float eps);
void oracle_qk_norm_rope_f32(float *q, float *k, const float *wq, const float *wk,
                             const float *cos_t, const float *sin_t, const int32_t *pos,
                             int seq, int n_q_heads, int n_kv_heads, int head_dim, float eps);
void oracle_swiglu_bf16(uint16_t *out, const uint16_t *gate_up, int seq, int inter);
void oracle_add_bf16(uint16_t *x, const uint16_t *y, int64_t n);

/* ---- linear_bf16 (src/tts_native.c:66-79): out[M,N] = in[M,K] @ W[N,K]^T, W BF16 ---- */
void oracle_linear_bf16(float *out, const float *in, const uint16_t *W, int M, int K, int N);

/* ---- causal self-attention over a sequence (qwen_causal_attention with T queries, as
 * src/tts_vocoder_xfmr.c:172-180 calls it; math tools/verify_xfmr.py:57-77) ----
 * q / out [T, H*hd], k / v [T, Hkv*hd]; row t attends keys 0..t; sums in acc_t. */
void oracle_causal_attention(float *out, const float *q, const float *k, const float *v, int T,
                             int n_heads, int n_kv_heads, int head_dim, float scale);

/* ---- the reference's other GPU weight formats (src/tts_pipeline.h:37-40,
 * src/tts_native.c:1185-1240; INT8 recipe tools/asr_benchmarks.md:342-352) ----
 * FP16 weights; INT8 weights with per-row scales, out = (sum_k q[n,k] x[m,k]) * scale[n];
 * F32 weights. oracle_quantize_rows_i8_bf16: scale = max|row| / 127 (F32),
 * q = roundf(w / scale) clamped to +-127, an all-zero row scale 0. IEEE binary16 <-> F32
 * conversions (exact decode; round-to-nearest-even encode, overflow to inf). */
float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);
void oracle_f32_to_f16_array(uint16_t *dst, const float *src, int64_t n);
void oracle_linear_f16(float *out, const float *in, const uint16_t *W, int M, int K, int N);
void oracle_linear_i8(float *out, const float *in, const int8_t *W, const float *scales, int M,
                      int K, int N);
void oracle_linear_f32(float *out, const float *in, const float *W, int M, int K, int N);
void oracle_quantize_rows_i8_bf16(int8_t *q, float *scales, const uint16_t *W, int N, int K);

/* ---- vocoder ResUnit, channels-first [C, T] F32 as the reference stores it ----
 * voc_conv1d_causal (src/tts_vocoder_ops.c:44-147, groups == 1): w [c_out, c_in, kernel] */
void oracle_voc_conv1d_causal(float *out, const float *in, const float *w, const float *bias,
                              int c_in, int c_out, int T, int kernel, int dilation);
/* run_resunit (src/tts_vocoder.c:540-583), in place on x; scratch holds 2 * C * T floats */
void oracle_voc_resunit(float *x, const float *ea1, const float *ieb1, const float *w1,
                        const float *b1, const float *ea2, const float *ieb2, const float *w2,
                        const float *b2, int C, int T, int dilation, float *scratch);

/* voc_conv_transpose1d (src/tts_vocoder_ops.c:153-221): w [c_in, c_out, kernel]; output
 * length (T + 1) * stride - kernel, trimming kernel - stride from each side */
void oracle_voc_conv_transpose1d(float *out, const float *in, const float *w, const float *bias,
                                 int c_in, int c_out, int T, int kernel, int stride);

/* ConvNeXt pieces (src/tts_vocoder_ops.c): depthwise causal conv (voc_conv1d_causal with
 * groups == channels, :52-73; w [C, 1, kernel]), LayerNorm over channels per time step
 * (voc_layer_norm_channels, :311-336), exact GELU (voc_gelu, :344-349); and the block
 * run_convnext (src/tts_vocoder.c:463-533) in place on x [C, T]; scratch 5 * C * T floats */
void oracle_voc_conv1d_depthwise(float *out, const float *in, const float *w, const float *bias,
                                 int channels, int T, int kernel);
void oracle_voc_layer_norm_channels(float *x, const float *w, const float *b, int channels, int T,
                                    float eps);
void oracle_voc_gelu(float *x, int64_t n);
void oracle_voc_convnext(float *x, const float *dw_w, const float *dw_b, const float *norm_w,
                         const float *norm_b, const float *pw1_w, const float *pw1_b,
                         const float *pw2_w, const float *pw2_b, const float *gamma, int C, int T,
                         float *scratch);

/* ---- decode attention, one query token per sequence (qwen_causal_attention with seq_q = 1,
 * src/tts_native.c:650-656; math of tools/verify_xfmr.py:57-77). q [n_seqs, n_heads*hd];
 * caches [n_seqs, max_seq, n_kv*hd]; keys 0..pos[s] (the reference appends the new k/v at
 * pos before attending, src/tts_native.c:650-651). Query head h reads kv head
 * h / (n_heads / n_kv). ---- */
void oracle_decode_attention(float *out, const float *q, const float *k_cache,
                             const float *v_cache, const int32_t *pos, int n_seqs, int n_heads,
                             int n_kv_heads, int head_dim, int max_seq, float scale);

/* ---- token sampling (src/tts_sampling.c) ----
 * tts_apply_repetition_penalty (:19-36): each distinct valid history token's logit is
 * divided by penalty if positive, else multiplied; nothing when penalty <= 1. */
void oracle_repetition_penalty(float *logits, int vocab, const int32_t *history, int history_len,
                               float penalty);
/* tts_sample_topk (:40-109) with the uniform draw u = rand()/RAND_MAX passed in instead of
 * taken from libc. Returns the token; *margin (may be NULL) receives the distance between
 * r = u * sum and the nearest cumulative boundary, *sum the softmax denominator. */
int oracle_sample_topk(const float *logits, int vocab, float temperature, int top_k, float u,
                       float *margin, float *sum);

/* ---- timed CPU reference: one decoder layer's elementwise chain, FP32, called in
 * the reference's own order (talker_prefill, src/tts_native.c:553-592) ---- */
void oracle_layer_chain_f32(float *x, const float *delta_attn, const float *delta_ffn,
                            float *x_norm, float *q, float *k, float *gate_up,
                            const float *w_in, const float *w_post, const float *wq,
                            const float *wk, const float *cos_t, const float *sin_t, int seq,
                            int dim, int n_q_heads, int n_kv_heads, int head_dim, int inter,
                            float eps);
int oracle_num_threads(void);
void oracle_set_threads(int n);

#ifdef __cplusplus
}
#endif
#endif

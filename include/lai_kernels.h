/*
 * lai_kernels.h - device-pointer C ABI of the B200 (sm_100a) per-layer kernels.
 *
 * Library: local-ai-server_b200/liblai_kernels.so. Plain C types only: device
 * pointers, element counts, a cudaStream_t (passed as void *; NULL = the legacy
 * default stream). Every entry returns LAI_OK (0) or a negative LAI_ERR_* code
 * and never synchronises the stream. Launch failures are reported from the
 * launch itself; data-dependent faults (an out-of-range token id or RoPE
 * position) never trap: the kernel skips that row and ORs a LAI_DEVERR_* bit
 * into the caller's device word `err` (may be NULL), which the caller reads
 * after synchronising.
 *
 * BF16 tensors are raw bit patterns (lai_bf16 = uint16_t). All arithmetic is
 * FP32; BF16 stores round to nearest even. Norm weights and RoPE tables are
 * FP32, as the reference keeps them (src/tts_native.c:125-133 load_f32,
 * src/tts_native.c:377-417).
 *
 * Reference functions replaced (their C source lives in the un-vendored qwen-asr
 * submodule; prototypes inferred from the call sites cited on each entry). The
 * exact reference-named, host-or-device FP32 drop-ins are in lai_qwen_dropin.h.
 */
#ifndef LAI_KERNELS_H
#define LAI_KERNELS_H

#include <stddef.h>
#include <stdint.h>

#ifndef LAI_API
#if defined(__GNUC__)
#define LAI_API __attribute__((visibility("default")))
#else
#define LAI_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef uint16_t lai_bf16;
typedef uint16_t lai_f16;   /* IEEE binary16 bit patterns */
typedef void *lai_stream_t; /* a cudaStream_t */

enum {
    LAI_OK = 0,
    LAI_ERR_INVALID = -1, /* bad size, NULL required pointer, unsupported head_dim */
    LAI_ERR_CUDA = -2,    /* a CUDA call or kernel launch failed */
    LAI_ERR_RANGE = -3,   /* an id / position was out of range (host-checked path) */
    LAI_ERR_ALIAS = -4,   /* output overlaps an input in an unsupported way */
    LAI_ERR_NOMEM = -5,   /* staging allocation failed (drop-in host path) */
    LAI_ERR_TOOBIG = -6   /* size beyond a stated maximum */
};

/* Bits ORed into the caller's device error word. LAI_DEVERR_TIMEOUT: a kernel's
 * bounded wait on its own asynchronous copies ran out (never expected; the kernel
 * drains what it issued and returns instead of hanging). LAI_DEVERR_SMEM_ALIGN: a
 * tensor-core kernel found its dynamic shared memory less than 1 KiB aligned and
 * computed nothing (never expected). */
enum { LAI_DEVERR_TOKEN_ID = 1, LAI_DEVERR_POSITION = 2, LAI_DEVERR_TIMEOUT = 4,
       LAI_DEVERR_SMEM_ALIGN = 8 };

LAI_API const char *lai_status_string(int status);
LAI_API int lai_version(void); /* major*10000 + minor*100 + patch */

/* ---- RMSNorm -------------------------------------------------------------
 * y[r,:] = x[r,:] / sqrt(mean(x[r,:]^2) + eps) * w      x,y [rows, dim], w [dim]
 * Replaces qwen_rms_norm(out, x, w, seq, dim, eps): src/tts_native.c:556, 584,
 * 637, 661, 674; src/tts_vocoder_xfmr.c:163, 189, 211. y == x is allowed.
 */
LAI_API int lai_rmsnorm_bf16(lai_bf16 *y, const lai_bf16 *x, const float *w, int64_t rows, int dim,
                     float eps, lai_stream_t stream);
LAI_API int lai_rmsnorm_f32(float *y, const float *x, const float *w, int64_t rows, int dim, float eps,
                    lai_stream_t stream);

/* ---- fused residual add + RMSNorm ------------------------------------------
 * x[r,:] += delta[r,:] (stored, BF16-rounded for the BF16 entry); y = RMSNorm(x).
 * Replaces the pair qwen_add_inplace(x, delta, seq*dim); qwen_rms_norm(y, x, w, ...)
 * at src/tts_native.c:582-584, 659-661, 738-740 (and the residual add at :591 /
 * :668 fused into the next layer's input norm at :556 / :637).
 * y must not overlap x or delta.
 */
LAI_API int lai_add_rmsnorm_bf16(lai_bf16 *x, const lai_bf16 *delta, const float *w, lai_bf16 *y,
                         int64_t rows, int dim, float eps, lai_stream_t stream);
LAI_API int lai_add_rmsnorm_f32(float *x, const float *delta, const float *w, float *y, int64_t rows,
                        int dim, float eps, lai_stream_t stream);

/* ---- fused per-head q/k RMSNorm + NeoX RoPE (in place) ----------------------
 * q [rows, n_q_heads*head_dim], k [rows, n_kv_heads*head_dim] (k may be NULL).
 * Per head: RMSNorm with wq / wk [head_dim] (NULL skips that norm), then NeoX
 * rotate-half with table row p = pos ? pos[r] : r of cos_t/sin_t [table_rows,
 * head_dim] (cos_t NULL skips RoPE). A row whose p is outside [0, table_rows) is
 * left unmodified and sets LAI_DEVERR_POSITION in *err.
 * Replaces qwen_rms_norm_per_head(q|k, w, seq, heads, hd, eps) x2 followed by
 * qwen_apply_rope_neox(q|k, cos, sin, seq, heads, hd) x2: src/tts_native.c:562-568,
 * 644-648, 724-730; src/tts_vocoder_xfmr.c:172-175 (RoPE only). head_dim even.
 */
LAI_API int lai_qk_norm_rope_bf16(lai_bf16 *q, lai_bf16 *k, const float *wq, const float *wk,
                          const float *cos_t, const float *sin_t, const int32_t *pos,
                          int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                          int head_dim, float eps, int *err, lai_stream_t stream);
LAI_API int lai_qk_norm_rope_f32(float *q, float *k, const float *wq, const float *wk,
                         const float *cos_t, const float *sin_t, const int32_t *pos,
                         int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                         int head_dim, float eps, int *err, lai_stream_t stream);

/* ---- RoPE table ---------------------------------------------------------------
 * cos_t/sin_t [n, head_dim]: row i holds cos/sin(p_i * inv_freq[d]) in both halves,
 * p_i = pos ? pos[i] : i, inv_freq[d] = 1/powf(theta, 2d/head_dim) computed on the
 * host exactly as ensure_rope_cache does (src/tts_native.c:377-417). Replaces
 * qwen_compute_rope_neox(cos, sin, pos, n, hd, theta): src/tts_vocoder_xfmr.c:150-156.
 * head_dim even, <= 512.
 */
LAI_API int lai_rope_table_f32(float *cos_t, float *sin_t, const int32_t *pos, int64_t n, int head_dim,
                       float theta, lai_stream_t stream);

/* ---- SwiGLU over the interleaved gate/up GEMM output ---------------------------
 * gate_up [rows, 2*inter] with rows interleaved [g0,u0,g1,u1,...] (fused weight,
 * src/tts_native.c:149-161); out[r,j] = silu(g[r,j]) * u[r,j], out [rows, inter].
 * out == gate_up compacts in place (the reference's call form, src/tts_native.c:588,
 * 665, 744) without scratch memory, using ordered passes; any other overlap is
 * LAI_ERR_ALIAS. Replaces qwen_swiglu_multiply(out, gate_up, seq, inter).
 */
LAI_API int lai_swiglu_bf16(lai_bf16 *out, const lai_bf16 *gate_up, int64_t rows, int inter,
                    lai_stream_t stream);
LAI_API int lai_swiglu_f32(float *out, const float *gate_up, int64_t rows, int inter,
                   lai_stream_t stream);

/* out[i] = silu(gate[i]) * up[i]: swiglu_separate, src/tts_vocoder_xfmr.c:73-80, 203. */
LAI_API int lai_swiglu_separate_f32(float *out, const float *gate, const float *up, int64_t n,
                            lai_stream_t stream);
/* x[i] = silu(x[i]) in place: qwen_silu(x, n), src/tts_native.c:504. */
LAI_API int lai_silu_f32(float *x, int64_t n, lai_stream_t stream);

/* ---- residual add: x[i] += y[i] ---------------------------------------------------
 * Replaces qwen_add_inplace(x, y, n): src/tts_native.c:582, 591, 659, 668, 738, 747,
 * 1142; src/tts_vocoder_xfmr.c:186, 206.
 */
LAI_API int lai_add_bf16(lai_bf16 *x, const lai_bf16 *y, int64_t n, lai_stream_t stream);
LAI_API int lai_add_f32(float *x, const float *y, int64_t n, lai_stream_t stream);

/* ---- BF16 token-embedding gather ----------------------------------------------------
 * out[r,:] = table[ids[r],:], table [vocab, dim] BF16; widened to F32 by the bit
 * shift of bf16_to_f32_row (bit-exact) or copied as BF16. An id outside [0, vocab)
 * zero-fills its row and sets LAI_DEVERR_TOKEN_ID in *err.
 * Replaces embed_lookup_bf16 / codec_embed_lookup (static, src/tts_native.c:35-40,
 * 473-476, 518-520; uses at :490-493, :930, :1121, :1138-1139).
 */
LAI_API int lai_embed_gather_bf16(lai_bf16 *out, const lai_bf16 *table, const int32_t *ids, int64_t n,
                          int dim, int64_t vocab, int *err, lai_stream_t stream);
LAI_API int lai_embed_gather_bf16_to_f32(float *out, const lai_bf16 *table, const int32_t *ids,
                                 int64_t n, int dim, int64_t vocab, int *err,
                                 lai_stream_t stream);

/* ---- SnakeBeta (in place, FP32) ---------------------------------------------------------
 * x [batch, channels, T]: x += inv_exp_beta[c] * sin(exp_alpha[c] * x)^2, params
 * pre-exponentiated (src/tts_vocoder.c:221-227). Replaces voc_snake_beta(x, ea, ieb,
 * channels, T) (src/tts_vocoder_ops.c:279-305; call sites src/tts_vocoder.c:548, 556,
 * 715, 745) for batch == 1, and a batch of such calls otherwise.
 */
LAI_API int lai_snake_beta_f32(float *x, const float *exp_alpha, const float *inv_exp_beta,
                       int64_t batch, int channels, int64_t T, lai_stream_t stream);

/* ---- decode-time linear layers with the layer's elementwise ops fused in -------------------
 * linear_bf16(out, in, W, M, K, N) computes out[M,N] = in[M,K] @ W[N,K]^T with BF16
 * weights and FP32 activations (src/tts_native.c:66-79). At decode (M = 1,
 * src/tts_native.c:637-667) the ops around it fuse in:
 *   lai_gemv_bf16w_f32:          y = W @ x, or W @ RMSNorm(x; norm_w, eps) when norm_w is
 *                                given  (qwen_rms_norm + q/k/v linear_bf16, :637-642)
 *   lai_gemv_residual_bf16w_f32: x_res += W @ a  (o_proj / down_proj linear_bf16 +
 *                                qwen_add_inplace, :658-659, :666-668)
 *   lai_gemv_swiglu_bf16w_f32:   out[m,j] = silu(W_gu[2j].xn) * (W_gu[2j+1].xn), xn = x or
 *                                RMSNorm(x)  (qwen_rms_norm + gate_up linear_bf16 +
 *                                qwen_swiglu_multiply, :661-665; rows interleaved :149-161)
 * x/a [M, K], outputs [M, N] (or [M, inter]); any M (passes of up to 8 rows); K*4 bytes
 * <= 200 KiB. Outputs must not overlap the inputs.
 */
LAI_API int lai_gemv_bf16w_f32(float *y, const float *x, const float *norm_w, float eps,
                               const lai_bf16 *W, int64_t M, int K, int N, lai_stream_t stream);
LAI_API int lai_gemv_residual_bf16w_f32(float *x_res, const float *a, const lai_bf16 *W,
                                        int64_t M, int K, int N, lai_stream_t stream);
LAI_API int lai_gemv_swiglu_bf16w_f32(float *out, const float *x, const float *norm_w, float eps,
                                      const lai_bf16 *W_gu, int64_t M, int K, int inter,
                                      lai_stream_t stream);

/* The same three decode linears over the reference's other GPU weight formats
 * (tts_pipeline_init's fp16 / int8 flags, src/tts_pipeline.h:37-40; upload_gpu_weights,
 * src/tts_native.c:1185-1240):
 *   _f16w: FP16 weights (its fp16 mode, and the codec head in int8 mode);
 *   _i8w:  INT8 weights with one F32 scale per output row, y = (q_row . x) * scale[row]
 *          (its int8 mode, tools/asr_benchmarks.md:342-352; make them with
 *          lai_quantize_rows_i8_bf16);
 *   _f32w: F32 weights (its default GPU mode).
 * Arguments, fusions and limits as for the BF16 entries above; the INT8 vector path
 * needs K % 16 == 0 (others fall back to scalar weight reads). */
LAI_API int lai_gemv_f16w_f32(float *y, const float *x, const float *norm_w, float eps,
                              const lai_f16 *W, int64_t M, int K, int N, lai_stream_t stream);
LAI_API int lai_gemv_residual_f16w_f32(float *x_res, const float *a, const lai_f16 *W, int64_t M,
                                       int K, int N, lai_stream_t stream);
LAI_API int lai_gemv_swiglu_f16w_f32(float *out, const float *x, const float *norm_w, float eps,
                                     const lai_f16 *W_gu, int64_t M, int K, int inter,
                                     lai_stream_t stream);
LAI_API int lai_gemv_i8w_f32(float *y, const float *x, const float *norm_w, float eps,
                             const int8_t *W, const float *scales, int64_t M, int K, int N,
                             lai_stream_t stream);
LAI_API int lai_gemv_residual_i8w_f32(float *x_res, const float *a, const int8_t *W,
                                      const float *scales, int64_t M, int K, int N,
                                      lai_stream_t stream);
LAI_API int lai_gemv_swiglu_i8w_f32(float *out, const float *x, const float *norm_w, float eps,
                                    const int8_t *W_gu, const float *scales, int64_t M, int K,
                                    int inter, lai_stream_t stream);
LAI_API int lai_gemv_f32w_f32(float *y, const float *x, const float *norm_w, float eps,
                              const float *W, int64_t M, int K, int N, lai_stream_t stream);
LAI_API int lai_gemv_residual_f32w_f32(float *x_res, const float *a, const float *W, int64_t M,
                                       int K, int N, lai_stream_t stream);
LAI_API int lai_gemv_swiglu_f32w_f32(float *out, const float *x, const float *norm_w, float eps,
                                     const float *W_gu, int64_t M, int K, int inter,
                                     lai_stream_t stream);

/* Load-time weight preparation (the reference converts BF16 safetensors when it uploads
 * weights, src/tts_native.c:1185-1240):
 *   lai_quantize_rows_i8_bf16: W [N, K] BF16 -> q [N, K] INT8 and scales [N] F32 with
 *     scale = max|row| / 127, q = round(w / scale) (halves away from zero), clamped to
 *     +-127; an all-zero row gets scale 0.
 *   lai_convert_bf16_to_f16: n values, round to nearest even (beyond FP16 range: +-inf). */
LAI_API int lai_quantize_rows_i8_bf16(int8_t *q, float *scales, const lai_bf16 *W, int N, int K,
                                      lai_stream_t stream);
LAI_API int lai_convert_bf16_to_f16(lai_f16 *dst, const lai_bf16 *src, int64_t n,
                                    lai_stream_t stream);

/* ---- a decode step's chain of fused GEMVs in one persistent kernel ------------------------
 * The M = 1 BF16 GEMVs above, run back to back as one cooperative launch (one CTA per SM):
 * op j reads what op j-1 wrote, as the per-layer decode sequence does (src/tts_native.c:
 * 637-668, each layer four ops: RMSNorm + q|k|v, o + residual, RMSNorm + gate|up + SwiGLU,
 * down + residual). Every CTA owns a fixed slice of rows of every matrix and streams its
 * slices of the coming ops into shared memory ahead of the dependency.
 *   epilogue LAI_CHAIN_STORE:    out[n]   = W . in'              (in' = RMSNorm(in; norm_w, eps)
 *            LAI_CHAIN_RESIDUAL: out[n]  += W . in'               when norm_w, else in)
 *            LAI_CHAIN_SWIGLU:   out[n/2] = silu(W[2j] . in') * (W[2j+1] . in')  (rows interleaved)
 * W [n, k] BF16, in/norm_w [k] FP32, all 16-byte aligned; k % 256 == 0 and k <= 6144
 * (LAI_ERR_TOOBIG beyond), at most 512 rows of an op per SM; out must not overlap in.
 * lai_gemv_chain_create validates the ops and copies the table to the device (synchronous, at
 * load time); lai_gemv_chain_run launches the chain on `stream` (capturable in a CUDA graph)
 * and sets *err (device int, never cleared) to 1 if a bounded wait in the kernel ran out.
 * Runs of one chain must not overlap in time (they share its grid counter).
 */
enum { LAI_CHAIN_STORE = 0, LAI_CHAIN_RESIDUAL = 1, LAI_CHAIN_SWIGLU = 2 };
typedef struct {
    const lai_bf16 *w;
    const float *in;
    const float *norm_w; /* NULL: no RMSNorm */
    float *out;
    int32_t n, k;
    int32_t epilogue; /* LAI_CHAIN_* */
    float eps;
} lai_gemv_chain_op_t;
typedef struct lai_gemv_chain lai_gemv_chain_t;
LAI_API int lai_gemv_chain_create(lai_gemv_chain_t **chain, const lai_gemv_chain_op_t *ops,
                                  int n_ops);
LAI_API int lai_gemv_chain_run(const lai_gemv_chain_t *chain, int *err, lai_stream_t stream);
LAI_API int lai_gemv_chain_grid(const lai_gemv_chain_t *chain); /* CTAs per launch */
LAI_API void lai_gemv_chain_destroy(lai_gemv_chain_t *chain);

/* ---- decode attention over the KV cache ----------------------------------------------------
 * One query token per sequence: the decode step's cache append + qwen_causal_attention
 * (src/tts_native.c:650-656: memcpy of k, v into kv_k_at / kv_v_at at pos, then
 * attention over keys 0..pos with scale 1/sqrt(hd)), for n_seqs independent sequences.
 *   q [n_seqs, n_heads*128] (RMSNorm'd + RoPE'd), k_new / v_new [n_seqs, n_kv*128]: this
 *   token's k (RMSNorm'd + RoPE'd) and v; k_cache / v_cache [n_seqs, max_seq, n_kv*128]
 *   (the reference's per-layer cache layout, one block per sequence); pos [n_seqs] device.
 * Writes out [n_seqs, n_heads*128] and k_new / v_new into cache row pos (the same launch).
 * Query head h reads kv head h / (n_heads / n_kv); n_heads / n_kv in {1, 2, 4, 8};
 * head_dim must be 128. scratch: lai_decode_attention_scratch_bytes() bytes, zeroed once
 * before first use (every call leaves it reusable). pos outside [0, max_seq) leaves that
 * sequence's output untouched and sets LAI_DEVERR_POSITION in *err.
 */
LAI_API size_t lai_decode_attention_scratch_bytes(int n_seqs, int n_heads, int n_kv_heads,
                                                  int max_seq);
LAI_API int lai_decode_attention_f32(float *out, const float *q, const float *k_new,
                                     const float *v_new, float *k_cache, float *v_cache,
                                     const int32_t *pos, int n_seqs, int n_heads, int n_kv_heads,
                                     int head_dim, int max_seq, float scale, void *scratch,
                                     int *err, lai_stream_t stream);
/* The same launch with the decode step's per-head q/k RMSNorm and NeoX RoPE folded in
 * (qwen_rms_norm_per_head + qwen_apply_rope_neox at the cache row, src/tts_native.c:644-648,
 * then :650-656): q and k_new are read raw and left unmodified, the attention uses the
 * normed, rotated q, and cache row pos receives the normed, rotated key. wq / wk [128] may be
 * NULL (no norm); cos_t / sin_t [table_rows, 128] both NULL (no RoPE) or both given, row pos
 * used; pos >= table_rows sets LAI_DEVERR_POSITION. */
LAI_API int lai_decode_attention_qk_f32(float *out, const float *q, const float *k_new,
                                        const float *v_new, float *k_cache, float *v_cache,
                                        const int32_t *pos, int n_seqs, int n_heads,
                                        int n_kv_heads, int head_dim, int max_seq, float scale,
                                        const float *wq, const float *wk, const float *cos_t,
                                        const float *sin_t, int64_t table_rows, float eps,
                                        void *scratch, int *err, lai_stream_t stream);

/* ---- causal self-attention over a whole sequence ------------------------------------------
 * qwen_causal_attention(out, q, k, v, T, T, n_heads, n_kv_heads, head_dim, scale, 0) as the
 * vocoder's pre-transformer calls it (src/tts_vocoder_xfmr.c:172-180): row t of q attends
 * keys 0..t. q / out [T, n_heads*head_dim], k / v [T, n_kv_heads*head_dim], F32, head_dim 64
 * or 128; query head h reads kv head h / (n_heads / n_kv_heads). */
LAI_API int lai_prefill_attention_f32(float *out, const float *q, const float *k, const float *v,
                                      int T, int n_heads, int n_kv_heads, int head_dim,
                                      float scale, lai_stream_t stream);
/* The same with the pre-transformer's NeoX RoPE (qwen_apply_rope_neox on q and k,
 * src/tts_vocoder_xfmr.c:172-175) folded in and row strides, so q / k / v can be the three
 * column blocks of one fused q|k|v projection output: q row t at q + t*ld_q, k / v rows at
 * + t*ld_kv; cos_t / sin_t [table_rows >= T, head_dim] give position t's row (both NULL:
 * no RoPE). out stays [T, n_heads*head_dim]. */
LAI_API int lai_prefill_attention_rope_f32(float *out, const float *q, const float *k,
                                           const float *v, int ld_q, int ld_kv, int T,
                                           int n_heads, int n_kv_heads, int head_dim, float scale,
                                           const float *cos_t, const float *sin_t,
                                           int64_t table_rows, lai_stream_t stream);

/* ---- token sampling on device logits ------------------------------------------------------
 * Per row r of logits [rows, vocab]: tts_apply_repetition_penalty(logits, vocab, history,
 * history_len, penalty) (src/tts_sampling.c:19-36; history [rows, history_stride] int32,
 * history_len [rows], both device, both NULL or neither; penalty <= 1 skips it), then
 * tts_sample_topk(logits, vocab, temperature, top_k) (:40-109) with its rand()/RAND_MAX
 * draw supplied as u[r] (device floats in [0, 1]); out_tokens[r] receives the token.
 * Same candidate order, softmax and cumulative walk as the reference, so the same u picks
 * the same token (up to the last bit of expf at a cumulative boundary). The penalty is
 * applied to logits in place, as the reference does. top_k <= 0 or > vocab means vocab.
 * LAI_ERR_TOOBIG when top_k * 8 + vocab / 8 bytes exceed 200 KiB.
 */
LAI_API int lai_sample_topk_f32(int32_t *out_tokens, float *logits, int vocab, int rows,
                                const int32_t *history, const int32_t *history_len,
                                int history_stride, float penalty, float temperature, int top_k,
                                const float *u, lai_stream_t stream);

/* run_decode_loop's bookkeeping around the sampler, on the device so a decode frame needs no
 * host round trip between its samples (src/tts_native.c:1092-1105):
 *   lai_logits_mask_range_f32: logits[r, c] = value for lo <= c < hi, c != keep (the
 *     suppression of [2048, 3072) except EOS with value -1e9);
 *   lai_history_append_i32: history[r, history_len[r]++] = tokens[r]; a full row
 *     (history_len[r] >= history_stride) is left as it is and sets LAI_DEVERR_POSITION. */
LAI_API int lai_logits_mask_range_f32(float *logits, int vocab, int rows, int lo, int hi,
                                      int keep, float value, lai_stream_t stream);
LAI_API int lai_history_append_i32(int32_t *history, int32_t *history_len, const int32_t *tokens,
                                   int rows, int history_stride, int *err, lai_stream_t stream);

/* ---- vocoder BigVGAN ResUnits on tensor cores ------------------------------------------------
 * run_resunit(x, ru, C, T, scratch) (src/tts_vocoder.c:540-583) for n_units consecutive
 * units, as tts_vocoder_run calls them per block (src/tts_vocoder.c:725-728):
 *   x = x + conv1x1(snake2(conv1d_causal(snake1(x), dilation))) with the biases
 * Activations are CHANNELS-LAST [batch, T, C] F32 (the reference stores [C, T]; convert
 * with lai_voc_transpose_f32). Snake parameters are pre-exponentiated as the reference
 * loads them (src/tts_vocoder.c:221-227). conv1_w / conv2_w are lai_voc_pack_conv_f32
 * images of the reference weights [C, C, 7] / [C, C, 1] (16-byte aligned).
 * scratch: 4 * batch * T * C floats (16-byte aligned, not overlapping x).
 * passes = 3: F32-faithful products (TF32 hi/lo split); passes = 1: plain TF32.
 * C must be a multiple of 32. A stalled pipeline wait ORs LAI_DEVERR_TIMEOUT into *err.
 */
typedef struct {
    const float *snake1_ea, *snake1_ieb; /* [C] exp(alpha), 1/exp(beta) of act1 */
    const float *conv1_w;                /* packed, 2 * 7 * C * C floats */
    const float *conv1_b;                /* [C] */
    const float *snake2_ea, *snake2_ieb; /* [C] of act2 */
    const float *conv2_w;                /* packed, 2 * C * C floats */
    const float *conv2_b;                /* [C] */
    int dilation;                        /* 1, 3, 9 in the reference (src/tts_vocoder.c:269) */
} lai_voc_resunit_t;

LAI_API int lai_voc_resunits_f32(float *x, float *scratch, const lai_voc_resunit_t *units,
                                 int n_units, int batch, int channels, int T, int passes,
                                 int *err, lai_stream_t stream);
/* ---- vocoder BigVGAN block: SnakeBeta -> ConvTranspose1d (kernel 2r, stride r) -> ResUnits --
 * One block of tts_vocoder_run (src/tts_vocoder.c:709-728): voc_snake_beta(x, snake) then
 * voc_conv_transpose1d (src/tts_vocoder_ops.c:153-221; T_out = (T - 1) r) then n_units
 * run_resunit calls. x [batch, T, c_in] -> out [batch, (T - 1) r, c_out], channels-last.
 * The transposed conv runs as r interleaved 2-tap convs on the tensor cores (output row
 * q r + f = W[.., f]^T x[q + 1] + W[.., r + f]^T x[q]); its epilogue also writes the first
 * unit's snake1 input. tconv_w: lai_voc_pack_tconv_f32 image of the reference weight
 * [c_in, c_out, 2r]. scratch: 2 batch T c_in + 4 batch T_out c_out floats. c_in, c_out
 * multiples of 32; T >= 2.
 */
typedef struct {
    const float *snake_ea, *snake_ieb; /* [c_in] the block's SnakeBeta, pre-exponentiated */
    const float *tconv_w;              /* lai_voc_pack_tconv_f32 image, kernel 2 * rate */
    const float *tconv_b;              /* [c_out] */
    int rate;                          /* 8, 5, 4, 3 in the reference (src/tts_vocoder.c:247) */
    int n_units;                       /* ResUnits that follow (3) */
    const lai_voc_resunit_t *units;    /* host array of n_units */
} lai_voc_bigvgan_block_t;

LAI_API int lai_voc_bigvgan_block_f32(float *out, const float *x, float *scratch,
                                      const lai_voc_bigvgan_block_t *blk, int batch, int c_in,
                                      int c_out, int T, int passes, int *err, lai_stream_t stream);
/* dst (2 * kernel * c_out * c_in floats) <- reference transposed-conv weight
 * w [c_in, c_out, kernel], kernel = stride or 2 * stride, regrouped per output phase into the
 * taps of the interleaved convs, TF32 high parts then remainders. */
LAI_API int lai_voc_pack_tconv_f32(float *dst, const float *w, int c_in, int c_out, int kernel,
                                   int stride, lai_stream_t stream);

/* ---- the vocoder decoder's other convolutions (channels-last [batch, T, C] F32) ------------
 * lai_voc_conv1d_f32: voc_conv1d_causal (src/tts_vocoder_ops.c:44-147, groups 1) with w the
 *   lai_voc_pack_conv_f32 image of [c_out, c_in, kernel]: out [batch, T, c_out] = conv(x) + bias
 *   (the BigVGAN init conv 1024 -> 1536, k=7, src/tts_vocoder.c:694-697). scratch:
 *   2 * batch * T * c_in floats.
 * lai_voc_conv_transpose1d_f32: voc_conv_transpose1d (:153-221) for kernel = stride (the
 *   ConvNeXt upsample stages, src/tts_vocoder.c:658-667) or 2 * stride, w the
 *   lai_voc_pack_tconv_f32 image; out [batch, (T + 1) stride - kernel, c_out]. scratch:
 *   2 * batch * T * c_in floats.
 * lai_voc_final_f32: the decoder's last step (src/tts_vocoder.c:748-758): voc_snake_beta over
 *   x [batch, T, channels], conv1d channels -> 1 (k = 7, w [1, channels, 7] as loaded, bias [1]),
 *   clamp to [-1, 1]; audio [batch, T]. channels in {32, 64, 96, 128} (the reference: 96).
 * c_in, c_out multiples of 32; passes as for the ResUnits.
 */
LAI_API int lai_voc_conv1d_f32(float *out, const float *x, float *scratch, const float *w,
                               const float *bias, int batch, int c_in, int c_out, int T,
                               int kernel, int dilation, int passes, int *err,
                               lai_stream_t stream);
LAI_API int lai_voc_conv_transpose1d_f32(float *out, const float *x, float *scratch,
                                         const float *w, const float *bias, int batch, int c_in,
                                         int c_out, int T, int kernel, int stride, int passes,
                                         int *err, lai_stream_t stream);
LAI_API int lai_voc_final_f32(float *audio, const float *x, const float *exp_alpha,
                              const float *inv_exp_beta, const float *w, const float *bias,
                              int batch, int channels, int T, lai_stream_t stream);

/* The vocoder's front (tts_vocoder_run stages 1 and 3, src/tts_vocoder.c:589-640):
 *   lai_voc_rvq_gather_f32: RVQ decode's lookups (rvq_decode, :428-455) as one gather,
 *     out [T, n_codebooks*dim] = row t holds codebooks[cb][codes[t, cb]] for cb in order;
 *     codebooks packed [n_codebooks*codebook_size, dim] F32, codes int64 [T, n_codebooks] as
 *     the reference passes them (out-of-range: zero row, LAI_DEVERR_TOKEN_ID). One GEMM
 *     against the n_codebooks projections laid side by side ([512, n_codebooks*dim], e.g. via
 *     lai_voc_conv1d_f32 with kernel 1) then sums the codebooks.
 *   lai_voc_linear_scale_residual_f32: x_res [rows, c_out] += gamma * (in [rows, c_in] . W^T
 *     + bias), the pre-transformer's o / down projection with LayerScale and residual
 *     (src/tts_vocoder_xfmr.c:182-186, 203-207); W packed by lai_voc_pack_conv_f32 (kernel 1);
 *     scratch 2*rows*c_in floats; c_in, c_out multiples of 32; passes 1 or 3 as for the convs. */
LAI_API int lai_voc_rvq_gather_f32(float *out, const float *codebooks, const int64_t *codes,
                                   int T, int n_codebooks, int codebook_size, int dim, int *err,
                                   lai_stream_t stream);
LAI_API int lai_voc_linear_scale_residual_f32(float *x_res, const float *in, float *scratch,
                                              const float *w, const float *bias,
                                              const float *gamma, int rows, int c_in, int c_out,
                                              int passes, int *err, lai_stream_t stream);

/* ---- vocoder ConvNeXt block (upsample stages) --------------------------------------------
 * run_convnext(x, C, T, cn) (src/tts_vocoder.c:463-533): depthwise causal conv k=7 + bias,
 * LayerNorm over channels (eps 1e-6), pointwise C -> 4C + bias, exact GELU, pointwise
 * 4C -> C + bias, * gamma, + residual; in place on channels-last x [batch, T, C].
 * C in {128, 256, 512, 1024, 2048} (the reference: 1024). scratch: 10 * batch * T * C
 * floats. passes as for the ResUnits. dw_b, norm_w, norm_b 16-byte aligned.
 */
typedef struct {
    const float *dw_w;             /* [C, 1, 7] depthwise weight, as loaded */
    const float *dw_b;             /* [C] */
    const float *norm_w, *norm_b;  /* [C] LayerNorm scale, shift */
    const float *pw1_w;            /* lai_voc_pack_conv_f32 image of [4C, C, 1] */
    const float *pw1_b;            /* [4C] */
    const float *pw2_w;            /* lai_voc_pack_conv_f32 image of [C, 4C, 1] */
    const float *pw2_b;            /* [C] */
    const float *gamma;            /* [C] layer scale */
} lai_voc_convnext_t;

LAI_API int lai_voc_convnext_f32(float *x, float *scratch, const lai_voc_convnext_t *p, int batch,
                                 int channels, int T, int passes, int *err, lai_stream_t stream);

/* dst (2 * c_out * c_in * kernel floats) <- reference conv weight w [c_out, c_in, kernel]
 * regrouped per tap as [2][kernel][c_out][c_in]: TF32 high parts, then the remainders. */
LAI_API int lai_voc_pack_conv_f32(float *dst, const float *w, int c_out, int c_in, int kernel,
                                  lai_stream_t stream);
/* dst[b][j][i] = src[b][i][j] for src [batch, rows, cols]: [C, T] <-> [T, C]. */
LAI_API int lai_voc_transpose_f32(float *dst, const float *src, int batch, int rows, int cols,
                                  lai_stream_t stream);

/* ---- seeded synthetic inputs (bench and test support) ------------------------------------
 * Counter-based: element i of a fill is a pure function of (seed, offset + i), so a
 * row-sharded fill on G devices equals the single-device fill of the same rows.
 * normal: mean + std * N(0,1); uniform ints in [lo, hi).
 */
LAI_API int lai_synth_normal_bf16(lai_bf16 *out, int64_t n, uint64_t seed, int64_t offset, float mean,
                          float std, lai_stream_t stream);
LAI_API int lai_synth_normal_f32(float *out, int64_t n, uint64_t seed, int64_t offset, float mean,
                         float std, lai_stream_t stream);
LAI_API int lai_synth_uniform_i32(int32_t *out, int64_t n, uint64_t seed, int64_t offset, int32_t lo,
                          int32_t hi, lai_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* LAI_KERNELS_H */

/*
 * lai_qwen_dropin.h - the reference's own kernel names, served by the B200 kernels.
 *
 * Library: local-ai-server_b200/liblai_kernels.so. These are the exact prototypes
 * the reference's C calls (FP32, void return). Their source lives in the
 * un-vendored qwen-asr submodule (qwen_asr_kernels.h, included at
 * src/tts_native.c:13, src/tts_vocoder_ops.c:10, src/tts_vocoder_xfmr.c:12), so
 * the prototypes are inferred from the call sites cited below; voc_snake_beta is
 * declared in the present header src/tts_vocoder.h:254-255.
 *
 * Pointer modes (decided per argument with cudaPointerGetAttributes):
 *   - device or managed memory: the kernel runs in place on the drop-in stream
 *     (lai_set_stream; default the legacy default stream); the call returns once
 *     the work is queued, like any CUDA library call.
 *   - host memory (pinned or pageable): rows are staged through device buffers
 *     in a 3-stream pipeline (copy-in, kernel, copy-out overlap across chunks);
 *     the call returns when the results are back in host memory, as the
 *     reference's CPU functions do. Pinned buffers copy at full PCIe speed.
 * There is no CPU fallback: without a usable GPU every call fails.
 *
 * Errors: the functions stay void like the reference's; a failure prints one
 * line to stderr and is kept for lai_last_error() (thread-local).
 */
#ifndef LAI_QWEN_DROPIN_H
#define LAI_QWEN_DROPIN_H

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

/* src/tts_native.c:556, 584, 637, 661, 674 (out == x); src/tts_vocoder_xfmr.c:163, 189, 211 */
LAI_API void qwen_rms_norm(float *out, const float *x, const float *w, int seq, int dim, float eps);
/* No counterpart in the reference. qwen_rms_norm's host-buffer semantics (out may
 * equal x; host or device pointers) for callers that cannot let a library
 * allocate device memory -- a process whose memory belongs to its own pool
 * allocator, or a loop that must not meet cudaMalloc/cudaFree's device-wide
 * synchronisation. It stages through a fixed 8 MiB array compiled into the
 * library (held on every GPU that loads it) and calls no allocator: seq*dim*4
 * plus dim*4 bytes (each rounded up to 256) must fit in 8 MiB, else
 * LAI_ERR_TOOBIG. With CUDA's default lazy module loading the array is claimed
 * when the library's device code first loads on a device, which is inside the
 * first call there: make that first call (or set CUDA_MODULE_LOADING=EAGER)
 * before a pool allocator reserves the device's memory, and before any stream
 * capture. Calls share the array: calls whose GPU work overlaps (several threads
 * or streams on one device) race; the call synchronises `stream` before it
 * returns, on error paths too. Returns a LAI_* status. */
LAI_API int lai_rmsnorm_f32_host_noalloc(float *out, const float *x, const float *w, int seq,
                                         int dim, float eps, void *stream);
/* src/tts_native.c:562-563, 644-645, 724-725 (in place) */
LAI_API void qwen_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim,
                            float eps);
/* src/tts_native.c:565-568 (table rows 0..seq-1), 647-648 (pointer at row pos, seq 1);
 * src/tts_vocoder_xfmr.c:172-175 */
LAI_API void qwen_apply_rope_neox(float *x, const float *cos, const float *sin, int seq, int n_heads,
                          int head_dim);
/* src/tts_vocoder_xfmr.c:150-156 */
LAI_API void qwen_compute_rope_neox(float *cos, float *sin, const int *pos, int n, int head_dim,
                            float theta);
/* src/tts_native.c:588, 665, 744 (out == gate_up, interleaved rows) */
LAI_API void qwen_swiglu_multiply(float *out, const float *gate_up, int seq, int inter);
/* src/tts_native.c:582, 591, 659, 668, 738, 747, 1142; src/tts_vocoder_xfmr.c:186, 206 */
LAI_API void qwen_add_inplace(float *x, const float *y, int n);
/* src/tts_native.c:504 */
LAI_API void qwen_silu(float *x, int n);
/* src/tts_vocoder.h:254-255; call sites src/tts_vocoder.c:548, 556, 715, 745 */
LAI_API void voc_snake_beta(float *x, const float *exp_alpha, const float *inv_exp_beta, int channels,
                    int T);

/* Synchronous, pointer-agnostic BF16 fused ops: the lai_kernels.h entries of the same
 * name without "_staged", for callers whose rows live in host memory. Every argument
 * may be host (pinned or pageable) or device memory; host rows go through the same
 * 3-stream staging pipeline as the qwen_* drop-ins, and the call returns when the
 * outputs are in place (LAI_* status). For the qk entry the cos/sin tables
 * [table_rows, head_dim] are copied whole and pos per row; pos NULL means row index.
 * Replace, on BF16 activations, the call pairs / quadruples cited in lai_kernels.h. */
LAI_API int lai_staged_add_rmsnorm_bf16(uint16_t *x, const uint16_t *delta, const float *w,
                                        uint16_t *y, int64_t rows, int dim, float eps);
LAI_API int lai_staged_qk_norm_rope_bf16(uint16_t *q, uint16_t *k, const float *wq,
                                         const float *wk, const float *cos_t,
                                         const float *sin_t, const int32_t *pos,
                                         int64_t table_rows, int64_t rows, int n_q_heads,
                                         int n_kv_heads, int head_dim, float eps);
LAI_API int lai_staged_swiglu_bf16(uint16_t *out, const uint16_t *gate_up, int64_t rows,
                                   int inter);

/* The static helper embed_lookup_bf16(dst, table, token_id, dim) of
 * src/tts_native.c:473-476 (a call-site one-liner forwards to this). The table
 * must be device memory, managed memory or host memory registered with
 * lai_register_host_table (it is read in place, one row per call); dst may be
 * host or device memory. vocab bounds the id (pass 0 to skip the check, which is
 * the reference's behaviour). */
LAI_API void lai_embed_lookup_bf16(float *dst, const uint16_t *table, int token_id, int dim,
                           int64_t vocab);
/* Pin and map a host table (e.g. the mmap'd BF16 embedding) for in-place reads. */
LAI_API int lai_register_host_table(const void *table, size_t bytes);
LAI_API int lai_unregister_host_table(const void *table);

/* Drop-in state (per calling thread). */
LAI_API int lai_last_error(void);             /* last LAI_* status of this thread, then cleared */
LAI_API void lai_set_stream(void *stream);    /* stream for device-pointer calls (NULL = legacy) */
LAI_API void *lai_get_stream(void);
LAI_API int lai_device_error_flags(void);     /* syncs, returns and clears LAI_DEVERR_* bits of
                                         device-pointer calls on this thread */
LAI_API void lai_shutdown(void);              /* frees this thread's staging buffers and streams */

#ifdef __cplusplus
}
#endif
#endif /* LAI_QWEN_DROPIN_H */

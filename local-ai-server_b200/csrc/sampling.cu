// sampling.cu - repetition penalty + top-k token sampling on device logits, one CTA per row.
//
// Reference: tts_apply_repetition_penalty (src/tts_sampling.c:19-36) and tts_sample_topk
// (:40-109), called once per decode step on the talker's codec logits
// (src/tts_native.c:1096-1099) and per code-predictor group (:1132).
//
// The token the reference picks for a given random draw depends on the ORDER of its
// candidate slots: the first top_k tokens fill the slots, then each later token strictly
// above the current minimum replaces the slot that holds it (first such slot), and the
// softmax / cumulative walk runs over the slots in that order. This kernel replays that
// scan exactly: warp 0 tests 32 tokens per ballot against the current minimum, applies
// the qualifying tokens one at a time in index order (the lowest set lane first, the
// minimum re-found by a warp-wide first-argmin over the slots after each), and re-tests
// the rest of the chunk against the new minimum. For top_k <= 64 the slots live in
// registers, two per lane, and the first-argmin is two hardware warp min-reductions (an
// order-preserving integer key of the value, then the lowest slot among the lanes holding
// it) instead of a shuffle tree over shared memory; larger top_k keep the slots in shared
// memory. Either way the replacements happen in the same order. One thread then runs the softmax and the
// cumulative walk sequentially so the float sums round in the reference's order. The
// uniform draw the reference takes from libc rand() comes in as u[row].
//
// The penalty marks each history token's bit in a shared-memory bitmap with atomicOr; the
// thread that sets the bit penalises the logit, so every distinct token is penalised once
// whatever the order of the history, as in the reference.
//
// Latency. The scan is sequential by nature (each replacement depends on the slots before
// it), so its per-chunk cost is the row's critical path: when the row fits (vocab floats
// within the shared-memory budget; the codec vocabularies are 12 and 8 KiB) all 256 threads
// first stage it into shared memory in one parallel pass and warp 0 scans that copy, instead
// of waiting on a global load per 32-token chunk (measured: one 3072-token row 100 us -> a
// few us, the decode frame's 16 samples were a quarter of its time).
#include "lai_common.cuh"

#include <float.h>
#include <limits.h>

namespace lai {
namespace {

constexpr int kThreads = 256;

// first index of the minimum over v[0..n): lowest index among equal minima
__device__ __forceinline__ void warp_argmin_first(const float *v, int n, float &mv, int &mi) {
    const int lane = threadIdx.x & 31;
    float bv = FLT_MAX;
    int bi = INT_MAX;
    for (int j = lane; j < n; j += 32) {
        const float x = v[j];
        if (bi == INT_MAX || x < bv) {  // strict: keeps this lane's first minimum
            bv = x;
            bi = j;
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov < bv || (ov == bv && oi < bi)) {
            bv = ov;
            bi = oi;
        }
    }
    mv = bv;
    mi = bi;
}

// Shared memory: k slot values, k slot indices, the penalty bitmap, then (staged) the row.
__host__ __device__ inline size_t sample_smem_bytes(int vocab, int k, bool staged) {
    const size_t words = (size_t)(vocab + 31) / 32;
    return (size_t)k * 8 + words * 4 + (staged ? (size_t)vocab * 4 : 0);
}

// Order-preserving 32-bit key of a float (smaller value <-> smaller key; -0 and +0 equal, as
// they compare equal), for the warp's hardware min-reduction.
__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// First minimum over the k <= 64 slots held two per lane (lane L: slots L and L + 32):
// min key over the warp, then the lowest slot index among the slots holding it.
__device__ __forceinline__ void reg_argmin_first(const float (&v)[2], int k, float &mv, int &mi) {
    const int lane = threadIdx.x & 31;
    uint32_t kb = 0xffffffffu;
    int ib = INT_MAX;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int slot = lane + 32 * h;
        if (slot < k) {
            const uint32_t key = order_key(v[h]);
            if (key < kb) {  // strict: slot L before slot L + 32 on a tie
                kb = key;
                ib = slot;
            }
        }
    }
    const uint32_t kmin = __reduce_min_sync(0xffffffffu, kb);
    mi = (int)__reduce_min_sync(0xffffffffu, kb == kmin ? (uint32_t)ib : 0xffffffffu);
    mv = __shfl_sync(0xffffffffu, mi < 32 ? v[0] : v[1], mi & 31);
}

__global__ void __launch_bounds__(kThreads)
sample_topk_kernel(int32_t *out, float *logits, int vocab, int64_t ld, const int32_t *history,
                   const int32_t *hist_len, int hist_stride, float penalty, float temperature,
                   int k, const float *u, int staged) {
    extern __shared__ uint8_t smem_raw[];
    float *sv = reinterpret_cast<float *>(smem_raw);
    int *si = reinterpret_cast<int *>(sv + k);
    uint32_t *seen = reinterpret_cast<uint32_t *>(si + k);
    float *srow = reinterpret_cast<float *>(seen + (vocab + 31) / 32);
    const int row = blockIdx.x, tid = threadIdx.x;
    float *lg = logits + (size_t)row * ld;
    pdl_wait_prior();  // the logits come from the kernel before (programmatic launch)
    pdl_launch_dependents();

    if (penalty > 1.0f && history && hist_len) {
        const int words = (vocab + 31) / 32;
        for (int w = tid; w < words; w += kThreads) seen[w] = 0u;
        __syncthreads();
        const int n = min(hist_len[row], hist_stride);  // never past this row's history
        const int32_t *h = history + (size_t)row * hist_stride;
        for (int i = tid; i < n; i += kThreads) {
            const int tok = h[i];
            if (tok < 0 || tok >= vocab) continue;
            const uint32_t bit = 1u << (tok & 31);
            if (atomicOr(&seen[tok >> 5], bit) & bit) continue;
            const float v = lg[tok];
            lg[tok] = v > 0.0f ? v / penalty : v * penalty;
        }
        __syncthreads();
    }
    // the (penalised) row the scan reads: a shared-memory copy when it fits
    const float *scan = lg;
    if (staged) {
        for (int i = tid; i < vocab; i += kThreads) srow[i] = lg[i];
        scan = srow;
    }
    __syncthreads();
    for (int i = tid; i < k; i += kThreads) {
        sv[i] = scan[i];
        si[i] = i;
    }
    __syncthreads();
    if (tid < 32 && k <= 64) {
        // the slots in registers, two per lane; the same scan and replacements as below
        const int lane = tid;
        float rv[2];
        int ri[2];
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int slot = lane + 32 * h;
            rv[h] = slot < k ? sv[slot] : 0.0f;
            ri[h] = slot;
        }
        float mv;
        int mi;
        reg_argmin_first(rv, k, mv, mi);
        for (int i0 = k; i0 < vocab; i0 += 32) {
            const int i = i0 + lane;
            const bool valid = i < vocab;
            const float v = valid ? scan[i] : 0.0f;
            uint32_t mask = __ballot_sync(0xffffffffu, valid && v > mv);
            while (mask) {
                const int f = __ffs(mask) - 1;
                const float vf = __shfl_sync(0xffffffffu, v, f);
                if (lane == (mi & 31)) {  // the lane holding the minimum slot replaces it
                    rv[mi >> 5] = vf;
                    ri[mi >> 5] = i0 + f;
                }
                reg_argmin_first(rv, k, mv, mi);
                mask = __ballot_sync(0xffffffffu, valid && lane > f && v > mv);
            }
        }
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int slot = lane + 32 * h;
            if (slot < k) {
                sv[slot] = rv[h];
                si[slot] = ri[h];
            }
        }
        __syncwarp();
    } else if (tid < 32) {
        const int lane = tid;
        float mv;
        int mi;
        warp_argmin_first(sv, k, mv, mi);
        for (int i0 = k; i0 < vocab; i0 += 32) {
            const int i = i0 + lane;
            const bool valid = i < vocab;
            const float v = valid ? scan[i] : 0.0f;
            uint32_t mask = __ballot_sync(0xffffffffu, valid && v > mv);
            while (mask) {
                const int f = __ffs(mask) - 1;
                const float vf = __shfl_sync(0xffffffffu, v, f);
                if (lane == 0) {
                    sv[mi] = vf;
                    si[mi] = i0 + f;
                }
                __syncwarp();
                warp_argmin_first(sv, k, mv, mi);
                mask = __ballot_sync(0xffffffffu, valid && lane > f && v > mv);
            }
        }
    }
    if (tid == 0) {  // softmax and cumulative walk over the slots in their order
        float mx = sv[0];
        for (int j = 1; j < k; j++)
            if (sv[j] > mx) mx = sv[j];
        float sum = 0.0f;
        for (int j = 0; j < k; j++) {
            sv[j] = expf((sv[j] - mx) / temperature);
            sum += sv[j];
        }
        const float r = u[row] * sum;
        float cum = 0.0f;
        int sel = si[0];
        for (int j = 0; j < k; j++) {
            cum += sv[j];
            if (cum >= r) {
                sel = si[j];
                break;
            }
        }
        out[row] = sel;
    }
}

}  // namespace
}  // namespace lai

extern "C" int lai_sample_topk_f32(int32_t *out_tokens, float *logits, int vocab, int rows,
                                   const int32_t *history, const int32_t *history_len,
                                   int history_stride, float penalty, float temperature,
                                   int top_k, const float *u, lai_stream_t stream) {
    using namespace lai;
    if (!out_tokens || !logits || !u || vocab <= 0 || rows < 0 ||
        ((history == nullptr) != (history_len == nullptr)) || history_stride < 0)
        return LAI_ERR_INVALID;
    if (rows == 0) return LAI_OK;
    const int k = (top_k <= 0 || top_k > vocab) ? vocab : top_k;
    const bool staged = sample_smem_bytes(vocab, k, true) <= 160 * 1024;
    const size_t smem = sample_smem_bytes(vocab, k, staged);
    if (smem > 200 * 1024) return LAI_ERR_TOOBIG;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(sample_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return LAI_ERR_CUDA;
    launch_pdl(sample_topk_kernel, dim3(rows), dim3(kThreads), smem, as_stream(stream),
               out_tokens, logits, vocab, (int64_t)vocab, history, history_len, history_stride,
               penalty, temperature, k, u, staged ? 1 : 0);
    return launch_status();
}

namespace lai {
namespace {

__global__ void mask_range_kernel(float *logits, int64_t vocab, int rows, int lo, int hi,
                                  int keep, float value) {
    pdl_wait_prior();
    pdl_launch_dependents();
    const int64_t n = (int64_t)rows * (hi - lo);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / (hi - lo);
        const int c = lo + (int)(i - r * (hi - lo));
        if (c != keep) logits[r * vocab + c] = value;
    }
}

__global__ void history_append_kernel(int32_t *history, int32_t *len, const int32_t *tokens,
                                      int rows, int stride, int *err) {
    pdl_wait_prior();
    pdl_launch_dependents();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int n = len[r];
    if (n < 0 || n >= stride) {  // full: the token is not recorded
        if (err) atomicOr(err, LAI_DEVERR_POSITION);
        return;
    }
    history[(int64_t)r * stride + n] = tokens[r];
    len[r] = n + 1;
}

}  // namespace
}  // namespace lai

// Suppression before sampling (run_decode_loop, src/tts_native.c:1092-1095: logits
// [suppress_start, vocab) set to -1e9 except EOS).
extern "C" int lai_logits_mask_range_f32(float *logits, int vocab, int rows, int lo, int hi,
                                         int keep, float value, lai_stream_t stream) {
    using namespace lai;
    if (!logits || vocab <= 0 || rows < 0 || lo < 0 || hi > vocab || lo > hi)
        return LAI_ERR_INVALID;
    if (rows == 0 || lo == hi) return LAI_OK;
    const int64_t n = (int64_t)rows * (hi - lo);
    launch_pdl(mask_range_kernel, dim3(grid_for(n, 256)), dim3(256), 0, as_stream(stream),
               logits, (int64_t)vocab, rows, lo, hi, keep, value);
    return launch_status();
}

// cb0_history[history_len++] = cb0 (src/tts_native.c:1105) for each row, on the device.
extern "C" int lai_history_append_i32(int32_t *history, int32_t *history_len,
                                      const int32_t *tokens, int rows, int history_stride,
                                      int *err, lai_stream_t stream) {
    using namespace lai;
    if (!history || !history_len || !tokens || rows < 0 || history_stride <= 0)
        return LAI_ERR_INVALID;
    if (rows == 0) return LAI_OK;
    launch_pdl(history_append_kernel, dim3((rows + 127) / 128), dim3(128), 0, as_stream(stream),
               history, history_len, tokens, rows, history_stride, err);
    return launch_status();
}

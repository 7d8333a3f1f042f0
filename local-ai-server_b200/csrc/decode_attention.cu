// decode_attention.cu - one query token per sequence attending over its KV cache (GQA,
// head_dim 128, F32 cache), with the token's own k/v appended to the cache by the same
// launch.
//
// Reference: the decode step (src/tts_native.c:634-656) copies the RoPE'd k and v of
// position pos into the layer's cache (kv_k_at / kv_v_at, :324-332, layout
// [layer][max_seq][n_kv * hd] F32, :650-651) and calls
// qwen_causal_attention(out, q, K, V, 1, pos + 1, n_heads, n_kv, hd, 1/sqrt(hd), pos)
// (:653-655; body in the absent qwen-asr submodule, math as tools/verify_xfmr.py:57-77:
// scores q.k * scale, max-subtracted softmax over keys 0..pos, weighted sum of v).
// Query head h reads kv head h / (n_heads / n_kv).
//
// Work split (flash-decoding): CTA (split, kv head, sequence) takes keys
// [256 split, 256 split + 256) of that sequence for all G = n_heads / n_kv query heads
// of the kv head, so each K/V row is read from HBM once per step. A half-warp owns a key
// (16 lanes x 8 dims = 128), both half-warps of a warp walk their own key streams, 4
// keys per half-warp in flight; scores live in log2 units (q pre-scaled by
// scale * log2 e) under an online softmax (running max, sum, 8 accumulator dims per
// lane). Half-warps, then warps, merge by log-sum-exp. A sequence of one split writes
// its output directly; otherwise each split leaves (max, sum, acc[128]) per head in
// scratch and the CTA that finishes last (atomic counter per (sequence, kv head))
// merges them and resets the counter to zero. The split holding key pos reads that key
// from k_new / v_new and writes it into the cache row.
//
// Roofline: HBM, 2 * (pos + 1) * hd * 4 bytes of K and V per (sequence, kv head).
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kHD = 128;
constexpr int kChunk = 256;  // keys per CTA
constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kUnroll = 4;   // keys per half-warp with loads in flight
constexpr int kPartial = kHD + 2;  // (max, sum, acc[128]) per (sequence, head, split)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kNegBig = -1e30f;  // finite "minus infinity": merges of empty states stay 0

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }

// Per-head q/k transform of the fused entry (lai_decode_attention_qk_f32): the decode step's
// qwen_rms_norm_per_head then qwen_apply_rope_neox at the cache row (src/tts_native.c:644-648)
// on this lane's 8 dims d0..d0+7 of a 128-dim head spread over a half-warp (lanes differ in
// bits 0-3). Sum of squares by an xor tree over the half-warp; the NeoX partner d +- 64 lives
// in lane ^ 8. The arithmetic per element is that of qk_norm_rope.cu's FP32 path (separately
// rounded products; only the sum of squares adds in another order).
__host__ __device__ constexpr int kv_dim_of(int n_kv) { return n_kv * kHD; }

struct QkArgs {
    const float *wq, *wk;       // per-head norm weights [128], or null (no norm)
    const float *cos_t, *sin_t;  // [table_rows, 128] RoPE tables, or null (no RoPE)
    int64_t table_rows;
    float eps;
};

__device__ __forceinline__ void norm_rope8(float (&a)[8], const float *w, const float (&cs)[8],
                                           const float (&sn)[8], bool rope, float eps,
                                           int d0) {
    if (w) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) ss = fmaf(a[e], a[e], ss);
#pragma unroll
        for (int o = 8; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float inv = 1.0f / sqrtf(ss / (float)kHD + eps);
        const float4 w0 = ld4(w + d0), w1 = ld4(w + d0 + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), wv[e]);
    }
    if (rope) {
        const bool first = d0 < kHD / 2;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float pa = __shfl_xor_sync(0xffffffffu, a[e], 8);
            a[e] = first ? __fsub_rn(__fmul_rn(a[e], cs[e]), __fmul_rn(pa, sn[e]))
                         : __fadd_rn(__fmul_rn(pa, sn[e]), __fmul_rn(a[e], cs[e]));
        }
    }
}

template <int G, bool QK>
__global__ void __launch_bounds__(kThreads)
decode_attn_kernel(float *out, const float *__restrict__ q, const float *__restrict__ k_new,
                   const float *__restrict__ v_new, float *k_cache, float *v_cache,
                   const int32_t *__restrict__ pos, int n_kv, int max_seq, float scale_log2,
                   float *partials, int *counters, int max_splits, int *err, const QkArgs qa) {
    const int split = blockIdx.x, kvh = blockIdx.y, s = blockIdx.z;
    // launched with programmatic dependent launch: q / k / v come from the kernel before,
    // and the kernel after (the o-projection GEMV) may start streaming its weights now
    pdl_wait_prior();
    pdl_launch_dependents();
    const int p = pos[s];
    if (p < 0 || p >= max_seq || (QK && qa.cos_t && p >= qa.table_rows)) {
        if (split == 0 && kvh == 0 && threadIdx.x == 0 && err) atomicOr(err, LAI_DEVERR_POSITION);
        return;
    }
    const int n_splits = p / kChunk + 1;  // keys 0..p
    if (split >= n_splits) return;

    const int n_heads = n_kv * G, kv_dim = n_kv * kHD;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int slot = lane >> 4;  // which half-warp: its own key stream
    const int d0 = (lane & 15) * 8;

    float cs[8], sn[8];  // RoPE row p for this lane's dims (fused entry)
    const bool rope = QK && qa.cos_t != nullptr;
    if (rope) {
        const float4 c0 = ld4(qa.cos_t + (size_t)p * kHD + d0), c1 = ld4(qa.cos_t + (size_t)p * kHD + d0 + 4);
        const float4 s0 = ld4(qa.sin_t + (size_t)p * kHD + d0), s1 = ld4(qa.sin_t + (size_t)p * kHD + d0 + 4);
        cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
        cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
        sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
        sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
    }
    float qr[G][8];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float *qp = q + (size_t)s * n_heads * kHD + (size_t)(kvh * G + g) * kHD + d0;
        const float4 a = ld4(qp), b = ld4(qp + 4);
        float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        if (QK) norm_rope8(x, qa.wq, cs, sn, rope, qa.eps, d0);
#pragma unroll
        for (int e = 0; e < 8; e++) qr[g][e] = x[e] * scale_log2;
    }
    // fused entry: this token's key, normed and rotated, in registers (both half-warps hold
    // the same 8 dims); it stands in for the row at j == p and is what the cache receives
    float kn[8];
    if (QK) {
        const float *kp = k_new + (size_t)s * kv_dim_of(n_kv) + (size_t)kvh * kHD + d0;
        const float4 a = ld4(kp), b = ld4(kp + 4);
        kn[0] = a.x; kn[1] = a.y; kn[2] = a.z; kn[3] = a.w;
        kn[4] = b.x; kn[5] = b.y; kn[6] = b.z; kn[7] = b.w;
        norm_rope8(kn, qa.wk, cs, sn, rope, qa.eps, d0);
    }
    float m[G], l[G], acc[G][8];
#pragma unroll
    for (int g = 0; g < G; g++) {
        m[g] = kNegBig;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < 8; e++) acc[g][e] = 0.f;
    }

    const size_t seq_base = (size_t)s * max_seq * kv_dim + (size_t)kvh * kHD + d0;
    const size_t new_base = (size_t)s * kv_dim + (size_t)kvh * kHD + d0;
    const int j0 = split * kChunk;
    const int j1 = min(p + 1, j0 + kChunk);
    constexpr int kStride = kWarps * 2;  // half-warps per CTA
    // jw is uniform across the warp (its shuffles need all 32 lanes); half-warp `slot`
    // takes key jw + slot + u * kStride and skips the state update past the range
    for (int jw = j0 + warp * 2; jw < j1; jw += kStride * kUnroll) {
        float kv[kUnroll][16];
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            const int j = jw + slot + u * kStride;
            if (j < j1) {
                const float *kr = j == p ? k_new + new_base : k_cache + seq_base + (size_t)j * kv_dim;
                const float *vr = j == p ? v_new + new_base : v_cache + seq_base + (size_t)j * kv_dim;
                const float4 a = ld4(kr), b = ld4(kr + 4), c = ld4(vr), d = ld4(vr + 4);
                kv[u][0] = a.x; kv[u][1] = a.y; kv[u][2] = a.z; kv[u][3] = a.w;
                kv[u][4] = b.x; kv[u][5] = b.y; kv[u][6] = b.z; kv[u][7] = b.w;
                if (QK && j == p) {
#pragma unroll
                    for (int e = 0; e < 8; e++) kv[u][e] = kn[e];
                }
                kv[u][8] = c.x; kv[u][9] = c.y; kv[u][10] = c.z; kv[u][11] = c.w;
                kv[u][12] = d.x; kv[u][13] = d.y; kv[u][14] = d.z; kv[u][15] = d.w;
            } else {
#pragma unroll
                for (int e = 0; e < 16; e++) kv[u][e] = 0.f;
            }
        }
#pragma unroll
        for (int u = 0; u < kUnroll; u++) {
            if (jw + u * kStride >= j1) break;  // warp-uniform: no key for either half
            const bool valid = jw + slot + u * kStride < j1;
#pragma unroll
            for (int g = 0; g < G; g++) {
                float dot = 0.f;
#pragma unroll
                for (int e = 0; e < 8; e++) dot = fmaf(qr[g][e], kv[u][e], dot);
                // the half-warp's 16 lanes hold the 16 partial sums of one key
                dot += __shfl_xor_sync(0xffffffffu, dot, 8);
                dot += __shfl_xor_sync(0xffffffffu, dot, 4);
                dot += __shfl_xor_sync(0xffffffffu, dot, 2);
                dot += __shfl_xor_sync(0xffffffffu, dot, 1);
                if (valid) {
                    const float mn = fmaxf(m[g], dot);
                    const float corr = exp2f(m[g] - mn), pj = exp2f(dot - mn);
                    m[g] = mn;
                    l[g] = fmaf(l[g], corr, pj);
#pragma unroll
                    for (int e = 0; e < 8; e++) acc[g][e] = fmaf(acc[g][e], corr, pj * kv[u][8 + e]);
                }
            }
        }
    }
    // Half-warp lanes that ran no key above stay at (kNegBig, 0, 0); the other half may not
    // have: merge the two halves (lane ^ 16 holds the same dims of the other key stream).
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float mo = __shfl_xor_sync(0xffffffffu, m[g], 16);
        const float lo = __shfl_xor_sync(0xffffffffu, l[g], 16);
        const float mn = fmaxf(m[g], mo);
        const float ca = exp2f(m[g] - mn), cb = exp2f(mo - mn);
        l[g] = l[g] * ca + lo * cb;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float ao = __shfl_xor_sync(0xffffffffu, acc[g][e], 16);
            acc[g][e] = acc[g][e] * ca + ao * cb;
        }
        m[g] = mn;
    }
    // warps -> shared memory -> one (max, sum, acc) per head for this CTA
    __shared__ float sm_m[kWarps][G], sm_l[kWarps][G];
    __shared__ float sm_acc[kWarps][G][kHD];
    __shared__ int sm_last;
    if (lane < 16) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            if (lane == 0) {
                sm_m[warp][g] = m[g];
                sm_l[warp][g] = l[g];
            }
#pragma unroll
            for (int e = 0; e < 8; e++) sm_acc[warp][g][d0 + e] = acc[g][e];
        }
    }
    __syncthreads();
    const int d = threadIdx.x;  // one output dim per thread (kThreads == kHD)
    float cm[G], cl[G], ca[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        float mx = sm_m[0][g];
#pragma unroll
        for (int w = 1; w < kWarps; w++) mx = fmaxf(mx, sm_m[w][g]);
        float sum = 0.f, a = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; w++) {
            const float c = exp2f(sm_m[w][g] - mx);
            sum = fmaf(sm_l[w][g], c, sum);
            a = fmaf(sm_acc[w][g][d], c, a);
        }
        cm[g] = mx;
        cl[g] = sum;
        ca[g] = a;
    }
    if (split == n_splits - 1 && threadIdx.x < 32) {  // append the token's k/v to the cache
        const size_t row = (size_t)s * max_seq * kv_dim + (size_t)p * kv_dim + (size_t)kvh * kHD;
        const size_t src = (size_t)s * kv_dim + (size_t)kvh * kHD;
        if (QK) {
            if (threadIdx.x < 16) {  // lanes 0-15 hold all 128 dims of the transformed key
                *reinterpret_cast<float4 *>(k_cache + row + d0) = make_float4(kn[0], kn[1], kn[2], kn[3]);
                *reinterpret_cast<float4 *>(k_cache + row + d0 + 4) = make_float4(kn[4], kn[5], kn[6], kn[7]);
            }
        } else {
            reinterpret_cast<float4 *>(k_cache + row)[threadIdx.x] =
                reinterpret_cast<const float4 *>(k_new + src)[threadIdx.x];
        }
        reinterpret_cast<float4 *>(v_cache + row)[threadIdx.x] =
            reinterpret_cast<const float4 *>(v_new + src)[threadIdx.x];
    }
    if (n_splits == 1) {
#pragma unroll
        for (int g = 0; g < G; g++)
            out[(size_t)s * n_heads * kHD + (size_t)(kvh * G + g) * kHD + d] = ca[g] / cl[g];
        return;
    }
    // several splits: publish this one, the last to finish merges
#pragma unroll
    for (int g = 0; g < G; g++) {
        float *pp = partials + (((size_t)s * n_heads + kvh * G + g) * max_splits + split) * kPartial;
        if (d == 0) {
            pp[0] = cm[g];
            pp[1] = cl[g];
        }
        pp[2 + d] = ca[g];
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int prev = atomicAdd(counters + (size_t)s * n_kv + kvh, 1);
        sm_last = prev == n_splits - 1;
    }
    __syncthreads();
    if (!sm_last) return;
    __threadfence();
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float *pp = partials + ((size_t)s * n_heads + kvh * G + g) * max_splits * kPartial;
        float mx = kNegBig;
        for (int i = 0; i < n_splits; i++) mx = fmaxf(mx, __ldcg(pp + (size_t)i * kPartial));
        float sum = 0.f, a = 0.f;
        for (int i = 0; i < n_splits; i++) {
            const float c = exp2f(__ldcg(pp + (size_t)i * kPartial) - mx);
            sum = fmaf(__ldcg(pp + (size_t)i * kPartial + 1), c, sum);
            a = fmaf(__ldcg(pp + (size_t)i * kPartial + 2 + d), c, a);
        }
        out[(size_t)s * n_heads * kHD + (size_t)(kvh * G + g) * kHD + d] = a / sum;
    }
    if (threadIdx.x == 0) counters[(size_t)s * n_kv + kvh] = 0;  // ready for the next call
}

template <int G>
void launch(float *out, const float *q, const float *k_new, const float *v_new, float *kc,
            float *vc, const int32_t *pos, int n_seqs, int n_kv, int max_seq, float scale_log2,
            float *partials, int *counters, int max_splits, int *err, const QkArgs *qa,
            cudaStream_t st) {
    const dim3 grid((unsigned)max_splits, (unsigned)n_kv, (unsigned)n_seqs);
    if (qa)
        launch_pdl(decode_attn_kernel<G, true>, grid, dim3(kThreads), 0, st, out, q, k_new,
                   v_new, kc, vc, pos, n_kv, max_seq, scale_log2, partials, counters, max_splits,
                   err, *qa);
    else
        launch_pdl(decode_attn_kernel<G, false>, grid, dim3(kThreads), 0, st, out, q, k_new,
                   v_new, kc, vc, pos, n_kv, max_seq, scale_log2, partials, counters, max_splits,
                   err, QkArgs{});
}

inline int splits_for(int max_seq) { return (max_seq + kChunk - 1) / kChunk; }

}  // namespace
}  // namespace lai

extern "C" size_t lai_decode_attention_scratch_bytes(int n_seqs, int n_heads, int n_kv_heads,
                                                     int max_seq) {
    if (n_seqs <= 0 || n_heads <= 0 || n_kv_heads <= 0 || max_seq <= 0) return 0;
    const size_t partials = (size_t)n_seqs * n_heads * lai::splits_for(max_seq) * lai::kPartial;
    return partials * sizeof(float) + (size_t)n_seqs * n_kv_heads * sizeof(int);
}

namespace lai {
namespace {
int attention_entry(float *out, const float *q, const float *k_new, const float *v_new,
                    float *k_cache, float *v_cache, const int32_t *pos, int n_seqs, int n_heads,
                    int n_kv_heads, int head_dim, int max_seq, float scale, void *scratch,
                    int *err, const QkArgs *qa, lai_stream_t stream) {
    if (!out || !q || !k_new || !v_new || !k_cache || !v_cache || !pos || !scratch ||
        n_seqs < 0 || n_heads <= 0 || n_kv_heads <= 0 || max_seq <= 0)
        return LAI_ERR_INVALID;
    if (n_seqs == 0) return LAI_OK;
    if (head_dim != kHD || n_heads % n_kv_heads != 0) return LAI_ERR_INVALID;
    const int G = n_heads / n_kv_heads;
    if (G != 1 && G != 2 && G != 4 && G != 8) return LAI_ERR_INVALID;
    if (n_seqs > 65535 || n_kv_heads > 65535) return LAI_ERR_RANGE;
    if (!aligned16(out) || !aligned16(q) || !aligned16(k_new) || !aligned16(v_new) ||
        !aligned16(k_cache) || !aligned16(v_cache) || !aligned16(scratch))
        return LAI_ERR_INVALID;
    if (qa && ((qa->wq && !aligned16(qa->wq)) || (qa->wk && !aligned16(qa->wk)) ||
               ((qa->cos_t == nullptr) != (qa->sin_t == nullptr)) ||
               (qa->cos_t && (!aligned16(qa->cos_t) || !aligned16(qa->sin_t) ||
                              qa->table_rows <= 0))))
        return LAI_ERR_INVALID;
    const size_t cache_bytes = (size_t)n_seqs * max_seq * n_kv_heads * kHD * sizeof(float);
    const size_t out_bytes = (size_t)n_seqs * n_heads * kHD * sizeof(float);
    if (overlaps(out, out_bytes, k_cache, cache_bytes) || overlaps(out, out_bytes, v_cache, cache_bytes) ||
        overlaps(k_cache, cache_bytes, v_cache, cache_bytes) || overlaps(out, out_bytes, q, out_bytes))
        return LAI_ERR_ALIAS;
    const int max_splits = splits_for(max_seq);
    float *partials = static_cast<float *>(scratch);
    int *counters = reinterpret_cast<int *>(
        partials + (size_t)n_seqs * n_heads * max_splits * kPartial);
    const float sl2 = scale * kLog2e;
    const cudaStream_t st = as_stream(stream);
    switch (G) {
        case 1: launch<1>(out, q, k_new, v_new, k_cache, v_cache, pos, n_seqs, n_kv_heads, max_seq, sl2, partials, counters, max_splits, err, qa, st); break;
        case 2: launch<2>(out, q, k_new, v_new, k_cache, v_cache, pos, n_seqs, n_kv_heads, max_seq, sl2, partials, counters, max_splits, err, qa, st); break;
        case 4: launch<4>(out, q, k_new, v_new, k_cache, v_cache, pos, n_seqs, n_kv_heads, max_seq, sl2, partials, counters, max_splits, err, qa, st); break;
        default: launch<8>(out, q, k_new, v_new, k_cache, v_cache, pos, n_seqs, n_kv_heads, max_seq, sl2, partials, counters, max_splits, err, qa, st); break;
    }
    return launch_status();
}
}  // namespace
}  // namespace lai

extern "C" int lai_decode_attention_f32(float *out, const float *q, const float *k_new,
                                        const float *v_new, float *k_cache, float *v_cache,
                                        const int32_t *pos, int n_seqs, int n_heads,
                                        int n_kv_heads, int head_dim, int max_seq, float scale,
                                        void *scratch, int *err, lai_stream_t stream) {
    return lai::attention_entry(out, q, k_new, v_new, k_cache, v_cache, pos, n_seqs, n_heads,
                                n_kv_heads, head_dim, max_seq, scale, scratch, err, nullptr,
                                stream);
}

extern "C" int lai_decode_attention_qk_f32(float *out, const float *q, const float *k_new,
                                           const float *v_new, float *k_cache, float *v_cache,
                                           const int32_t *pos, int n_seqs, int n_heads,
                                           int n_kv_heads, int head_dim, int max_seq, float scale,
                                           const float *wq, const float *wk, const float *cos_t,
                                           const float *sin_t, int64_t table_rows, float eps,
                                           void *scratch, int *err, lai_stream_t stream) {
    const lai::QkArgs qa{wq, wk, cos_t, sin_t, table_rows, eps};
    return lai::attention_entry(out, q, k_new, v_new, k_cache, v_cache, pos, n_seqs, n_heads,
                                n_kv_heads, head_dim, max_seq, scale, scratch, err, &qa, stream);
}

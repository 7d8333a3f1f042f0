// prefill_attention.cu - causal self-attention over a whole sequence (every row a query).
//
// Reference: qwen_causal_attention(out, q, k, v, T, T, heads, kv_heads, hd, scale, 0) as the
// vocoder's pre-transformer calls it (src/tts_vocoder_xfmr.c:172-180: 16 heads, no GQA,
// head_dim 64, T = the codec frame count), after qwen_apply_rope_neox on q and k
// (:172-175); math as tools/verify_xfmr.py:37-77 (NeoX rotate-half, scores q.k * scale over
// keys 0..t, max-subtracted softmax, weighted sum of v). Query head h reads kv head
// h / (heads / kv_heads).
//
// Work split: a CTA takes 32 consecutive query rows of one head, one row per lane, and its
// four warps split every 32-key tile of shared memory into quarters (keys stream through
// shared memory, every lane of a warp reading the same key: a broadcast). Each warp keeps
// an online softmax in log2 units for its quarter of the keys; the four partial states
// merge through shared memory at the end, and the output tile leaves in coalesced rows.
// The RoPE variant rotates q while staging it and k while filling each key tile, so q / k /
// v can be read straight from one fused q|k|v projection output (row strides ld_q, ld_kv).
// The sequence is short (the codec frames of one utterance) and the work T^2 * hd per head,
// so plain F32 FMAs on CUDA cores suffice.
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kQRows = 32;                 // query rows per CTA (one per lane)
constexpr int kSplit = 4;                  // warps per CTA, each a quarter of every key tile
constexpr int kKeys = 32;                  // keys per shared-memory tile
constexpr int kThreads = kQRows * kSplit;  // 128
constexpr float kLog2eP = 1.4426950408889634f;

// NeoX rotate-half, in the reference's float order: x1*c - x2*s and x1*s + x2*c.
__device__ __forceinline__ float rope_first(float own, float partner, float c, float s) {
    return __fsub_rn(__fmul_rn(own, c), __fmul_rn(partner, s));
}
__device__ __forceinline__ float rope_second(float own, float partner, float c, float s) {
    return __fadd_rn(__fmul_rn(partner, s), __fmul_rn(own, c));
}

template <int HD>
struct PrefillSmem {
    union {
        struct {
            float k[kKeys][HD];
            float v[kKeys][HD];
        } tile;
        float rows[2][kQRows][HD + 1];  // q staging, partial accumulators, the output tile
    };
    float m[2][kQRows], l[2][kQRows];
};

// Fold another partial softmax state (mo, lo, ao) into (m, l, acc).
template <int HD>
__device__ __forceinline__ void merge_state(float &m, float &l, float (&acc)[HD], float mo,
                                            float lo, const float *ao) {
    const float mn = fmaxf(m, mo);
    const float ca = exp2f(m - mn), cb = exp2f(mo - mn);
    l = fmaf(l, ca, lo * cb);
#pragma unroll
    for (int d = 0; d < HD; d++) acc[d] = fmaf(acc[d], ca, ao[d] * cb);
    m = mn;
}

__device__ __forceinline__ float4 ldg4(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
}

__device__ __forceinline__ float4 rope4_first(float4 a, float4 b, float4 c, float4 s) {
    return make_float4(rope_first(a.x, b.x, c.x, s.x), rope_first(a.y, b.y, c.y, s.y),
                       rope_first(a.z, b.z, c.z, s.z), rope_first(a.w, b.w, c.w, s.w));
}
__device__ __forceinline__ float4 rope4_second(float4 b, float4 a, float4 c, float4 s) {
    return make_float4(rope_second(b.x, a.x, c.x, s.x), rope_second(b.y, a.y, c.y, s.y),
                       rope_second(b.z, a.z, c.z, s.z), rope_second(b.w, a.w, c.w, s.w));
}

// Load one row's float4 group g of both halves (d = 4g.. and H2 + 4g..) of a head, rotated
// with table row `row` when ROPE; zeros past the sequence end.
template <int HD, bool ROPE>
__device__ __forceinline__ void load_pair(const float *base, bool valid, const float *cos_t,
                                          const float *sin_t, int row, int g, float4 &a,
                                          float4 &b) {
    constexpr int H2 = HD / 2;
    a = b = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!valid) return;
    a = ldg4(base + 4 * g);
    b = ldg4(base + H2 + 4 * g);
    if (ROPE) {
        const float *c = cos_t + (size_t)row * HD, *s = sin_t + (size_t)row * HD;
        const float4 ca = ldg4(c + 4 * g), cb = ldg4(c + H2 + 4 * g);
        const float4 sa = ldg4(s + 4 * g), sb = ldg4(s + H2 + 4 * g);
        const float4 a2 = rope4_first(a, b, ca, sa);
        b = rope4_second(b, a, cb, sb);
        a = a2;
    }
}

template <int HD, bool ROPE>
__global__ void __launch_bounds__(kThreads)
prefill_attn_kernel(float *__restrict__ out, const float *__restrict__ q,
                    const float *__restrict__ k, const float *__restrict__ v, int T, int n_heads,
                    int n_kv, int ld_q, int ld_kv, const float *__restrict__ cos_t,
                    const float *__restrict__ sin_t, float scale_log2) {
    constexpr int H2 = HD / 2, H4 = H2 / 4;
    constexpr int kQItems = kQRows * H4 / kThreads;  // (row, group) pairs per thread
    constexpr int kKItems = kKeys * H4 / kThreads;
    constexpr int kVItems = kKeys * (HD / 4) / kThreads;
    constexpr int kGroup = kKeys / kSplit;           // keys per warp per tile
    static_assert(kQItems * kThreads == kQRows * H4 && kVItems * kThreads == kKeys * HD / 4,
                  "tile loads must divide evenly among the threads");
    __shared__ __align__(16) PrefillSmem<HD> sm;
    const int h = blockIdx.y, kvh = h / (n_heads / n_kv);
    const int r0 = blockIdx.x * kQRows;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int t = r0 + lane;

    // stage the CTA's q rows (coalesced float4), rotated and pre-scaled into log2 units
#pragma unroll
    for (int it = 0; it < kQItems; it++) {
        const int i = threadIdx.x + it * kThreads, rr = i / H4, g = i - rr * H4, row = r0 + rr;
        float4 a, b;
        load_pair<HD, ROPE>(q + (size_t)row * ld_q + (size_t)h * HD, row < T, cos_t, sin_t, row,
                            g, a, b);
        float *dst = sm.rows[0][rr];
        dst[4 * g] = a.x * scale_log2;
        dst[4 * g + 1] = a.y * scale_log2;
        dst[4 * g + 2] = a.z * scale_log2;
        dst[4 * g + 3] = a.w * scale_log2;
        dst[H2 + 4 * g] = b.x * scale_log2;
        dst[H2 + 4 * g + 1] = b.y * scale_log2;
        dst[H2 + 4 * g + 2] = b.z * scale_log2;
        dst[H2 + 4 * g + 3] = b.w * scale_log2;
    }
    __syncthreads();
    float qr[HD], acc[HD];
#pragma unroll
    for (int d = 0; d < HD; d++) {
        qr[d] = sm.rows[0][lane][d];
        acc[d] = 0.f;
    }
    float m = -1e30f, l = 0.f;

    const int last = min(T, r0 + kQRows) - 1;  // the CTA's last query row
    const int jb = w * kGroup;                 // this warp's keys of each tile
    for (int j0 = 0; j0 <= last; j0 += kKeys) {
        // issue every load of the tile before the first store (one round trip per tile)
        float4 ka[kKItems], kb[kKItems], va[kVItems];
#pragma unroll
        for (int it = 0; it < kKItems; it++) {
            const int i = threadIdx.x + it * kThreads, jj = i / H4, g = i - jj * H4, j = j0 + jj;
            load_pair<HD, ROPE>(k + (size_t)j * ld_kv + (size_t)kvh * HD, j < T, cos_t, sin_t, j,
                                g, ka[it], kb[it]);
        }
#pragma unroll
        for (int it = 0; it < kVItems; it++) {
            const int i = threadIdx.x + it * kThreads, jj = i / (HD / 4), g = i - jj * (HD / 4);
            const int j = j0 + jj;
            va[it] = j < T ? ldg4(v + (size_t)j * ld_kv + (size_t)kvh * HD + 4 * g)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();  // the previous tile (or the q staging) is fully read
#pragma unroll
        for (int it = 0; it < kKItems; it++) {
            const int i = threadIdx.x + it * kThreads, jj = i / H4, g = i - jj * H4;
            *reinterpret_cast<float4 *>(&sm.tile.k[jj][4 * g]) = ka[it];
            *reinterpret_cast<float4 *>(&sm.tile.k[jj][H2 + 4 * g]) = kb[it];
        }
#pragma unroll
        for (int it = 0; it < kVItems; it++) {
            const int i = threadIdx.x + it * kThreads, jj = i / (HD / 4), g = i - jj * (HD / 4);
            *reinterpret_cast<float4 *>(&sm.tile.v[jj][4 * g]) = va[it];
        }
        __syncthreads();
        const int nk = min(kGroup, t - j0 - jb + 1);  // this warp's keys at or before t
        if (t < T && nk > 0) {
            // the group's scores as independent dot products, one rescale for the group
            float sc[kGroup];
            float mn = m;
#pragma unroll
            for (int jj = 0; jj < kGroup; jj++) {
                const float4 *kr = reinterpret_cast<const float4 *>(sm.tile.k[jb + jj]);
                // four partial sums as two packed pairs (FFMA2: the same per-lane FMAs)
                float2 s01 = make_float2(0.f, 0.f), s23 = make_float2(0.f, 0.f);
#pragma unroll
                for (int d4 = 0; d4 < HD / 4; d4++) {
                    const float4 kk = kr[d4];
                    s01 = __ffma2_rn(make_float2(qr[4 * d4], qr[4 * d4 + 1]),
                                     make_float2(kk.x, kk.y), s01);
                    s23 = __ffma2_rn(make_float2(qr[4 * d4 + 2], qr[4 * d4 + 3]),
                                     make_float2(kk.z, kk.w), s23);
                }
                sc[jj] = (s01.x + s01.y) + (s23.x + s23.y);
                if (jj < nk) mn = fmaxf(mn, sc[jj]);
            }
            const float corr = exp2f(m - mn);
            float psum = 0.f;
#pragma unroll
            for (int jj = 0; jj < kGroup; jj++) {
                sc[jj] = jj < nk ? exp2f(sc[jj] - mn) : 0.f;
                psum += sc[jj];
            }
            m = mn;
            l = fmaf(l, corr, psum);
#pragma unroll
            for (int d4 = 0; d4 < HD / 4; d4++) {
                const float2 c2 = make_float2(corr, corr);
                float2 a01 = __fmul2_rn(make_float2(acc[4 * d4], acc[4 * d4 + 1]), c2);
                float2 a23 = __fmul2_rn(make_float2(acc[4 * d4 + 2], acc[4 * d4 + 3]), c2);
#pragma unroll
                for (int jj = 0; jj < kGroup; jj++) {
                    const float4 vv = reinterpret_cast<const float4 *>(sm.tile.v[jb + jj])[d4];
                    const float2 p2 = make_float2(sc[jj], sc[jj]);
                    a01 = __ffma2_rn(p2, make_float2(vv.x, vv.y), a01);
                    a23 = __ffma2_rn(p2, make_float2(vv.z, vv.w), a23);
                }
                acc[4 * d4] = a01.x;
                acc[4 * d4 + 1] = a01.y;
                acc[4 * d4 + 2] = a23.x;
                acc[4 * d4 + 3] = a23.y;
            }
        }
    }

    // merge the four partial states: warps 2, 3 into 0, 1, then 1 into 0. Warp 0 always saw
    // key 0, so the merged l of a real row is positive.
    __syncthreads();  // the last tile is read before the union is reused
    if (w >= 2) {
#pragma unroll
        for (int d = 0; d < HD; d++) sm.rows[w - 2][lane][d] = acc[d];
        sm.m[w - 2][lane] = m;
        sm.l[w - 2][lane] = l;
    }
    __syncthreads();
    if (w < 2) merge_state<HD>(m, l, acc, sm.m[w][lane], sm.l[w][lane], sm.rows[w][lane]);
    __syncthreads();
    if (w == 1) {
#pragma unroll
        for (int d = 0; d < HD; d++) sm.rows[0][lane][d] = acc[d];
        sm.m[0][lane] = m;
        sm.l[0][lane] = l;
    }
    __syncthreads();
    if (w == 0) {
        merge_state<HD>(m, l, acc, sm.m[0][lane], sm.l[0][lane], sm.rows[0][lane]);
        const float inv = t < T ? 1.0f / l : 0.f;
#pragma unroll
        for (int d = 0; d < HD; d++) sm.rows[1][lane][d] = acc[d] * inv;
    }
    __syncthreads();
    const int ldo = n_heads * HD;
    for (int i = threadIdx.x; i < kQRows * HD; i += kThreads) {
        const int rr = i / HD, d = i - rr * HD, row = r0 + rr;
        if (row < T) out[(size_t)row * ldo + (size_t)h * HD + d] = sm.rows[1][rr][d];
    }
}

int prefill_entry(float *out, const float *q, const float *k, const float *v, int ld_q,
                  int ld_kv, int T, int n_heads, int n_kv_heads, int head_dim, float scale,
                  const float *cos_t, const float *sin_t, int64_t table_rows,
                  lai_stream_t stream) {
    if (!out || !q || !k || !v || T < 0 || n_heads <= 0 || n_kv_heads <= 0 ||
        n_heads % n_kv_heads != 0 || (head_dim != 64 && head_dim != 128) ||
        (cos_t == nullptr) != (sin_t == nullptr) || ld_q < n_heads * head_dim ||
        ld_kv < n_kv_heads * head_dim || ld_q % 4 != 0 || ld_kv % 4 != 0 || !aligned16(q) ||
        !aligned16(k) || !aligned16(v) || (cos_t && (!aligned16(cos_t) || !aligned16(sin_t))))
        return LAI_ERR_INVALID;
    if (T == 0) return LAI_OK;
    if (n_heads > 65535 || (cos_t && table_rows < T)) return LAI_ERR_RANGE;
    const size_t ob = (size_t)T * n_heads * head_dim * 4;
    const size_t qb = ((size_t)(T - 1) * ld_q + (size_t)n_heads * head_dim) * 4;
    const size_t kb = ((size_t)(T - 1) * ld_kv + (size_t)n_kv_heads * head_dim) * 4;
    if (overlaps(out, ob, q, qb) || overlaps(out, ob, k, kb) || overlaps(out, ob, v, kb))
        return LAI_ERR_ALIAS;
    const dim3 grid((unsigned)((T + kQRows - 1) / kQRows), (unsigned)n_heads);
    const float sl2 = scale * kLog2eP;
    const cudaStream_t st = as_stream(stream);
    const bool rope = cos_t != nullptr;
#define LAI_PREFILL(HD, R)                                                                    \
    prefill_attn_kernel<HD, R><<<grid, kThreads, 0, st>>>(out, q, k, v, T, n_heads, n_kv_heads, \
                                                          ld_q, ld_kv, cos_t, sin_t, sl2)
    if (head_dim == 64) {
        if (rope) LAI_PREFILL(64, true); else LAI_PREFILL(64, false);
    } else {
        if (rope) LAI_PREFILL(128, true); else LAI_PREFILL(128, false);
    }
#undef LAI_PREFILL
    return launch_status();
}

}  // namespace
}  // namespace lai

extern "C" int lai_prefill_attention_f32(float *out, const float *q, const float *k,
                                         const float *v, int T, int n_heads, int n_kv_heads,
                                         int head_dim, float scale, lai_stream_t stream) {
    return lai::prefill_entry(out, q, k, v, n_heads * head_dim, n_kv_heads * head_dim, T, n_heads,
                              n_kv_heads, head_dim, scale, nullptr, nullptr, 0, stream);
}

extern "C" int lai_prefill_attention_rope_f32(float *out, const float *q, const float *k,
                                              const float *v, int ld_q, int ld_kv, int T,
                                              int n_heads, int n_kv_heads, int head_dim,
                                              float scale, const float *cos_t,
                                              const float *sin_t, int64_t table_rows,
                                              lai_stream_t stream) {
    return lai::prefill_entry(out, q, k, v, ld_q, ld_kv, T, n_heads, n_kv_heads, head_dim, scale,
                              cos_t, sin_t, table_rows, stream);
}

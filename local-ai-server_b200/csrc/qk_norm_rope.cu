// qk_norm_rope.cu - fused per-head q/k RMSNorm + NeoX RoPE, and the RoPE table.
//
// Reference semantics: qwen_rms_norm_per_head(q|k, w, seq, heads, hd, eps) then
// qwen_apply_rope_neox(q|k, cos, sin, seq, heads, hd), as talker_prefill calls them
// (src/tts_native.c:562-568); RoPE formula tools/verify_xfmr.py:49-53; table rows
// hold cos/sin with duplicated halves (src/tts_native.c:402-412).
//
// Roofline: HBM. Algorithmic bytes per token: 2 * (n_q + n_kv) * hd * s (q and k
// read once, written once in place); the [hd] weights and the table rows are
// shared (L1/L2-resident) and not counted.
//
// Layout of the fast path. One warp owns one (token, q-or-k) segment. A head of
// hd elements spans LPH = hd*s/16 lanes (16 for BF16 hd=128), each lane one
// 16-byte vector, so a warp-wide 16-byte load covers 32/LPH heads and the whole
// segment is `slots` such loads, issued back to back before any arithmetic. The
// per-head sum of squares is an xor-shuffle tree over the LPH lanes; the RoPE
// partner element (d <-> d + hd/2) sits in lane ^ LPH/2, one shuffle per element.
// Each lane loads its hd/LPH weights and its cos/sin entries once per segment.
// RoPE uses separately rounded products (no contraction), so with identical
// inputs it reproduces the reference's scalar C bit for bit.
#include "lai_common.cuh"

#include <math.h>

namespace lai {
namespace {

constexpr int kItemsPerCta = 8;  // warps per CTA, one (token, segment) each
constexpr int kMaxSlots = 8;     // 16-byte loads in flight per lane per pass

__device__ __forceinline__ float rope_first(float own, float partner, float c, float s) {
    return __fsub_rn(__fmul_rn(own, c), __fmul_rn(partner, s));  // x1*c - x2*s
}
__device__ __forceinline__ float rope_second(float own, float partner, float c, float s) {
    return __fadd_rn(__fmul_rn(partner, s), __fmul_rn(own, c));  // x1*s + x2*c
}

template <typename T, int HD>
__global__ void __launch_bounds__(kItemsPerCta * 32)
qk_warp_kernel(T *q, T *k, const float *__restrict__ wq, const float *__restrict__ wk,
               const float *__restrict__ cos_t, const float *__restrict__ sin_t,
               const int32_t *__restrict__ pos, int64_t table_rows, int64_t rows, int nq,
               int nkv, float eps, int *err) {
    constexpr int E = Elt<T>::N;
    constexpr int LPH = HD * (int)sizeof(T) / 16;  // lanes per head
    constexpr int HL = LPH / 2;
    static_assert(LPH >= 2 && LPH <= 32 && (32 % LPH) == 0, "head must span 2..32 lanes");

    const int lane = threadIdx.x & 31;
    const int nseg = k ? 2 : 1;
    const int64_t item = (int64_t)blockIdx.x * kItemsPerCta + (threadIdx.x >> 5);
    if (item >= rows * nseg) return;
    const int64_t row = nseg == 2 ? (item >> 1) : item;
    const int seg = nseg == 2 ? (int)(item & 1) : 0;

    const int heads = seg == 0 ? nq : nkv;
    T *base = seg == 0 ? q + (size_t)row * nq * HD : k + (size_t)row * nkv * HD;
    const float *w = seg == 0 ? wq : wk;
    const bool rope = cos_t != nullptr;

    int64_t p = pos ? (int64_t)pos[row] : row;
    if (rope && (p < 0 || p >= table_rows)) {
        if (lane == 0 && err && seg == 0) atomicOr(err, LAI_DEVERR_POSITION);
        return;
    }

    const int hl = lane % LPH;
    const int c0 = hl * E;  // first column of this lane within its head
    const bool first = hl < HL;
    float wv[E], cs[E], sn[E];
    if (w) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            float4 t = ld_f4(w + c0 + e);
            wv[e] = t.x; wv[e + 1] = t.y; wv[e + 2] = t.z; wv[e + 3] = t.w;
        }
    }
    if (rope) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            float4 a = ld_f4(cos_t + (size_t)p * HD + c0 + e);
            float4 b = ld_f4(sin_t + (size_t)p * HD + c0 + e);
            cs[e] = a.x; cs[e + 1] = a.y; cs[e + 2] = a.z; cs[e + 3] = a.w;
            sn[e] = b.x; sn[e + 1] = b.y; sn[e + 2] = b.z; sn[e + 3] = b.w;
        }
    }

    const int slots = heads * LPH / 32;
    for (int s0 = 0; s0 < slots; s0 += kMaxSlots) {
        uint4 v[kMaxSlots];
#pragma unroll
        for (int j = 0; j < kMaxSlots; j++)
            if (s0 + j < slots) v[j] = ld_stream(base + ((size_t)(s0 + j) * 32 + lane) * E);
#pragma unroll
        for (int j = 0; j < kMaxSlots; j++) {
            if (s0 + j >= slots) break;  // warp-uniform
            float a[E];
            unpack<T>(v[j], a);
            if (w) {
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < E; e++) ss = fmaf(a[e], a[e], ss);
                ss = group_sum<LPH>(ss);
                const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
                for (int e = 0; e < E; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), wv[e]);
            }
            if (rope) {
#pragma unroll
                for (int e = 0; e < E; e++) {
                    const float pa = __shfl_xor_sync(0xffffffffu, a[e], HL);
                    a[e] = first ? rope_first(a[e], pa, cs[e], sn[e])
                                 : rope_second(a[e], pa, cs[e], sn[e]);
                }
            }
            st_vec(base + ((size_t)(s0 + j) * 32 + lane) * E, pack<T>(a));
        }
    }
}

// Any even head_dim / alignment / head count: one warp per (token, head).
template <typename T>
__global__ void __launch_bounds__(256)
qk_generic_kernel(T *q, T *k, const float *wq, const float *wk, const float *cos_t,
                  const float *sin_t, const int32_t *pos, int64_t table_rows, int64_t rows,
                  int nq, int nkv, int hd, float eps, int *err) {
    const int lane = threadIdx.x & 31;
    const int nh = nq + (k ? nkv : 0);
    const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= rows * nh) return;
    const int64_t row = item / nh;
    const int h = (int)(item % nh);
    T *xh = h < nq ? q + ((size_t)row * nq + h) * hd : k + ((size_t)row * nkv + (h - nq)) * hd;
    const float *w = h < nq ? wq : wk;
    const bool rope = cos_t != nullptr;
    int64_t p = pos ? (int64_t)pos[row] : row;
    if (rope && (p < 0 || p >= table_rows)) {
        if (lane == 0 && err && h == 0) atomicOr(err, LAI_DEVERR_POSITION);
        return;
    }
    float inv = 1.f;
    if (w) {
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) {
            float a = to_f(xh[d]);
            ss = fmaf(a, a, ss);
        }
        ss = group_sum<32>(ss);
        inv = 1.0f / sqrtf(ss / (float)hd + eps);
    }
    const int half = hd / 2;
    const float *c = rope ? cos_t + (size_t)p * hd : nullptr;
    const float *s = rope ? sin_t + (size_t)p * hd : nullptr;
    for (int d = lane; d < half; d += 32) {
        float x1 = to_f(xh[d]), x2 = to_f(xh[d + half]);
        if (w) {
            x1 = __fmul_rn(__fmul_rn(x1, inv), w[d]);
            x2 = __fmul_rn(__fmul_rn(x2, inv), w[d + half]);
        }
        if (rope) {
            const float r1 = rope_first(x1, x2, c[d], s[d]);
            const float r2 = rope_second(x2, x1, c[d + half], s[d + half]);
            x1 = r1;
            x2 = r2;
        }
        xh[d] = from_f<T>(x1);
        xh[d + half] = from_f<T>(x2);
    }
}

template <typename T, int HD>
bool try_fast(T *q, T *k, const float *wq, const float *wk, const float *cos_t,
              const float *sin_t, const int32_t *pos, int64_t table_rows, int64_t rows, int nq,
              int nkv, float eps, int *err, cudaStream_t s) {
    constexpr int LPH = HD * (int)sizeof(T) / 16;
    if constexpr (LPH > 32) {
        return false;  // a head wider than one warp-wide load: generic kernel
    } else {
        if ((nq * LPH) % 32 != 0 || (k && (nkv * LPH) % 32 != 0)) return false;
        if (!aligned16(q) || (k && !aligned16(k)) || (wq && !aligned16(wq)) ||
            (k && wk && !aligned16(wk)) || (cos_t && (!aligned16(cos_t) || !aligned16(sin_t))))
            return false;
        const int64_t items = rows * (k ? 2 : 1);
        qk_warp_kernel<T, HD><<<grid_for(items, kItemsPerCta), kItemsPerCta * 32, 0, s>>>(
            q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err);
        return true;
    }
}

template <typename T>
int run(T *q, T *k, const float *wq, const float *wk, const float *cos_t, const float *sin_t,
        const int32_t *pos, int64_t table_rows, int64_t rows, int nq, int nkv, int hd, float eps,
        int *err, lai_stream_t stream) {
    if (!q || rows < 0 || nq <= 0 || hd <= 0 || (hd & 1) || (k && nkv <= 0)) return LAI_ERR_INVALID;
    if (cos_t && (!sin_t || table_rows <= 0)) return LAI_ERR_INVALID;
    if (!cos_t && !wq && !wk) return LAI_ERR_INVALID;  // nothing to do is a caller bug
    if (rows == 0) return LAI_OK;
    if (k && overlaps(q, (size_t)rows * nq * hd * sizeof(T), k, (size_t)rows * nkv * hd * sizeof(T)))
        return LAI_ERR_ALIAS;
    cudaStream_t s = as_stream(stream);
    bool done = false;
    switch (hd) {
        case 64: done = try_fast<T, 64>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err, s); break;
        case 128: done = try_fast<T, 128>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err, s); break;
        case 256: done = try_fast<T, 256>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err, s); break;
        default: break;
    }
    if (!done) {
        const int64_t items = rows * (nq + (k ? nkv : 0));
        qk_generic_kernel<T><<<grid_for(items, 8), 256, 0, s>>>(q, k, wq, wk, cos_t, sin_t, pos,
                                                               table_rows, rows, nq, nkv, hd, eps, err);
    }
    return launch_status();
}

// ---- RoPE table -----------------------------------------------------------------
struct InvFreq {
    float f[256];
};

__global__ void __launch_bounds__(256)
rope_table_kernel(float *cos_t, float *sin_t, const int32_t *pos, int64_t n, int hd, InvFreq inv) {
    const int half = hd / 2;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n * half) return;
    const int64_t i = idx / half;
    const int d = (int)(idx % half);
    const int p = pos ? pos[i] : (int)i;
    const float angle = __fmul_rn((float)p, inv.f[d]);
    const float c = cosf(angle), s = sinf(angle);
    cos_t[i * hd + d] = c;
    cos_t[i * hd + half + d] = c;
    sin_t[i * hd + d] = s;
    sin_t[i * hd + half + d] = s;
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_qk_norm_rope_bf16(lai_bf16 *q, lai_bf16 *k, const float *wq, const float *wk,
                          const float *cos_t, const float *sin_t, const int32_t *pos,
                          int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                          int head_dim, float eps, int *err, lai_stream_t stream) {
    return lai::run<uint16_t>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, n_q_heads,
                              n_kv_heads, head_dim, eps, err, stream);
}

int lai_qk_norm_rope_f32(float *q, float *k, const float *wq, const float *wk,
                         const float *cos_t, const float *sin_t, const int32_t *pos,
                         int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                         int head_dim, float eps, int *err, lai_stream_t stream) {
    return lai::run<float>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, n_q_heads,
                           n_kv_heads, head_dim, eps, err, stream);
}

int lai_rope_table_f32(float *cos_t, float *sin_t, const int32_t *pos, int64_t n, int head_dim,
                       float theta, lai_stream_t stream) {
    if (!cos_t || !sin_t || n < 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 512)
        return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    lai::InvFreq inv;
    // Host-side, with the host libm, exactly as ensure_rope_cache computes it
    // (src/tts_native.c:383-388), so the device table sees identical frequencies.
    for (int d = 0; d < head_dim / 2; d++)
        inv.f[d] = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
    const int64_t work = n * (head_dim / 2);
    lai::rope_table_kernel<<<lai::grid_for(work, 256), 256, 0, lai::as_stream(stream)>>>(
        cos_t, sin_t, pos, n, head_dim, inv);
    return lai::launch_status();
}

}  // extern "C"

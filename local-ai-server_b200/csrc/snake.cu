// snake.cu - vocoder SnakeBeta activation, FP32, in place.
//
// Reference: voc_snake_beta(x, exp_alpha, inv_exp_beta, C, T)
// (src/tts_vocoder_ops.c:279-305): x[c,t] += ieb[c] * sin(ea[c] * x[c,t])^2 with the
// parameters pre-exponentiated at load (src/tts_vocoder.c:221-227). The scalar
// branch of the reference computes x + ((ieb * s) * s), s = sinf(ea * x); this
// kernel evaluates sin^2 directly (sin2_fast below) and lands within ~1e-7 of it.
//
// Roofline: HBM, 8 bytes per element (read + write). With a full-range sinf the
// kernel was issue-bound (ncu: 85% issue-active, ~41 instructions per element);
// sin2_fast brought that to ~20, still ~60% of the issue rate the HBM rate needs at the
// 1.7 GHz the power cap allows over a long sweep, so the vector body runs two elements per
// instruction (snake2, Blackwell's packed FP32 FMA / MUL / ADD; same bits as snake1).
//
// Layout: snake_flat_kernel treats [batch*C rows, T] as one run of float4 vectors
// and recovers each vector's row and channel by multiply-high division, so short
// rows waste no threads. snake_kernel (unaligned base, T < 4, or >= 2^32 elements)
// walks rows on grid y and 16 KiB segments on grid x with scalar head and tail.
#include "lai_common.cuh"
#include "snake_math.cuh"

namespace lai {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;  // float4 per thread: 2 beat 1, 4 and 8 over the c4 sweep (676-680 vs 684 us at 4)
constexpr int kSegVec = kThreads * kUnroll;  // float4 vectors per CTA segment

__global__ void __launch_bounds__(kThreads)
snake_kernel(float *x, const float *__restrict__ ea, const float *__restrict__ ieb,
             int64_t rows, int channels, int64_t T, bool vec) {
    for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
        const int c = (int)(row % channels);
        const float a = __ldg(ea + c), b = __ldg(ieb + c);
        float *xr = x + (size_t)row * T;
        int64_t head = 0;
        if (vec) head = (4 - (int64_t)(((size_t)row * T) & 3)) & 3;
        if (head > T) head = T;
        const int64_t nv = vec ? (T - head) / 4 : 0;
        const int64_t body_end = head + nv * 4;
        float4 *xv = reinterpret_cast<float4 *>(xr + head);
        const int64_t v0 = (int64_t)blockIdx.x * kSegVec + threadIdx.x;
        float4 v[kUnroll];
#pragma unroll
        for (int i = 0; i < kUnroll; i++) {
            const int64_t k = v0 + (int64_t)i * kThreads;
            if (k < nv) v[i] = xv[k];
        }
#pragma unroll
        for (int i = 0; i < kUnroll; i++) {
            const int64_t k = v0 + (int64_t)i * kThreads;
            if (k < nv) {
                const float2 a2 = make_float2(a, a), b2 = make_float2(b, b);
                const float2 lo = snake2(make_float2(v[i].x, v[i].y), a2, b2);
                const float2 hi = snake2(make_float2(v[i].z, v[i].w), a2, b2);
                xv[k] = make_float4(lo.x, lo.y, hi.x, hi.y);
            }
        }
        if (blockIdx.x == 0) {
            // scalar head, scalar tail (whole row when !vec), strided over the CTA
            for (int64_t t = threadIdx.x; t < head; t += kThreads) xr[t] = snake1(xr[t], a, b);
            for (int64_t t = body_end + threadIdx.x; t < T; t += kThreads) xr[t] = snake1(xr[t], a, b);
        }
    }
}

// Unsigned division by an invariant 32-bit divisor as multiply-high and shifts
// (Granlund & Montgomery, "Division by invariant integers using multiplication",
// PLDI 1994, fig. 4.1): exact for every 32-bit dividend.
struct FastDiv {
    uint32_t d, m, s1, s2;
};
inline FastDiv make_fastdiv(uint32_t d) {
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) l++;  // l = ceil(log2 d)
    const uint64_t m = ((1ull << 32) * ((1ull << l) - d)) / d + 1;
    return FastDiv{d, (uint32_t)m, l < 1 ? l : 1u, l > 0 ? l - 1 : 0u};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
    const uint32_t t = __umulhi(f.m, n);
    return (t + ((n - t) >> f.s1)) >> f.s2;
}

// The whole [rows, T] tensor as one flat run of float4 vectors: uniform work per
// thread whatever the row length (short rows waste no threads). Needs a 16-byte
// aligned base, T >= 4 (a vector spans at most two rows) and < 2^32 elements.
__global__ void __launch_bounds__(kThreads)
snake_flat_kernel(float *x, const float *__restrict__ ea, const float *__restrict__ ieb,
                  uint32_t total, uint32_t T, uint32_t C, FastDiv divT, FastDiv divC) {
    const uint32_t nvec = total / 4;
    const uint32_t base = blockIdx.x * (uint32_t)kSegVec + threadIdx.x;
    float4 *xv = reinterpret_cast<float4 *>(x);
    pdl_wait_prior();  // launched with programmatic dependent launch: inputs after this
    float4 v[kUnroll];
#pragma unroll
    for (int i = 0; i < kUnroll; i++) {
        const uint32_t k = base + i * kThreads;
        if (k < nvec) v[i] = xv[k];
    }
#pragma unroll
    for (int i = 0; i < kUnroll; i++) {
        const uint32_t k = base + i * kThreads;
        if (k >= nvec) continue;
        const uint32_t e = 4 * k;
        const uint32_t row = fdiv(e, divT);
        const uint32_t col = e - row * T;
        const uint32_t c = row - fdiv(row, divC) * C;
        const float a = __ldg(ea + c), b = __ldg(ieb + c);
        float4 r;
        if (col + 3 < T) {
            const float2 a2 = make_float2(a, a), b2 = make_float2(b, b);
            const float2 lo = snake2(make_float2(v[i].x, v[i].y), a2, b2);
            const float2 hi = snake2(make_float2(v[i].z, v[i].w), a2, b2);
            r = make_float4(lo.x, lo.y, hi.x, hi.y);
        } else {  // the vector crosses into the next row (T % 4 != 0)
            const uint32_t c2 = c + 1 == C ? 0 : c + 1;
            const float a2 = __ldg(ea + c2), b2 = __ldg(ieb + c2);
            r.x = col + 0 < T ? snake1(v[i].x, a, b) : snake1(v[i].x, a2, b2);
            r.y = col + 1 < T ? snake1(v[i].y, a, b) : snake1(v[i].y, a2, b2);
            r.z = col + 2 < T ? snake1(v[i].z, a, b) : snake1(v[i].z, a2, b2);
            r.w = snake1(v[i].w, a2, b2);
        }
        xv[k] = r;
    }
    if (blockIdx.x == 0 && threadIdx.x < total - 4 * nvec) {  // the last 1-3 elements
        const uint32_t e = 4 * nvec + threadIdx.x;
        const uint32_t row = fdiv(e, divT);
        const uint32_t c = row - fdiv(row, divC) * C;
        x[e] = snake1(x[e], __ldg(ea + c), __ldg(ieb + c));
    }
    pdl_launch_dependents();
}

}  // namespace
}  // namespace lai

extern "C" int lai_snake_beta_f32(float *x, const float *exp_alpha, const float *inv_exp_beta,
                                  int64_t batch, int channels, int64_t T, lai_stream_t stream) {
    if (!x || !exp_alpha || !inv_exp_beta || batch < 0 || channels <= 0 || T < 0)
        return LAI_ERR_INVALID;
    const int64_t rows = batch * channels;
    if (rows == 0 || T == 0) return LAI_OK;
    const bool vec = lai::aligned16(x);
    const int64_t total = rows * T;
    if (vec && T >= 4 && total < (int64_t)0xffffffffll) {
        const int64_t nvec = total / 4;
        lai::launch_pdl(lai::snake_flat_kernel, dim3(lai::grid_for(nvec > 0 ? nvec : 1, lai::kSegVec)),
                        dim3(lai::kThreads), 0, lai::as_stream(stream), x, exp_alpha, inv_exp_beta,
                        (uint32_t)total, (uint32_t)T, (uint32_t)channels,
                        lai::make_fastdiv((uint32_t)T), lai::make_fastdiv((uint32_t)channels));
        return lai::launch_status();
    }
    const int64_t nv_max = vec ? T / 4 + 1 : 0;
    const unsigned gx = lai::grid_for(nv_max, lai::kSegVec);
    const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
    lai::snake_kernel<<<dim3(gx, gy), lai::kThreads, 0, lai::as_stream(stream)>>>(
        x, exp_alpha, inv_exp_beta, rows, channels, T, vec);
    return lai::launch_status();
}

// snake.cu - vocoder SnakeBeta activation, FP32, in place.
//
// Reference: voc_snake_beta(x, exp_alpha, inv_exp_beta, C, T)
// (src/tts_vocoder_ops.c:279-305): x[c,t] += ieb[c] * sin(ea[c] * x[c,t])^2 with the
// parameters pre-exponentiated at load (src/tts_vocoder.c:221-227). The scalar
// branch of the reference computes x + ((ieb * s) * s) with separately rounded
// operations; this kernel does the same with CUDA's full-accuracy sinf (no fast
// math), so it differs from the reference only where the two sinf differ.
//
// Roofline: HBM, 8 bytes per element (read + write). The per-element arithmetic
// (sinf's range reduction and polynomial, ~30 instructions) keeps the kernel
// within reach of the FP32 issue rate at HBM speed.
//
// Layout: x is [batch*C rows, T]. Grid y walks rows, grid x walks 16 KiB
// segments of a row. A row starts 16-byte aligned only when row*T % 4 == 0, so
// each row is a scalar head (to the first aligned element), an aligned body of
// float4 vectors, and a scalar tail; CTA x == 0 of each row takes head and tail.
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kSegVec = kThreads * kUnroll;  // float4 vectors per CTA segment

__device__ __forceinline__ float snake1(float x, float ea, float ieb) {
    const float s = sinf(__fmul_rn(ea, x));
    return __fadd_rn(x, __fmul_rn(__fmul_rn(ieb, s), s));
}

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
                float4 r;
                r.x = snake1(v[i].x, a, b); r.y = snake1(v[i].y, a, b);
                r.z = snake1(v[i].z, a, b); r.w = snake1(v[i].w, a, b);
                xv[k] = r;
            }
        }
        if (blockIdx.x == 0) {
            // scalar head, scalar tail (whole row when !vec), strided over the CTA
            for (int64_t t = threadIdx.x; t < head; t += kThreads) xr[t] = snake1(xr[t], a, b);
            for (int64_t t = body_end + threadIdx.x; t < T; t += kThreads) xr[t] = snake1(xr[t], a, b);
        }
    }
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
    const int64_t nv_max = vec ? T / 4 + 1 : 0;
    const unsigned gx = lai::grid_for(nv_max, lai::kSegVec);
    const unsigned gy = (unsigned)(rows < 65535 ? rows : 65535);
    lai::snake_kernel<<<dim3(gx, gy), lai::kThreads, 0, lai::as_stream(stream)>>>(
        x, exp_alpha, inv_exp_beta, rows, channels, T, vec);
    return lai::launch_status();
}

// weights.cu - load-time weight preparation for the decode GEMVs (gemv.cu).
//
// The reference stores GPU decode weights as FP16 in its fp16 mode and as INT8 with a
// per-row scale in its int8 mode, converting from the BF16 safetensors when the model
// loads (src/tts_native.c:1185-1240; the recipe is in tools/asr_benchmarks.md:342-352:
// scale = max(abs(row)) / 127, int8[j] = round(row[j] / scale)). The conversion code
// itself lives in the qwen-asr GPU sources, which the reference does not vendor, so the
// rounding rules below are this file's statement of that recipe:
//   * BF16 -> FP16: round to nearest even (values beyond FP16's range become +-inf);
//   * INT8: scale = absmax / 127 in F32; q = round(w / scale) with IEEE division and
//     halves rounded away from zero (C roundf), clamped to [-127, 127]; a row of zeros
//     gets scale 0 and q = 0.
// One warp per row: a max-reduction pass, then the quantising pass (both coalesced, the
// row re-read from L2). Runs once per model load, not on the decode path.
#include "lai_common.cuh"

#include <cuda_fp16.h>
#include <math.h>

namespace lai {
namespace {

constexpr int kRowsPerCta = 8;  // one warp per row

__global__ void __launch_bounds__(32 * kRowsPerCta)
quantize_rows_i8_kernel(int8_t *q, float *scales, const uint16_t *__restrict__ w, int N, int K) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    if (row >= N) return;
    const uint16_t *wr = w + (size_t)row * K;
    float amax = 0.0f;
    for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(to_f(wr[k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = amax / 127.0f;
    if (lane == 0) scales[row] = scale;
    int8_t *qr = q + (size_t)row * K;
    for (int k = lane; k < K; k += 32) {
        float v = scale > 0.0f ? roundf(to_f(wr[k]) / scale) : 0.0f;
        v = fminf(fmaxf(v, -127.0f), 127.0f);
        qr[k] = (int8_t)(int)v;
    }
}

__global__ void bf16_to_f16_kernel(uint16_t *dst, const uint16_t *__restrict__ src, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        dst[i] = __half_as_ushort(__float2half_rn(to_f(src[i])));
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_quantize_rows_i8_bf16(int8_t *q, float *scales, const lai_bf16 *W, int N, int K,
                              lai_stream_t stream) {
    if (!q || !scales || !W || N < 0 || K <= 0) return LAI_ERR_INVALID;
    if (N == 0) return LAI_OK;
    if (lai::overlaps(q, (size_t)N * K, W, (size_t)N * K * 2) ||
        lai::overlaps(scales, (size_t)N * 4, W, (size_t)N * K * 2))
        return LAI_ERR_ALIAS;
    const unsigned grid = (unsigned)((N + lai::kRowsPerCta - 1) / lai::kRowsPerCta);
    lai::quantize_rows_i8_kernel<<<grid, 32 * lai::kRowsPerCta, 0, lai::as_stream(stream)>>>(
        q, scales, W, N, K);
    return lai::launch_status();
}

int lai_convert_bf16_to_f16(lai_f16 *dst, const lai_bf16 *src, int64_t n, lai_stream_t stream) {
    if (!dst || !src || n < 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    if (lai::overlaps(dst, (size_t)n * 2, src, (size_t)n * 2)) return LAI_ERR_ALIAS;
    lai::bf16_to_f16_kernel<<<lai::grid_for(n, 256), 256, 0, lai::as_stream(stream)>>>(dst, src, n);
    return lai::launch_status();
}

}  // extern "C"

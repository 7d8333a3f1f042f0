// synth.cu - seeded, counter-based synthetic inputs for benchmarks and tests.
//
// Element i of a fill is a pure function of (seed, offset + i): a SplitMix64
// finaliser over the counter gives 64 random bits, Box-Muller turns two 32-bit
// halves into one normal sample. A row-sharded fill on G devices (offset = first
// global element of the shard) therefore equals the single-device fill.
#include "lai_common.cuh"

namespace lai {
namespace {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
    const uint64_t r = mix64(seed * 0xd1b54a32d192ed03ull + i);
    const float u1 = ((uint32_t)(r >> 40) + 1u) * (1.0f / 16777217.0f);  // (0, 1]
    const float u2 = (uint32_t)(r & 0xffffffu) * (1.0f / 16777216.0f);   // [0, 1)
    return sqrtf(-2.0f * __logf(u1)) * __cosf(6.28318530718f * u2);
}

template <typename T>
__global__ void __launch_bounds__(256)
normal_kernel(T *out, int64_t n, uint64_t seed, int64_t offset, float mean, float stdv) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        out[i] = from_f<T>(fmaf(stdv, normal_at(seed, (uint64_t)(offset + i)), mean));
}

__global__ void __launch_bounds__(256)
uniform_i32_kernel(int32_t *out, int64_t n, uint64_t seed, int64_t offset, int32_t lo, uint32_t span) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const uint64_t r = mix64(seed * 0xd1b54a32d192ed03ull + (uint64_t)(offset + i));
        out[i] = lo + (int32_t)(((r >> 32) * (uint64_t)span) >> 32);
    }
}

inline unsigned fill_grid(int64_t n) {
    const int64_t g = (n + 255) / 256;
    return (unsigned)(g < 1 ? 1 : (g > 148 * 64 ? 148 * 64 : g));
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_synth_normal_bf16(lai_bf16 *out, int64_t n, uint64_t seed, int64_t offset, float mean,
                          float std, lai_stream_t stream) {
    if (!out || n < 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    lai::normal_kernel<uint16_t><<<lai::fill_grid(n), 256, 0, lai::as_stream(stream)>>>(
        out, n, seed, offset, mean, std);
    return lai::launch_status();
}

int lai_synth_normal_f32(float *out, int64_t n, uint64_t seed, int64_t offset, float mean,
                         float std, lai_stream_t stream) {
    if (!out || n < 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    lai::normal_kernel<float><<<lai::fill_grid(n), 256, 0, lai::as_stream(stream)>>>(
        out, n, seed, offset, mean, std);
    return lai::launch_status();
}

int lai_synth_uniform_i32(int32_t *out, int64_t n, uint64_t seed, int64_t offset, int32_t lo,
                          int32_t hi, lai_stream_t stream) {
    if (!out || n < 0 || hi <= lo) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    lai::uniform_i32_kernel<<<lai::fill_grid(n), 256, 0, lai::as_stream(stream)>>>(
        out, n, seed, offset, lo, (uint32_t)((int64_t)hi - lo));
    return lai::launch_status();
}

}  // extern "C"

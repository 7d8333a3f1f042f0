// lai_common.cuh - shared device helpers for the sm_100a per-layer kernels.
//
// Every kernel here is HBM-bound elementwise or row-reduction work: 16-byte
// vector loads/stores (8 BF16 or 4 FP32 per lane), FP32 arithmetic, warp-shuffle
// reductions. No tensor cores (nothing here is a contraction).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lai_kernels.h"

namespace lai {

constexpr int kWarp = 32;

// ---- status helpers -------------------------------------------------------
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LAI_OK : LAI_ERR_CUDA;
}
inline cudaStream_t as_stream(lai_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- programmatic dependent launch ------------------------------------------------
// A kernel launched with launch_pdl may start while the previous kernel on the stream is
// still finishing: it must call pdl_wait_prior() before it reads anything that kernel
// wrote, and pdl_launch_dependents() lets the next PDL-launched kernel start in turn.
// Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Byte ranges [a, a+na) and [b, b+nb) overlap.
inline bool overlaps(const void *a, size_t na, const void *b, size_t nb) {
    uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + nb && y < x + na;
}

// Grid helper: CTAs needed for `work` items at `per_cta` items each.
inline unsigned grid_for(int64_t work, int64_t per_cta) {
    int64_t g = (work + per_cta - 1) / per_cta;
    return static_cast<unsigned>(g < 1 ? 1 : g);
}

// ---- BF16 bit helpers -----------------------------------------------------
// Widening is exact (bits << 16). Narrowing is round-to-nearest-even.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// RNE narrowing with the hardware conversion (NaN -> canonical 0x7fff).
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    unsigned short r;
    asm("cvt.rn.bf16.f32 %0, %1;" : "=h"(r) : "f"(f));
    return r;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---- 16-byte vector <-> floats ------------------------------------------------
// Elt<T>::N elements per 16-byte vector: 8 for BF16 (uint16_t), 4 for FP32.
template <typename T> struct Elt;
template <> struct Elt<uint16_t> { static constexpr int N = 8; };
template <> struct Elt<float> { static constexpr int N = 4; };

template <typename T>
__device__ __forceinline__ void unpack(const uint4 &v, float (&f)[Elt<T>::N]);
template <>
__device__ __forceinline__ void unpack<uint16_t>(const uint4 &v, float (&f)[8]) {
    f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x); f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
    f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z); f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
}
template <>
__device__ __forceinline__ void unpack<float>(const uint4 &v, float (&f)[4]) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
}

template <typename T>
__device__ __forceinline__ uint4 pack(const float (&f)[Elt<T>::N]);
template <>
__device__ __forceinline__ uint4 pack<uint16_t>(const float (&f)[8]) {
    return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                      pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}
template <>
__device__ __forceinline__ uint4 pack<float>(const float (&f)[4]) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
}

// Scalar element access for the ragged / unaligned fallbacks.
__device__ __forceinline__ float to_f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }
__device__ __forceinline__ float to_f(float f) { return f; }
template <typename T> __device__ __forceinline__ T from_f(float f);
template <> __device__ __forceinline__ uint16_t from_f<uint16_t>(float f) {
    return static_cast<uint16_t>(f32_to_bf16_bits(f));
}
template <> __device__ __forceinline__ float from_f<float>(float f) { return f; }

// ---- memory access -------------------------------------------------------------
// Streaming reads of data touched once: non-coherent path, no L1 allocation.
__device__ __forceinline__ uint4 ld_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
// Reads of data this kernel may also write (in-place rows): coherent path.
__device__ __forceinline__ uint4 ld_rw(const void *p) {
    return *reinterpret_cast<const uint4 *>(p);
}
__device__ __forceinline__ void st_vec(void *p, const uint4 &v) {
    *reinterpret_cast<uint4 *>(p) = v;
}
__device__ __forceinline__ float4 ld_f4(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
}

// ---- reductions ------------------------------------------------------------------
template <int WIDTH = 32>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Sum over a CTA (blockDim.x a multiple of 32, <= 1024); every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float *smem32) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = group_sum<32>(v);
    __syncthreads();  // smem32 may still be in use by a previous call
    if (lane == 0) smem32[wid] = v;
    __syncthreads();
    float t = lane < nw ? smem32[lane] : 0.f;
    return group_sum<32>(t);
}

}  // namespace lai

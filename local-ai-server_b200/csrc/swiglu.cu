// swiglu.cu - SwiGLU over the interleaved gate/up GEMM output, SiLU, SiLU*up.
//
// Reference semantics: qwen_swiglu_multiply(out, gate_up, seq, inter) with the
// gate/up weight rows interleaved (src/tts_native.c:149-161), called with
// out == gate_up (src/tts_native.c:588, 665, 744); SiLU*up written as
// src/tts_vocoder_xfmr.c:76-78. Flattened over rows the op is
// out[k] = silu(in[2k]) * in[2k+1], k < rows*inter.
//
// Roofline: HBM. Algorithmic bytes per token: 3 * inter * s (read 2*inter, write
// inter). A "unit" is one 16-byte input vector (4 BF16 or 2 FP32 gate/up pairs)
// producing one 8-byte output; warps read 512 contiguous bytes and write 256.
//
// In place without scratch. Unit k reads input bytes [16k, 16k+16) and writes
// output bytes [8k, 8k+8), which hold the input of unit k/2. Units are therefore
// processed in waves [L, 2L): a wave reads [16L, 32L) and writes [8L, 16L) --
// disjoint -- and its writes only clobber inputs of the previous wave. Wave 0
// ([0, kHeadUnits)) runs inside one CTA as sub-waves [0,1), [1,2), [2,4), ...
// separated by __syncthreads; every later wave is one launch, ordered by the
// stream. The ragged tail (inter*rows not a multiple of the unit width) is one
// final serial step. log2(units / kHeadUnits) + 2 launches in total.
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int64_t kHeadUnits = 8192;

// silu(g) * u. BF16 results are rounded to 8 significant bits, so the fast
// exponential and divide (relative error ~1e-6) are used there; FP32 uses the
// correctly rounded forms of the reference expression (g * (1/(1+e^-g))) * u.
template <typename T> __device__ __forceinline__ float silu_mul(float g, float u);
template <> __device__ __forceinline__ float silu_mul<uint16_t>(float g, float u) {
    return __fdividef(g, 1.0f + __expf(-g)) * u;
}
template <> __device__ __forceinline__ float silu_mul<float>(float g, float u) {
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

template <typename T> __device__ __forceinline__ uint2 unit_op(const uint4 &v);
template <> __device__ __forceinline__ uint2 unit_op<uint16_t>(const uint4 &v) {
    return make_uint2(pack_bf16x2(silu_mul<uint16_t>(bf16_lo(v.x), bf16_hi(v.x)),
                                  silu_mul<uint16_t>(bf16_lo(v.y), bf16_hi(v.y))),
                      pack_bf16x2(silu_mul<uint16_t>(bf16_lo(v.z), bf16_hi(v.z)),
                                  silu_mul<uint16_t>(bf16_lo(v.w), bf16_hi(v.w))));
}
template <> __device__ __forceinline__ uint2 unit_op<float>(const uint4 &v) {
    return make_uint2(
        __float_as_uint(silu_mul<float>(__uint_as_float(v.x), __uint_as_float(v.y))),
        __float_as_uint(silu_mul<float>(__uint_as_float(v.z), __uint_as_float(v.w))));
}

// Units [u0, u1), each CTA a contiguous block of kThreads*kUnroll units.
// Loads are all issued before any store; reads and writes never overlap here
// (out-of-place, or one wave of the in-place schedule).
template <typename T>
__global__ void __launch_bounds__(kThreads)
swiglu_units_kernel(uint2 *out, const uint4 *in, int64_t u0, int64_t u1) {
    const int64_t base = u0 + (int64_t)blockIdx.x * (kThreads * kUnroll) + threadIdx.x;
    uint4 v[kUnroll];
#pragma unroll
    for (int i = 0; i < kUnroll; i++) {
        const int64_t k = base + (int64_t)i * kThreads;
        if (k < u1) v[i] = ld_stream(in + k);
    }
#pragma unroll
    for (int i = 0; i < kUnroll; i++) {
        const int64_t k = base + (int64_t)i * kThreads;
        if (k < u1) out[k] = unit_op<T>(v[i]);
    }
}

// Scalar elements [k0, k1) in increasing order by one thread: the ragged tail,
// in place or not (the serial order is the reference's own).
template <typename T>
__global__ void swiglu_serial_kernel(T *out, const T *in, int64_t k0, int64_t k1) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (int64_t k = k0; k < k1; k++) out[k] = from_f<T>(silu_mul<T>(to_f(in[2 * k]), to_f(in[2 * k + 1])));
}

// Wave 0 of the in-place schedule in one CTA: sub-waves [0,1), [1,2), [2,4), ...
// up to `u1` units, then (if `tail_k1` > `tail_k0`) the serial tail.
template <typename T>
__global__ void __launch_bounds__(1024)
swiglu_inplace_head_kernel(T *buf, int64_t u1, int64_t tail_k0, int64_t tail_k1) {
    uint2 *out = reinterpret_cast<uint2 *>(buf);
    const uint4 *in = reinterpret_cast<const uint4 *>(buf);
    int64_t lo = 0, hi = u1 < 1 ? u1 : 1;
    while (lo < u1) {
        for (int64_t k = lo + threadIdx.x; k < hi; k += blockDim.x) {
            const uint4 v = ld_rw(in + k);  // written earlier in this kernel? never: reads run ahead
            out[k] = unit_op<T>(v);
        }
        __syncthreads();
        lo = hi;
        hi = 2 * hi < u1 ? 2 * hi : u1;
    }
    if (threadIdx.x == 0)
        for (int64_t k = tail_k0; k < tail_k1; k++)
            buf[k] = from_f<T>(silu_mul<T>(to_f(buf[2 * k]), to_f(buf[2 * k + 1])));
}

// Scalar-unit variant of the wave schedule for unaligned in-place buffers:
// unit = one output element (reads 2 elements, writes 1); same wave algebra.
template <typename T>
__global__ void __launch_bounds__(kThreads)
swiglu_scalar_units_kernel(T *out, const T *in, int64_t u0, int64_t u1) {
    const int64_t k = u0 + (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (k < u1) {
        const float g = to_f(in[2 * k]), u = to_f(in[2 * k + 1]);
        out[k] = from_f<T>(silu_mul<T>(g, u));
    }
}
template <typename T>
__global__ void __launch_bounds__(1024) swiglu_scalar_head_kernel(T *buf, int64_t u1) {
    int64_t lo = 0, hi = u1 < 1 ? u1 : 1;
    while (lo < u1) {
        for (int64_t k = lo + threadIdx.x; k < hi; k += blockDim.x) {
            const float g = to_f(buf[2 * k]), u = to_f(buf[2 * k + 1]);
            buf[k] = from_f<T>(silu_mul<T>(g, u));
        }
        __syncthreads();
        lo = hi;
        hi = 2 * hi < u1 ? 2 * hi : u1;
    }
}

template <typename T>
int run(T *out, const T *in, int64_t rows, int inter, lai_stream_t stream) {
    if (!out || !in || rows < 0 || inter <= 0) return LAI_ERR_INVALID;
    const int64_t n = rows * (int64_t)inter;  // outputs
    if (n == 0) return LAI_OK;
    const bool inplace = static_cast<const void *>(out) == static_cast<const void *>(in);
    if (!inplace && overlaps(out, (size_t)n * sizeof(T), in, (size_t)2 * n * sizeof(T)))
        return LAI_ERR_ALIAS;
    cudaStream_t s = as_stream(stream);
    constexpr int P = 8 / (int)sizeof(T);  // outputs per unit
    const bool vec = aligned16(in) && aligned16(out);

    if (vec) {
        const int64_t units = n / P, tail0 = units * P;
        uint2 *o = reinterpret_cast<uint2 *>(out);
        const uint4 *iv = reinterpret_cast<const uint4 *>(in);
        if (!inplace) {
            if (units > 0)
                swiglu_units_kernel<T><<<grid_for(units, kThreads * kUnroll), kThreads, 0, s>>>(o, iv, 0, units);
            if (tail0 < n) swiglu_serial_kernel<T><<<1, 32, 0, s>>>(out, in, tail0, n);
            return launch_status();
        }
        const int64_t head = units < kHeadUnits ? units : kHeadUnits;
        const bool tail_in_head = head == units;
        swiglu_inplace_head_kernel<T><<<1, 1024, 0, s>>>(out, head, tail_in_head ? tail0 : 0,
                                                         tail_in_head ? n : 0);
        for (int64_t lo = head; lo < units;) {
            const int64_t hi = 2 * lo < units ? 2 * lo : units;
            swiglu_units_kernel<T><<<grid_for(hi - lo, kThreads * kUnroll), kThreads, 0, s>>>(o, iv, lo, hi);
            lo = hi;
        }
        if (!tail_in_head && tail0 < n) swiglu_serial_kernel<T><<<1, 32, 0, s>>>(out, in, tail0, n);
        return launch_status();
    }

    if (!inplace) {
        swiglu_scalar_units_kernel<T><<<grid_for(n, kThreads), kThreads, 0, s>>>(out, in, 0, n);
        return launch_status();
    }
    const int64_t head = n < kHeadUnits ? n : kHeadUnits;
    swiglu_scalar_head_kernel<T><<<1, 1024, 0, s>>>(out, head);
    for (int64_t lo = head; lo < n;) {
        const int64_t hi = 2 * lo < n ? 2 * lo : n;
        swiglu_scalar_units_kernel<T><<<grid_for(hi - lo, kThreads), kThreads, 0, s>>>(out, in, lo, hi);
        lo = hi;
    }
    return launch_status();
}

// ---- flat FP32 elementwise: SiLU in place, SiLU(gate)*up --------------------------
__device__ __forceinline__ float silu_f32(float g) {
    return __fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))));
}

__global__ void __launch_bounds__(kThreads) silu_kernel(float *x, int64_t n) {
    const int64_t nv = n / 4;
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (i < nv) {
        float4 v = reinterpret_cast<float4 *>(x)[i];
        v.x = silu_f32(v.x); v.y = silu_f32(v.y); v.z = silu_f32(v.z); v.w = silu_f32(v.w);
        reinterpret_cast<float4 *>(x)[i] = v;
    }
    if (i < n - nv * 4) x[nv * 4 + i] = silu_f32(x[nv * 4 + i]);
}
__global__ void __launch_bounds__(kThreads) silu_scalar_kernel(float *x, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (i < n) x[i] = silu_f32(x[i]);
}

__global__ void __launch_bounds__(kThreads)
swiglu_sep_kernel(float *out, const float *gate, const float *up, int64_t n) {
    const int64_t nv = n / 4;
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (i < nv) {
        const float4 g = __ldg(reinterpret_cast<const float4 *>(gate) + i);
        const float4 u = __ldg(reinterpret_cast<const float4 *>(up) + i);
        float4 r;
        r.x = silu_mul<float>(g.x, u.x); r.y = silu_mul<float>(g.y, u.y);
        r.z = silu_mul<float>(g.z, u.z); r.w = silu_mul<float>(g.w, u.w);
        reinterpret_cast<float4 *>(out)[i] = r;
    }
    if (i < n - nv * 4) out[nv * 4 + i] = silu_mul<float>(gate[nv * 4 + i], up[nv * 4 + i]);
}
__global__ void __launch_bounds__(kThreads)
swiglu_sep_scalar_kernel(float *out, const float *gate, const float *up, int64_t n) {
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (i < n) out[i] = silu_mul<float>(gate[i], up[i]);
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_swiglu_bf16(lai_bf16 *out, const lai_bf16 *gate_up, int64_t rows, int inter,
                    lai_stream_t stream) {
    return lai::run<uint16_t>(out, gate_up, rows, inter, stream);
}
int lai_swiglu_f32(float *out, const float *gate_up, int64_t rows, int inter,
                   lai_stream_t stream) {
    return lai::run<float>(out, gate_up, rows, inter, stream);
}

int lai_silu_f32(float *x, int64_t n, lai_stream_t stream) {
    if (!x || n < 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    cudaStream_t s = lai::as_stream(stream);
    if (lai::aligned16(x))
        lai::silu_kernel<<<lai::grid_for(n / 4 > 4 ? n / 4 : 4, lai::kThreads), lai::kThreads, 0, s>>>(x, n);
    else
        lai::silu_scalar_kernel<<<lai::grid_for(n, lai::kThreads), lai::kThreads, 0, s>>>(x, n);
    return lai::launch_status();
}

int lai_swiglu_separate_f32(float *out, const float *gate, const float *up, int64_t n,
                            lai_stream_t stream) {
    if (!out || !gate || !up || n < 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    const size_t b = (size_t)n * 4;
    if ((out != gate && lai::overlaps(out, b, gate, b)) || (out != up && lai::overlaps(out, b, up, b)))
        return LAI_ERR_ALIAS;
    cudaStream_t s = lai::as_stream(stream);
    if (lai::aligned16(out) && lai::aligned16(gate) && lai::aligned16(up))
        lai::swiglu_sep_kernel<<<lai::grid_for(n / 4 > 4 ? n / 4 : 4, lai::kThreads), lai::kThreads, 0, s>>>(out, gate, up, n);
    else
        lai::swiglu_sep_scalar_kernel<<<lai::grid_for(n, lai::kThreads), lai::kThreads, 0, s>>>(out, gate, up, n);
    return lai::launch_status();
}

}  // extern "C"

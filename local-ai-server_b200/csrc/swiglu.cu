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
// disjoint -- and its writes only clobber inputs of the previous wave, so a wave's
// writes may start once every read of the previous wave is done. A cooperative
// launch (every CTA resident) runs the start of the schedule: a head of H units (H =
// the grid's threads x kHeadRegs, ~0.9M) is read into registers, one grid-wide
// barrier, then written; the small waves [H, 2H), [2H, 4H), ... follow, each separated
// from the next by one grid-wide barrier (the wave right after the head needs none: its
// writes clobber head inputs, all read before the head's barrier). Waves of
// kCoopWaveMax units or more are ordinary launches ordered by the stream (the
// persistent grid-stride loop streams them ~30% below a fresh grid). The ragged tail
// (inter*rows not a multiple of the unit width) is one serial step at the end. At
// 65536 x 6144 that is one cooperative launch and 4 wave launches; one launch per wave
// with a one-CTA head, as before, cost 19% over the out-of-place form there (launch gaps
// and tails of ~15 dependent launches), the whole schedule in the cooperative launch 43%.
// Unaligned buffers keep the per-launch wave form with scalar units.
#include <cooperative_groups.h>

#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 2;      // units per thread: 2 beat 4 and 8 (65 536 x 6144: 345 vs 350 us)
constexpr int kSiluUnroll = 4;  // float4 per thread in silu_kernel
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
    pdl_wait_prior();  // launched with programmatic dependent launch: inputs after this
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
    pdl_launch_dependents();
}

// The whole in-place schedule in one cooperative launch (described at the top).
constexpr int kCoopThreads = 256;
constexpr int kCoopMinCtas = 6;  // 1536 threads per SM without spills
constexpr int kHeadRegs = 4;     // head units held in registers per thread
constexpr int64_t kCoopWaveMax = 4 << 20;  // units: larger waves are ordinary launches

__device__ __forceinline__ uint4 ld_l2(const uint4 *p) {  // L2 only: bytes change under us
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// The head and every wave up to unit `u_stop` (a wave boundary); with u_stop == units
// also the ragged tail [tail0, n).
template <typename T>
__global__ void __launch_bounds__(kCoopThreads, kCoopMinCtas)
swiglu_inplace_coop_kernel(T *buf, int64_t units, int64_t u_stop, int64_t tail0, int64_t n) {
    namespace cg = cooperative_groups;
    cg::grid_group grid = cg::this_grid();
    uint2 *out = reinterpret_cast<uint2 *>(buf);
    const uint4 *in = reinterpret_cast<const uint4 *>(buf);
    const int64_t nt = (int64_t)gridDim.x * kCoopThreads;
    const int64_t t = (int64_t)blockIdx.x * kCoopThreads + threadIdx.x;
    const int64_t head = units < nt * kHeadRegs ? units : nt * kHeadRegs;
    {
        uint4 v[kHeadRegs];
#pragma unroll
        for (int r = 0; r < kHeadRegs; r++)
            if (t + r * nt < head) v[r] = ld_l2(in + t + r * nt);
        grid.sync();  // every head unit read before any is written
#pragma unroll
        for (int r = 0; r < kHeadRegs; r++)
            if (t + r * nt < head) out[t + r * nt] = unit_op<T>(v[r]);
    }
    // waves: each CTA takes contiguous blocks of kCoopThreads * kUnroll units (8 KB read)
    constexpr int64_t kBlock = (int64_t)kCoopThreads * kUnroll;
    for (int64_t lo = head; lo < u_stop;) {
        const int64_t hi = 2 * lo < units ? 2 * lo : units;
        if (lo > head) grid.sync();  // the previous wave's reads before this wave's writes
        for (int64_t b0 = lo + (int64_t)blockIdx.x * kBlock + threadIdx.x; b0 < hi;
             b0 += (int64_t)gridDim.x * kBlock) {
            uint4 v[kUnroll];
#pragma unroll
            for (int i = 0; i < kUnroll; i++)
                if (b0 + i * kCoopThreads < hi) v[i] = ld_l2(in + b0 + i * kCoopThreads);
#pragma unroll
            for (int i = 0; i < kUnroll; i++)
                if (b0 + i * kCoopThreads < hi) out[b0 + i * kCoopThreads] = unit_op<T>(v[i]);
        }
        lo = hi;
    }
    if (u_stop == units && tail0 < n) {
        grid.sync();  // the last wave's reads before the tail's writes
        if (t == 0)
            for (int64_t k = tail0; k < n; k++)
                buf[k] = from_f<T>(silu_mul<T>(to_f(buf[2 * k]), to_f(buf[2 * k + 1])));
    }
}

// Scalar elements [k0, k1) in increasing order by one thread: the ragged tail,
// in place or not (the serial order is the reference's own).
template <typename T>
__global__ void swiglu_serial_kernel(T *out, const T *in, int64_t k0, int64_t k1) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    for (int64_t k = k0; k < k1; k++) out[k] = from_f<T>(silu_mul<T>(to_f(in[2 * k]), to_f(in[2 * k + 1])));
}

// Scalar-unit wave schedule for unaligned in-place buffers: unit = one output element
// (reads 2 elements, writes 1); the same wave algebra, wave 0 as sub-waves inside one
// CTA separated by __syncthreads, every later wave one launch ordered by the stream.
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

// CTAs of a cooperative launch of `kern` for `units` units: every SM's resident
// share (cached per device), no more than the units need. 0 on error.
template <typename K>
int coop_grid(K kern, int64_t units) {
    static int resident[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (resident[dev] == 0) {
        int sms = 0, per_sm = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kCoopThreads, 0) !=
                cudaSuccess || per_sm <= 0) {
            cudaGetLastError();
            return 0;
        }
        resident[dev] = sms * per_sm;
    }
    const int64_t need = (units + kCoopThreads - 1) / kCoopThreads;
    return (int)(need < resident[dev] ? need : resident[dev]);
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
                launch_pdl(swiglu_units_kernel<T>, dim3(grid_for(units, kThreads * kUnroll)),
                           dim3(kThreads), 0, s, o, iv, (int64_t)0, units);
            if (tail0 < n) swiglu_serial_kernel<T><<<1, 32, 0, s>>>(out, in, tail0, n);
            return launch_status();
        }
        if (units == 0) {
            swiglu_serial_kernel<T><<<1, 32, 0, s>>>(out, in, 0, n);
            return launch_status();
        }
        const int grid = coop_grid(swiglu_inplace_coop_kernel<T>, units);
        if (grid <= 0) return LAI_ERR_CUDA;
        // the same wave boundaries as the kernel: head, then doubling waves; the
        // cooperative launch stops before the first wave of kCoopWaveMax units or more
        const int64_t head_cap = (int64_t)grid * kCoopThreads * kHeadRegs;
        int64_t u_stop = units < head_cap ? units : head_cap;
        while (u_stop < units) {
            const int64_t hi = 2 * u_stop < units ? 2 * u_stop : units;
            if (hi - u_stop >= kCoopWaveMax) break;
            u_stop = hi;
        }
        int64_t units_a = units, stop_a = u_stop, tail_a = tail0, n_a = n;
        void *args[] = {&out, &units_a, &stop_a, &tail_a, &n_a};
        if (cudaLaunchCooperativeKernel((const void *)swiglu_inplace_coop_kernel<T>, grid,
                                        kCoopThreads, args, 0, s) != cudaSuccess) {
            cudaGetLastError();
            return LAI_ERR_CUDA;
        }
        for (int64_t lo = u_stop; lo < units;) {
            const int64_t hi = 2 * lo < units ? 2 * lo : units;
            launch_pdl(swiglu_units_kernel<T>, dim3(grid_for(hi - lo, kThreads * kUnroll)),
                       dim3(kThreads), 0, s, o, iv, lo, hi);
            lo = hi;
        }
        if (u_stop < units && tail0 < n) swiglu_serial_kernel<T><<<1, 32, 0, s>>>(out, in, tail0, n);
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

// kSiluUnroll float4 per thread, all loaded before any store; threads of block 0 also take
// the 1-3 trailing elements.
__global__ void __launch_bounds__(kThreads) silu_kernel(float *x, int64_t n) {
    const int64_t nv = n / 4;
    const int64_t base = (int64_t)blockIdx.x * (kThreads * kSiluUnroll) + threadIdx.x;
    float4 v[kSiluUnroll];
#pragma unroll
    for (int j = 0; j < kSiluUnroll; j++) {
        const int64_t i = base + (int64_t)j * kThreads;
        if (i < nv) v[j] = reinterpret_cast<float4 *>(x)[i];
    }
#pragma unroll
    for (int j = 0; j < kSiluUnroll; j++) {
        const int64_t i = base + (int64_t)j * kThreads;
        if (i < nv) {
            float4 t = v[j];
            t.x = silu_f32(t.x); t.y = silu_f32(t.y); t.z = silu_f32(t.z); t.w = silu_f32(t.w);
            reinterpret_cast<float4 *>(x)[i] = t;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x < n - nv * 4) x[nv * 4 + threadIdx.x] = silu_f32(x[nv * 4 + threadIdx.x]);
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
        lai::silu_kernel<<<lai::grid_for(n / 4 > 0 ? n / 4 : 1, lai::kThreads * lai::kSiluUnroll),
                           lai::kThreads, 0, s>>>(x, n);
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

// rmsnorm.cu - RMSNorm and fused residual-add + RMSNorm (BF16 and FP32 storage).
//
// Reference semantics: qwen_rms_norm(out, x, w, seq, dim, eps) and the pair
// qwen_add_inplace(x, delta) ; qwen_rms_norm(y, x, w) as talker_prefill calls them
// (src/tts_native.c:556, 582-584); math per tools/verify_xfmr.py:32-35.
//
// Roofline: HBM. Algorithmic bytes per row: RMSNorm 2*D*s (read x, write y),
// add+RMSNorm 4*D*s (read x, delta; write x', y), s = element size; the weight
// vector (D*4 bytes) is shared by every row and stays in L1/L2.
//
// Fast path: one warp per row, NV 16-byte vectors per lane held in registers, so
// the row makes exactly one trip from HBM and one back. The sum of squares is a
// per-lane FP32 partial then a 5-step xor-shuffle tree. Rows that are not a
// multiple of 256 bytes per warp pass, or unaligned pointers, take the block
// fallback (any width, one CTA per row, second pass re-reads the row from L1/L2).
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kRowsPerCta = 8;  // 8 warps, one row each
// RMSNorm alone runs three CTAs per SM (<= 85 registers): 0.90 -> 0.92-0.93 of the measured
// copy bandwidth at 65 536 x 2048 (ptxas otherwise settles at 96 registers, two CTAs per SM).
// The fused add form keeps the default: at three CTAs per SM it was 1% slower.
constexpr int kPlainMinCtas = 3;

template <typename T, int NV, bool ADD>
__device__ __forceinline__ void rmsnorm_warp_body(T *__restrict__ y, T *x, const T *__restrict__ delta,
                                                  const float *__restrict__ w, int64_t rows, int dim,
                                                  float eps) {
    constexpr int E = Elt<T>::N;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
    if (row >= rows) return;
    pdl_wait_prior();  // launched with programmatic dependent launch: inputs after this

    const size_t off = (size_t)row * dim;
    uint4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; i++) v[i] = ld_stream(x + off + (size_t)(i * 32 + lane) * E);

    float ss = 0.f;
    if constexpr (ADD) {
        uint4 d[NV];
#pragma unroll
        for (int i = 0; i < NV; i++) d[i] = ld_stream(delta + off + (size_t)(i * 32 + lane) * E);
#pragma unroll
        for (int i = 0; i < NV; i++) {
            float a[E], b[E];
            unpack<T>(v[i], a);
            unpack<T>(d[i], b);
#pragma unroll
            for (int e = 0; e < E; e++) a[e] = __fadd_rn(a[e], b[e]);
            v[i] = pack<T>(a);  // x' rounded to storage precision, then normalised
            st_vec(x + off + (size_t)(i * 32 + lane) * E, v[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < NV; i++) {
        float a[E];
        unpack<T>(v[i], a);
#pragma unroll
        for (int e = 0; e < E; e++) ss = fmaf(a[e], a[e], ss);
    }
    ss = group_sum<32>(ss);
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);

#pragma unroll
    for (int i = 0; i < NV; i++) {
        const int c = (i * 32 + lane) * E;
        float a[E], wv[E];
        unpack<T>(v[i], a);
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            float4 t = ld_f4(w + c + e);
            wv[e] = t.x; wv[e + 1] = t.y; wv[e + 2] = t.z; wv[e + 3] = t.w;
        }
#pragma unroll
        for (int e = 0; e < E; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), wv[e]);
        st_vec(y + off + c, pack<T>(a));
    }
    pdl_launch_dependents();  // this row is done: the next kernel may start launching
}

template <typename T, int NV>
__global__ void __launch_bounds__(kRowsPerCta * 32)
rmsnorm_warp_add_kernel(T *__restrict__ y, T *x, const T *__restrict__ delta,
                        const float *__restrict__ w, int64_t rows, int dim, float eps) {
    rmsnorm_warp_body<T, NV, true>(y, x, delta, w, rows, dim, eps);
}
template <typename T, int NV>
__global__ void __launch_bounds__(kRowsPerCta * 32, kPlainMinCtas)
rmsnorm_warp_kernel(T *__restrict__ y, T *x, const T *__restrict__ delta,
                    const float *__restrict__ w, int64_t rows, int dim, float eps) {
    rmsnorm_warp_body<T, NV, false>(y, x, delta, w, rows, dim, eps);
}

// Any width / alignment: one CTA per row (grid-stride over rows).
template <typename T, bool ADD>
__global__ void __launch_bounds__(256)
rmsnorm_block_kernel(T *y, T *x, const T *delta, const float *__restrict__ w, int64_t rows,
                     int dim, float eps) {
    __shared__ float red[32];
    for (int64_t row = blockIdx.x; row < rows; row += gridDim.x) {
        T *xr = x + (size_t)row * dim;
        float ss = 0.f;
        for (int i = threadIdx.x; i < dim; i += blockDim.x) {
            float a = to_f(xr[i]);
            if constexpr (ADD) {
                T r = from_f<T>(__fadd_rn(a, to_f(delta[(size_t)row * dim + i])));
                xr[i] = r;
                a = to_f(r);
            }
            ss = fmaf(a, a, ss);
        }
        ss = block_sum(ss, red);
        const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
        T *yr = y + (size_t)row * dim;
        for (int i = threadIdx.x; i < dim; i += blockDim.x)
            yr[i] = from_f<T>(__fmul_rn(__fmul_rn(to_f(xr[i]), inv), w[i]));
    }
}

template <typename T, bool ADD, int NV>
void launch_warp(T *y, T *x, const T *delta, const float *w, int64_t rows, int dim, float eps,
                 cudaStream_t s) {
    launch_pdl(ADD ? rmsnorm_warp_add_kernel<T, NV> : rmsnorm_warp_kernel<T, NV>,
               dim3(grid_for(rows, kRowsPerCta)), dim3(kRowsPerCta * 32), 0, s, y, x, delta, w,
               rows, dim, eps);
}

template <typename T, bool ADD>
int run(T *y, T *x, const T *delta, const float *w, int64_t rows, int dim, float eps,
        lai_stream_t stream) {
    if (rows < 0 || dim <= 0 || !x || !y || !w || (ADD && !delta)) return LAI_ERR_INVALID;
    if (rows == 0) return LAI_OK;
    const size_t bytes = (size_t)rows * dim * sizeof(T);
    if (ADD && (overlaps(y, bytes, x, bytes) || overlaps(y, bytes, delta, bytes)))
        return LAI_ERR_ALIAS;
    cudaStream_t s = as_stream(stream);
    constexpr int E = Elt<T>::N;
    const bool vec_ok = dim % (32 * E) == 0 && aligned16(x) && aligned16(y) && aligned16(w) &&
                        (!ADD || aligned16(delta));
    const int nv = dim / (32 * E);
    if (vec_ok) {
        switch (nv) {
            case 1: launch_warp<T, ADD, 1>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 2: launch_warp<T, ADD, 2>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 3: launch_warp<T, ADD, 3>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 4: launch_warp<T, ADD, 4>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 6: launch_warp<T, ADD, 6>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 8: launch_warp<T, ADD, 8>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 12: launch_warp<T, ADD, 12>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            case 16: launch_warp<T, ADD, 16>(y, x, delta, w, rows, dim, eps, s); return launch_status();
            default: break;
        }
    }
    const int64_t g = rows < 65536 * 16 ? rows : 65536 * 16;
    rmsnorm_block_kernel<T, ADD><<<(unsigned)g, 256, 0, s>>>(y, x, delta, w, rows, dim, eps);
    return launch_status();
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_rmsnorm_bf16(lai_bf16 *y, const lai_bf16 *x, const float *w, int64_t rows, int dim,
                     float eps, lai_stream_t stream) {
    return lai::run<uint16_t, false>(y, const_cast<uint16_t *>(x), nullptr, w, rows, dim, eps,
                                     stream);
}
int lai_rmsnorm_f32(float *y, const float *x, const float *w, int64_t rows, int dim, float eps,
                    lai_stream_t stream) {
    return lai::run<float, false>(y, const_cast<float *>(x), nullptr, w, rows, dim, eps, stream);
}
int lai_add_rmsnorm_bf16(lai_bf16 *x, const lai_bf16 *delta, const float *w, lai_bf16 *y,
                         int64_t rows, int dim, float eps, lai_stream_t stream) {
    return lai::run<uint16_t, true>(y, x, delta, w, rows, dim, eps, stream);
}
int lai_add_rmsnorm_f32(float *x, const float *delta, const float *w, float *y, int64_t rows,
                        int dim, float eps, lai_stream_t stream) {
    return lai::run<float, true>(y, x, delta, w, rows, dim, eps, stream);
}

}  // extern "C"

// gemv.cu - decode-time linear layers with the layer's elementwise ops fused in.
//
// Reference: linear_bf16(ctx, out, in, W, M, K, N) = in[M,K] @ W[N,K]^T with BF16
// weights and FP32 activations (src/tts_native.c:66-79), called at decode with M = 1
// (talker_forward, src/tts_native.c:637-667) between the per-layer elementwise ops:
//   qwen_rms_norm -> q/k/v projections            (:637-642)   -> lai_gemv_bf16w_f32 (norm prologue)
//   o_proj -> qwen_add_inplace                    (:658-659)   -> lai_gemv_residual_bf16w_f32
//   qwen_rms_norm -> gate_up -> qwen_swiglu_multiply (:661-665) -> lai_gemv_swiglu_bf16w_f32
//   down_proj -> qwen_add_inplace                 (:666-668)   -> lai_gemv_residual_bf16w_f32
// so the normalised, activated and projected vectors never make an HBM round trip.
//
// Roofline: HBM on the weights. Algorithmic bytes per launch: N*K*2 (weights, read
// once) + M*(K + N)*4 (activations; the residual epilogue reads and writes its
// output). At M <= 8 the FLOPs (2*M*N*K) are far below what the weights' bytes cost
// at HBM speed, so CUDA cores are the right unit; a batched (large-M) projection
// would be a tensor-core GEMM, which this file does not attempt.
//
// Launch: programmatic dependent launch. A GEMV issues its first weight loads before
// it waits (griddepcontrol.wait) for the previous kernel's results, and lets the next
// kernel start launching once its own weight stream has been read, so one layer's
// weight stream overlaps the previous kernel's tail.
//
// Weight formats (the reference's GPU decode modes, src/tts_pipeline.h:37-40 and
// src/tts_native.c:1185-1240): BF16 as stored in the safetensors (linear_bf16), FP16
// (its fp16 mode; also the codec head in int8 mode), INT8 with one F32 scale per row
// (its int8 mode: scale = max|row| / 127, q = round(w / scale), the scale applied after
// the row's reduction, tools/asr_benchmarks.md:342-352) and F32. One kernel template
// serves them all; a format only changes how a 16-byte weight vector becomes floats
// (8 BF16 or FP16, 16 INT8, 4 F32 elements), and INT8 multiplies each row's total by
// its scale. The conversions avoid the narrow XU pipe: BF16 is a shift, INT8 a byte
// permute into a float's mantissa and one subtraction.
//
// Layout: each CTA first stages the M input rows in shared memory (normalising
// them when a norm weight is given: every CTA recomputes the norm of the <= 8 short
// rows, cheaper than a separate launch and its HBM round trip). Each warp then owns
// RPW output rows (2 for SwiGLU: the interleaved gate row 2j and up row 2j+1,
// src/tts_native.c:149-161) and streams them in 16-byte vectors, 8 per lane in
// flight, against the staged inputs; a warp-shuffle tree reduces each dot product.
#include "lai_common.cuh"

#include <cuda_fp16.h>
#include <math.h>

namespace lai {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxM = 8;
constexpr int kUnrollK = 8;  // 16-byte weight vectors in flight per lane per row (K <= 2048: one trip)
// M = 1 rows longer than one trip of kUnrollK vectors (BF16 K > 2048, e.g. the down
// projection's K = 3072): 16 in flight, so the whole row (or two trips for K = 6144) is
// requested before the kernel waits for its predecessor instead of a second trip's loads
// waiting behind that dependency: talker step (g1) 483 -> 451 us, 1.7B step (g2) 966 ->
// 921 us. With 16 for every shape the K = 1024 projections were slower and K = 2048 mixed.
constexpr int kUnrollDeep = 16;
// M = 1 rows of at most 4 vectors per lane (BF16 K <= 1024) hold only those: half the weight
// registers of the 8-vector form, so more CTAs stay resident and the next GEMV's CTAs (and
// their weight loads) fit beside this one's (the 0.6B talker's gate|up GEMV needed two waves
// of CTAs at 96 registers)
constexpr int kUnrollShort = 4;
// ... and for those rows a warp takes several consecutive row groups (16 weight vectors per
// lane for plain rows: 4 rows; SwiGLU: 2 gate/up pairs), fewer CTAs each staging (and
// normalising) the input row once for more rows: the talker's q|k|v GEMV 4.26 -> 3.80 us,
// gate|up 4.68 -> 4.61 us (4 pairs per warp: 5.30 us).
constexpr int kShortGroups = 4, kShortPairs = 2;
// Plain M = 1 rows of 5-8 vectors per lane (BF16 K = 2048): 2 rows per warp, 16 vectors in all
// (1.7B step: q|k|v 7.17 -> 5.69 us, o 4.10 -> 3.58 us; talker o 3.07 -> 2.84 us).
constexpr int kMidGroups = 2;
constexpr size_t kMaxSmem = 200 * 1024;

enum Epi { kStore = 0, kResidual = 1, kSwiglu = 2 };

// ---- weight formats: storage type, elements per 16-byte vector, conversions ----------
struct WBf16 {
    using T = uint16_t;
    static constexpr int kEpv = 8;
    static constexpr bool kScaled = false;
    static __device__ __forceinline__ void unpack(const uint4 &v, float (&f)[kEpv]) {
        lai::unpack<uint16_t>(v, f);
    }
    static __device__ __forceinline__ float to_f(T w) { return lai::to_f(w); }
};
struct WF16 {
    using T = uint16_t;  // IEEE binary16 bit patterns
    static constexpr int kEpv = 8;
    static constexpr bool kScaled = false;
    static __device__ __forceinline__ float2 pair(uint32_t u) {
        return __half22float2(*reinterpret_cast<const __half2 *>(&u));
    }
    static __device__ __forceinline__ void unpack(const uint4 &v, float (&f)[kEpv]) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 p = pair(w[i]);
            f[2 * i] = p.x;
            f[2 * i + 1] = p.y;
        }
    }
    static __device__ __forceinline__ float to_f(T w) { return __half2float(__ushort_as_half(w)); }
};
struct WI8 {
    using T = int8_t;
    static constexpr int kEpv = 16;
    static constexpr bool kScaled = true;
    // A signed byte b becomes b + 128 when its top bit flips; placed as the low mantissa
    // byte of 2^23 (exponent byte 0x4B) it reads as the float 2^23 + b + 128, and one
    // exact subtraction leaves b.
    static __device__ __forceinline__ void four(uint32_t u, float *f) {
        const uint32_t b = u ^ 0x80808080u;
#pragma unroll
        for (int i = 0; i < 4; i++)
            f[i] = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7440u + i)) - 8388736.0f;
    }
    static __device__ __forceinline__ void unpack(const uint4 &v, float (&f)[kEpv]) {
        four(v.x, f);
        four(v.y, f + 4);
        four(v.z, f + 8);
        four(v.w, f + 12);
    }
    static __device__ __forceinline__ float to_f(T w) { return (float)w; }
};
struct WF32 {
    using T = float;
    static constexpr int kEpv = 4;
    static constexpr bool kScaled = false;
    static __device__ __forceinline__ void unpack(const uint4 &v, float (&f)[kEpv]) {
        lai::unpack<float>(v, f);
    }
    static __device__ __forceinline__ float to_f(T w) { return w; }
};


// Stage x[M,K] in shared memory as FP32, normalised by RMSNorm when norm_w != NULL.
template <int M>
__device__ __forceinline__ void stage_inputs(float *xs, const float *x, const float *norm_w,
                                             float eps, int K) {
    __shared__ float red[M][kWarps];
    float ss[M];
#pragma unroll
    for (int m = 0; m < M; m++) ss[m] = 0.f;
    for (int i = threadIdx.x; i < K; i += kThreads) {
#pragma unroll
        for (int m = 0; m < M; m++) {
            const float v = x[(size_t)m * K + i];
            xs[m * K + i] = v;
            ss[m] = fmaf(v, v, ss[m]);
        }
    }
    if (norm_w) {
        const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
        for (int m = 0; m < M; m++) {
            const float t = group_sum<32>(ss[m]);
            if (lane == 0) red[m][wid] = t;
        }
        __syncthreads();
        float inv[M];
#pragma unroll
        for (int m = 0; m < M; m++) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < kWarps; w++) t += red[m][w];
            inv[m] = 1.0f / sqrtf(t / (float)K + eps);
        }
        for (int i = threadIdx.x; i < K; i += kThreads) {
            const float wi = norm_w[i];
#pragma unroll
            for (int m = 0; m < M; m++) xs[m * K + i] = __fmul_rn(__fmul_rn(xs[m * K + i], inv[m]), wi);
        }
    }
    __syncthreads();
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

// K % (elements per vector) == 0 and W 16-byte aligned: 16-byte weight vectors.
template <typename WF, int M, int EPI, int U, int R>  // R: row groups (1 row, 2 for SwiGLU) per warp
__global__ void __launch_bounds__(kThreads)
gemv_vec_kernel(float *y, const float *x, const float *norm_w, float eps,
                const typename WF::T *__restrict__ W, const float *__restrict__ scales, int K,
                int N, int ldy) {
    using T = typename WF::T;
    constexpr int RW = (EPI == kSwiglu ? 2 : 1) * R;  // consecutive weight rows per warp
    constexpr int E = WF::kEpv;   // weight elements per 16-byte vector
    constexpr int S = 32 * E;     // elements one warp covers per vector step
    extern __shared__ __align__(16) float xs[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = (blockIdx.x * kWarps + warp) * RW;
    const bool active = row0 < N;
    const T *wr[RW];
    bool rv[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) {
        rv[r] = row0 + r < N;
        wr[r] = W + (size_t)(rv[r] ? row0 + r : 0) * K;
    }
    // the weights depend on nothing earlier on the stream: their first chunk is in
    // flight before this kernel waits for the previous one and stages its inputs
    uint4 wv[U][RW];
#pragma unroll
    for (int u = 0; u < U; u++) {
        const int k0 = u * S + lane * E;
#pragma unroll
        for (int r = 0; r < RW; r++)
            if (rv[r] && k0 < K) wv[u][r] = ld_stream(wr[r] + k0);
    }
    // the row scales are weights too (no dependency): in flight with them
    float sc[RW];
#pragma unroll
    for (int r = 0; r < RW; r++) sc[r] = WF::kScaled && rv[r] ? __ldg(scales + row0 + r) : 1.0f;
    pdl_wait_prior();
    // the residual this lane adds into (written by the previous kernel): read now, so the
    // epilogue does not wait on a load after the reduction
    float res[RW];
#pragma unroll
    for (int r = 0; r < RW; r++)
        res[r] = EPI == kResidual && rv[r] && lane < M ? y[(size_t)lane * ldy + row0 + r] : 0.0f;
    stage_inputs<M>(xs, x, norm_w, eps, K);
    if (!active) {
        pdl_launch_dependents();
        return;
    }
    float acc[RW][M];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
        for (int m = 0; m < M; m++) acc[r][m] = 0.f;

    for (int kb = 0; kb < K; kb += S * U) {
        if (kb > 0) {
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int k0 = kb + u * S + lane * E;
#pragma unroll
                for (int r = 0; r < RW; r++)
                    if (rv[r] && k0 < K) wv[u][r] = ld_stream(wr[r] + k0);
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int k0 = kb + u * S + lane * E;
            if (k0 >= K) break;
            float wf[RW][E];
#pragma unroll
            for (int r = 0; r < RW; r++) WF::unpack(wv[u][r], wf[r]);
#pragma unroll
            for (int m = 0; m < M; m++) {
#pragma unroll
                for (int q = 0; q < E / 4; q++) {
                    const float4 a = *reinterpret_cast<const float4 *>(xs + m * K + k0 + 4 * q);
                    const float xv[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int r = 0; r < RW; r++)
#pragma unroll
                        for (int e = 0; e < 4; e++)
                            acc[r][m] = fmaf(wf[r][4 * q + e], xv[e], acc[r][m]);
                }
            }
        }
    }
    // this warp's weights are read: the next kernel may start launching (its CTAs
    // stream their own weights, then wait for this grid before reading activations)
    pdl_launch_dependents();
#pragma unroll
    for (int r = 0; r < RW; r++) {
#pragma unroll
        for (int m = 0; m < M; m++) {
            acc[r][m] = group_sum<32>(acc[r][m]);
            if (WF::kScaled) acc[r][m] *= sc[r];
        }
    }
    // lane m writes input m's results (all lanes hold every total after the tree)
#pragma unroll
    for (int m = 0; m < M; m++) {
        if (lane != m) continue;
        if constexpr (EPI == kSwiglu) {
#pragma unroll
            for (int r = 0; r < RW; r += 2)
                if (rv[r]) y[(size_t)m * ldy + (row0 + r) / 2] = silu_mul(acc[r][m], acc[r + 1][m]);
        } else {
#pragma unroll
            for (int r = 0; r < RW; r++) {
                if (!rv[r]) continue;
                if constexpr (EPI == kStore) y[(size_t)m * ldy + row0 + r] = acc[r][m];
                if constexpr (EPI == kResidual) y[(size_t)m * ldy + row0 + r] = res[r] + acc[r][m];
            }
        }
    }
}

// Any K / alignment: scalar weight reads, same structure.
template <typename WF, int M, int EPI>
__global__ void __launch_bounds__(kThreads)
gemv_scalar_kernel(float *y, const float *x, const float *norm_w, float eps,
                   const typename WF::T *W, const float *scales, int K, int N, int ldy) {
    constexpr int RPW = EPI == kSwiglu ? 2 : 1;
    extern __shared__ __align__(16) float xs[];
    pdl_launch_dependents();
    pdl_wait_prior();
    stage_inputs<M>(xs, x, norm_w, eps, K);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row0 = (blockIdx.x * kWarps + warp) * RPW;
    if (row0 >= N) return;
    float acc[RPW][M] = {};
    for (int k = lane; k < K; k += 32)
#pragma unroll
        for (int r = 0; r < RPW; r++) {
            const float wf = WF::to_f(W[(size_t)(row0 + r) * K + k]);
#pragma unroll
            for (int m = 0; m < M; m++) acc[r][m] = fmaf(wf, xs[m * K + k], acc[r][m]);
        }
#pragma unroll
    for (int r = 0; r < RPW; r++) {
        const float sc = WF::kScaled ? scales[row0 + r] : 1.0f;
#pragma unroll
        for (int m = 0; m < M; m++) {
            acc[r][m] = group_sum<32>(acc[r][m]);
            if (WF::kScaled) acc[r][m] *= sc;
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        if (lane != m) continue;
        if constexpr (EPI == kStore) y[(size_t)m * ldy + row0] = acc[0][m];
        if constexpr (EPI == kResidual) y[(size_t)m * ldy + row0] += acc[0][m];
        if constexpr (EPI == kSwiglu) y[(size_t)m * ldy + row0 / 2] = silu_mul(acc[0][m], acc[1][m]);
    }
}

template <typename WF, int M, int EPI>
int launch(float *y, const float *x, const float *norm_w, float eps, const typename WF::T *W,
           const float *scales, int K, int N, int ldy, bool vec, cudaStream_t s) {
    constexpr int RPW = EPI == kSwiglu ? 2 : 1;
    const size_t smem = (size_t)M * K * sizeof(float);
    const bool deep = M == 1 && K > kUnrollK * 32 * WF::kEpv;
    const bool shallow = M == 1 && K <= kUnrollShort * 32 * WF::kEpv;
    constexpr int RS = M != 1 ? 1 : EPI == kSwiglu ? kShortPairs : kShortGroups;
    constexpr int RM = M != 1 || EPI == kSwiglu ? 1 : kMidGroups;
    auto kern = !vec ? gemv_scalar_kernel<WF, M, EPI>
                : deep ? gemv_vec_kernel<WF, M, EPI, (M == 1 ? kUnrollDeep : kUnrollK), 1>
                : shallow ? gemv_vec_kernel<WF, M, EPI, (M == 1 ? kUnrollShort : kUnrollK), RS>
                          : gemv_vec_kernel<WF, M, EPI, kUnrollK, RM>;
    const int rows_per_cta = kWarps * RPW * (!vec || deep ? 1 : shallow ? RS : RM);
    // opt in above 47 KiB: the default 48 KiB limit also covers the kernel's small static array
    if (smem > 47 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
        cudaGetLastError();
        return LAI_ERR_CUDA;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid_for(N, rows_per_cta));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see pdl_wait_prior
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, y, x, norm_w, eps, W, scales, K, N, ldy) != cudaSuccess) {
        cudaGetLastError();
        return LAI_ERR_CUDA;
    }
    return launch_status();
}

template <typename WF, int EPI>
int run(float *y, const float *x, const float *norm_w, float eps, const typename WF::T *W,
        const float *scales, int64_t M, int K, int N, lai_stream_t stream) {
    if (!y || !x || !W || M < 0 || K <= 0 || N <= 0 || (EPI == kSwiglu && (N & 1)) ||
        (WF::kScaled && !scales))
        return LAI_ERR_INVALID;
    if (M == 0) return LAI_OK;
    const int ny = EPI == kSwiglu ? N / 2 : N;  // output row length
    if (overlaps(y, (size_t)M * ny * 4, x, (size_t)M * K * 4)) return LAI_ERR_ALIAS;
    // inputs per pass: as many rows (<= 8) as fit in shared memory
    int64_t per = kMaxM;
    while (per > 1 && (size_t)per * K * 4 > kMaxSmem) per /= 2;
    if ((size_t)K * 4 > kMaxSmem) return LAI_ERR_TOOBIG;
    const bool vec = K % WF::kEpv == 0 && aligned16(W);
    cudaStream_t s = as_stream(stream);
    for (int64_t m0 = 0; m0 < M;) {
        const int64_t cap = M - m0 < per ? M - m0 : per;
        const int take = cap >= 8 ? 8 : cap >= 4 ? 4 : cap >= 2 ? 2 : 1;  // rows this pass
        float *yp = y + m0 * ny;
        const float *xp = x + m0 * K;
        int st;
        switch (take) {
            case 8: st = launch<WF, 8, EPI>(yp, xp, norm_w, eps, W, scales, K, N, ny, vec, s); break;
            case 4: st = launch<WF, 4, EPI>(yp, xp, norm_w, eps, W, scales, K, N, ny, vec, s); break;
            case 2: st = launch<WF, 2, EPI>(yp, xp, norm_w, eps, W, scales, K, N, ny, vec, s); break;
            default: st = launch<WF, 1, EPI>(yp, xp, norm_w, eps, W, scales, K, N, ny, vec, s); break;
        }
        if (st != LAI_OK) return st;
        m0 += take;
    }
    return LAI_OK;
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_gemv_bf16w_f32(float *y, const float *x, const float *norm_w, float eps, const lai_bf16 *W,
                       int64_t M, int K, int N, lai_stream_t stream) {
    return lai::run<lai::WBf16, lai::kStore>(y, x, norm_w, eps, W, nullptr, M, K, N, stream);
}

int lai_gemv_residual_bf16w_f32(float *x_res, const float *a, const lai_bf16 *W, int64_t M, int K,
                                int N, lai_stream_t stream) {
    return lai::run<lai::WBf16, lai::kResidual>(x_res, a, nullptr, 0.f, W, nullptr, M, K, N, stream);
}

int lai_gemv_swiglu_bf16w_f32(float *out, const float *x, const float *norm_w, float eps,
                              const lai_bf16 *W_gu, int64_t M, int K, int inter,
                              lai_stream_t stream) {
    if (inter <= 0 || inter > (1 << 29)) return LAI_ERR_INVALID;
    return lai::run<lai::WBf16, lai::kSwiglu>(out, x, norm_w, eps, W_gu, nullptr, M, K, 2 * inter,
                                              stream);
}

int lai_gemv_f16w_f32(float *y, const float *x, const float *norm_w, float eps, const lai_f16 *W,
                      int64_t M, int K, int N, lai_stream_t stream) {
    return lai::run<lai::WF16, lai::kStore>(y, x, norm_w, eps, W, nullptr, M, K, N, stream);
}

int lai_gemv_residual_f16w_f32(float *x_res, const float *a, const lai_f16 *W, int64_t M, int K,
                               int N, lai_stream_t stream) {
    return lai::run<lai::WF16, lai::kResidual>(x_res, a, nullptr, 0.f, W, nullptr, M, K, N, stream);
}

int lai_gemv_swiglu_f16w_f32(float *out, const float *x, const float *norm_w, float eps,
                             const lai_f16 *W_gu, int64_t M, int K, int inter,
                             lai_stream_t stream) {
    if (inter <= 0 || inter > (1 << 29)) return LAI_ERR_INVALID;
    return lai::run<lai::WF16, lai::kSwiglu>(out, x, norm_w, eps, W_gu, nullptr, M, K, 2 * inter,
                                             stream);
}

int lai_gemv_i8w_f32(float *y, const float *x, const float *norm_w, float eps, const int8_t *W,
                     const float *scales, int64_t M, int K, int N, lai_stream_t stream) {
    return lai::run<lai::WI8, lai::kStore>(y, x, norm_w, eps, W, scales, M, K, N, stream);
}

int lai_gemv_residual_i8w_f32(float *x_res, const float *a, const int8_t *W, const float *scales,
                              int64_t M, int K, int N, lai_stream_t stream) {
    return lai::run<lai::WI8, lai::kResidual>(x_res, a, nullptr, 0.f, W, scales, M, K, N, stream);
}

int lai_gemv_swiglu_i8w_f32(float *out, const float *x, const float *norm_w, float eps,
                            const int8_t *W_gu, const float *scales, int64_t M, int K, int inter,
                            lai_stream_t stream) {
    if (inter <= 0 || inter > (1 << 29)) return LAI_ERR_INVALID;
    return lai::run<lai::WI8, lai::kSwiglu>(out, x, norm_w, eps, W_gu, scales, M, K, 2 * inter,
                                            stream);
}

int lai_gemv_f32w_f32(float *y, const float *x, const float *norm_w, float eps, const float *W,
                      int64_t M, int K, int N, lai_stream_t stream) {
    return lai::run<lai::WF32, lai::kStore>(y, x, norm_w, eps, W, nullptr, M, K, N, stream);
}

int lai_gemv_residual_f32w_f32(float *x_res, const float *a, const float *W, int64_t M, int K,
                               int N, lai_stream_t stream) {
    return lai::run<lai::WF32, lai::kResidual>(x_res, a, nullptr, 0.f, W, nullptr, M, K, N, stream);
}

int lai_gemv_swiglu_f32w_f32(float *out, const float *x, const float *norm_w, float eps,
                             const float *W_gu, int64_t M, int K, int inter,
                             lai_stream_t stream) {
    if (inter <= 0 || inter > (1 << 29)) return LAI_ERR_INVALID;
    return lai::run<lai::WF32, lai::kSwiglu>(out, x, norm_w, eps, W_gu, nullptr, M, K, 2 * inter,
                                             stream);
}

}  // extern "C"

// voc_decoder.cu - the vocoder decoder's remaining convolutions, channels-last F32:
//   lai_voc_conv1d_f32           causal conv1d (the BigVGAN init conv 1024 -> 1536, k=7,
//                                src/tts_vocoder.c:694-697) on the tensor-core GEMM
//   lai_voc_conv_transpose1d_f32 transposed conv with kernel = stride (the ConvNeXt upsample
//                                stages, :658-667) or kernel = 2 stride (BigVGAN blocks)
//   lai_voc_final_f32            SnakeBeta -> conv1d C -> 1 (k=7) -> clamp(-1, 1), the decoder's
//                                last step (:748-758), fused into one HBM pass
// The GEMM forms (voc_conv.cuh) read their input in the 3xTF32 hi/lo split, made here by a
// plain split kernel; the transposed conv runs `stride` interleaved convs of kernel / stride
// taps, output row (t - trim) * stride + f for phase f (trim 1 for kernel 2 stride, else 0).
#include "voc_conv.cuh"

namespace lai {
namespace {

// hi = tf32(x), lo = x - hi over n elements (n % 4 == 0)
template <int PASSES>
__global__ void __launch_bounds__(256)
split_kernel(const float *__restrict__ x, float *hi, float *lo, int64_t n4) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        const float4 h = make_float4(umma::tf32_round(v.x), umma::tf32_round(v.y),
                                     umma::tf32_round(v.z), umma::tf32_round(v.w));
        reinterpret_cast<float4 *>(hi)[i] = h;
        if (PASSES == 3)
            reinterpret_cast<float4 *>(lo)[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z,
                                                            v.w - h.w);
    }
}

int launch_split(const float *x, float *hi, float *lo, size_t n, int passes, cudaStream_t st) {
    const int64_t n4 = (int64_t)n / 4;
    const unsigned g = grid_for(n4, 256) < 148u * 16 ? grid_for(n4, 256) : 148u * 16;
    if (passes == 3)
        split_kernel<3><<<g, 256, 0, st>>>(x, hi, lo, n4);
    else
        split_kernel<1><<<g, 256, 0, st>>>(x, hi, lo, n4);
    return launch_status();
}

// Final step: one CTA writes kFinalRows consecutive samples of one item. It stages input rows
// [t0 - 6, t0 + kFinalRows) of x [T, C] through SnakeBeta into shared memory (zero before
// t = 0; rows padded to C + 1 floats so the per-thread row reads hit distinct banks), loading
// float4 vectors eight per thread at a time so enough bytes are in flight to cover HBM
// latency, then each thread sums its sample's 7 x C window and clamps.
constexpr int kFinalRows = 256;
constexpr int kFinalBatch = 8;  // float4 loads in flight per thread while staging

template <int C>
__global__ void __launch_bounds__(kFinalRows)
final_kernel(float *audio, const float *__restrict__ x, const float *__restrict__ ea,
             const float *__restrict__ ieb, const float *__restrict__ w,
             const float *__restrict__ bias, int T) {
    constexpr int pitch = C + 1;
    constexpr int V = C / 4;                       // float4 vectors per row
    constexpr int NV = (kFinalRows + 6) * V;
    extern __shared__ float sm[];
    float *s = sm;                                 // [kFinalRows + 6][C + 1]
    float *wt = s + (kFinalRows + 6) * pitch;      // [7][C]: tap-major weights
    float *sa = wt + 7 * C, *sb = sa + C;          // snake parameters
    const int b = blockIdx.y, t0 = blockIdx.x * kFinalRows;
    const float *xb = x + (size_t)b * T * C;
    for (int i = threadIdx.x; i < 7 * C; i += kFinalRows) {
        const int c = i / 7, k = i - c * 7;
        wt[k * C + c] = w[i];  // w [1, C, 7] as loaded
    }
    for (int i = threadIdx.x; i < C; i += kFinalRows) {
        sa[i] = ea[i];
        sb[i] = ieb[i];
    }
    __syncthreads();
    for (int base = threadIdx.x; base < NV; base += kFinalRows * kFinalBatch) {
        float4 v[kFinalBatch];
#pragma unroll
        for (int u = 0; u < kFinalBatch; u++) {
            const int i = base + u * kFinalRows;
            const int r = i / V, c4 = i - r * V, t = t0 - 6 + r;
            v[u] = (i < NV && t >= 0 && t < T)
                       ? *reinterpret_cast<const float4 *>(xb + (size_t)t * C + 4 * c4)
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < kFinalBatch; u++) {
            const int i = base + u * kFinalRows;
            if (i < NV) {
                const int r = i / V, c = 4 * (i - r * V), t = t0 - 6 + r;
                const bool in = t >= 0 && t < T;
                float *dst = s + r * pitch + c;
                // two channels per instruction (snake2: same bits as snake1)
                const float2 p0 = snake2(make_float2(v[u].x, v[u].y), make_float2(sa[c], sa[c + 1]),
                                         make_float2(sb[c], sb[c + 1]));
                const float2 p1 = snake2(make_float2(v[u].z, v[u].w),
                                         make_float2(sa[c + 2], sa[c + 3]),
                                         make_float2(sb[c + 2], sb[c + 3]));
                dst[0] = in ? p0.x : 0.f;
                dst[1] = in ? p0.y : 0.f;
                dst[2] = in ? p1.x : 0.f;
                dst[3] = in ? p1.y : 0.f;
            }
        }
    }
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t >= T) return;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < 7; k++) {
        const float *row = s + (threadIdx.x + k) * pitch;
        const float *wk = wt + k * C;
#pragma unroll 8
        for (int c = 0; c < C; c++) acc = fmaf(wk[c], row[c], acc);
    }
    acc += __ldg(bias);
    audio[(size_t)b * T + t] = fminf(fmaxf(acc, -1.0f), 1.0f);
}

template <int C>
int launch_final(float *audio, const float *x, const float *ea, const float *ieb, const float *w,
                 const float *bias, int batch, int T, cudaStream_t st) {
    const size_t smem = ((size_t)(kFinalRows + 6) * (C + 1) + 9 * C) * sizeof(float);
    auto kern = final_kernel<C>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return LAI_ERR_CUDA;
    const dim3 grid((unsigned)((T + kFinalRows - 1) / kFinalRows), (unsigned)batch);
    kern<<<grid, kFinalRows, smem, st>>>(audio, x, ea, ieb, w, bias, T);
    return launch_status();
}

// RVQ decode's gather: row t of out is the 16 codebook rows codes[t, 0..n_cb) laid side by
// side, [T, n_cb * dim]; one GEMM against the packed projections then sums the codebooks.
__global__ void rvq_gather_kernel(float4 *__restrict__ out, const float4 *__restrict__ books,
                                  const int64_t *__restrict__ codes, int64_t T, int n_cb,
                                  int cb_size, int dim4, int *err) {
    const int64_t n = T * n_cb * dim4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tc = i / dim4;  // (t, cb)
        const int d = (int)(i - tc * dim4);
        const int cb = (int)(tc % n_cb);
        const int64_t code = codes[tc];
        if (code < 0 || code >= cb_size) {
            out[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (d == 0 && err) atomicOr(err, LAI_DEVERR_TOKEN_ID);
            continue;
        }
        out[i] = books[((int64_t)cb * cb_size + code) * dim4 + d];
    }
}

}  // namespace
}  // namespace lai

extern "C" int lai_voc_rvq_gather_f32(float *out, const float *codebooks, const int64_t *codes,
                                      int T, int n_codebooks, int codebook_size, int dim,
                                      int *err, lai_stream_t stream) {
    using namespace lai;
    if (!out || !codebooks || !codes || T < 0 || n_codebooks <= 0 || codebook_size <= 0 ||
        dim <= 0 || dim % 4 != 0 || !aligned16(out) || !aligned16(codebooks))
        return LAI_ERR_INVALID;
    if (T == 0) return LAI_OK;
    const size_t ob = (size_t)T * n_codebooks * dim * 4;
    if (overlaps(out, ob, codebooks, (size_t)n_codebooks * codebook_size * dim * 4))
        return LAI_ERR_ALIAS;
    const int64_t n = (int64_t)T * n_codebooks * (dim / 4);
    rvq_gather_kernel<<<grid_for(n, 256), 256, 0, as_stream(stream)>>>(
        reinterpret_cast<float4 *>(out), reinterpret_cast<const float4 *>(codebooks), codes, T,
        n_codebooks, codebook_size, dim / 4, err);
    return launch_status();
}

// x_res[rows, c_out] += gamma * (in[rows, c_in] . W^T + bias): the pre-transformer's o / down
// projection with its LayerScale and residual (src/tts_vocoder_xfmr.c:182-186, 203-207), on
// the same tcgen05 kernel as the convolutions (k = 1), F32 through the 3xTF32 split.
extern "C" int lai_voc_linear_scale_residual_f32(float *x_res, const float *in, float *scratch,
                                                 const float *w, const float *bias,
                                                 const float *gamma, int rows, int c_in,
                                                 int c_out, int passes, int *err,
                                                 lai_stream_t stream) {
    using namespace lai;
    if (!x_res || !in || !scratch || !w || !bias || !gamma || rows < 0 ||
        (passes != 1 && passes != 3))
        return LAI_ERR_INVALID;
    if (rows == 0) return LAI_OK;
    if (c_in % 32 != 0 || c_out % 32 != 0 || !aligned16(x_res) || !aligned16(in) ||
        !aligned16(scratch) || !aligned16(w))
        return LAI_ERR_INVALID;
    const size_t in_plane = (size_t)rows * c_in, out_plane = (size_t)rows * c_out;
    if (overlaps(x_res, out_plane * 4, in, in_plane * 4) ||
        overlaps(x_res, out_plane * 4, scratch, 2 * in_plane * 4) ||
        overlaps(in, in_plane * 4, scratch, 2 * in_plane * 4))
        return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    const cudaStream_t st = as_stream(stream);
    int rc = launch_split(in, scratch, scratch + in_plane, in_plane, passes, st);
    if (rc != LAI_OK) return rc;
    CUtensorMap am, wm;
    if (!act_map(&am, scratch, 1, rows, c_in) ||
        !weight_map(&wm, w, 1, c_out, c_in, pick_bn(c_out)))
        return LAI_ERR_INVALID;
    const ConvArgs a{nullptr, nullptr, x_res, bias, nullptr, nullptr, gamma,
                     rows, c_in, c_out, 1, 1, err, 1, rows, 0};
    return launch_conv<kEpiScaleResidual>(passes, am, wm, a, 1, st);
}

extern "C" int lai_voc_conv1d_f32(float *out, const float *x, float *scratch, const float *w,
                                  const float *bias, int batch, int c_in, int c_out, int T,
                                  int kernel, int dilation, int passes, int *err,
                                  lai_stream_t stream) {
    using namespace lai;
    if (!out || !x || !scratch || !w || !bias || batch < 0 || T < 0 || kernel <= 0 ||
        dilation <= 0 || (passes != 1 && passes != 3))
        return LAI_ERR_INVALID;
    if (batch == 0 || T == 0) return LAI_OK;
    if (c_in % 32 != 0 || c_out % 32 != 0 || !aligned16(out) || !aligned16(x) ||
        !aligned16(scratch) || !aligned16(w) || (int64_t)(kernel - 1) * dilation > (1 << 30))
        return LAI_ERR_INVALID;
    if (batch > 65535) return LAI_ERR_RANGE;
    const size_t in_plane = (size_t)batch * T * c_in, out_plane = (size_t)batch * T * c_out;
    if (overlaps(out, out_plane * 4, x, in_plane * 4) ||
        overlaps(out, out_plane * 4, scratch, 2 * in_plane * 4) ||
        overlaps(x, in_plane * 4, scratch, 2 * in_plane * 4))
        return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    const cudaStream_t st = as_stream(stream);
    int rc = launch_split(x, scratch, scratch + in_plane, in_plane, passes, st);
    if (rc != LAI_OK) return rc;
    CUtensorMap am, wm;
    if (!act_map(&am, scratch, batch, T, c_in) ||
        !weight_map(&wm, w, kernel, c_out, c_in, pick_bn(c_out)))
        return LAI_ERR_INVALID;
    const ConvArgs a{nullptr, nullptr, out, bias, nullptr, nullptr, nullptr,
                     T, c_in, c_out, kernel, dilation, err, 1, T, 0};
    return launch_conv<kEpiStoreSnake>(passes, am, wm, a, batch, st);
}

extern "C" int lai_voc_conv_transpose1d_f32(float *out, const float *x, float *scratch,
                                            const float *w, const float *bias, int batch,
                                            int c_in, int c_out, int T, int kernel, int stride,
                                            int passes, int *err, lai_stream_t stream) {
    using namespace lai;
    if (!out || !x || !scratch || !w || !bias || batch < 0 || T < 0 || stride <= 0 ||
        (kernel != stride && kernel != 2 * stride) || (passes != 1 && passes != 3))
        return LAI_ERR_INVALID;
    if (batch == 0 || T == 0) return LAI_OK;
    const int taps = kernel / stride, trim = taps - 1;
    const int T_out = (T + 1) * stride - kernel;
    if (T_out <= 0) return LAI_ERR_INVALID;
    if (c_in % 32 != 0 || c_out % 32 != 0 || !aligned16(out) || !aligned16(x) ||
        !aligned16(scratch) || !aligned16(w))
        return LAI_ERR_INVALID;
    if ((int64_t)batch * stride > 65535) return LAI_ERR_RANGE;
    const size_t in_plane = (size_t)batch * T * c_in, out_plane = (size_t)batch * T_out * c_out;
    if (overlaps(out, out_plane * 4, x, in_plane * 4) ||
        overlaps(out, out_plane * 4, scratch, 2 * in_plane * 4) ||
        overlaps(x, in_plane * 4, scratch, 2 * in_plane * 4))
        return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    const cudaStream_t st = as_stream(stream);
    int rc = launch_split(x, scratch, scratch + in_plane, in_plane, passes, st);
    if (rc != LAI_OK) return rc;
    CUtensorMap am, wm;
    if (!act_map(&am, scratch, batch, T, c_in) ||
        !weight_map(&wm, w, kernel, c_out, c_in, pick_bn(c_out)))
        return LAI_ERR_INVALID;
    const ConvArgs a{nullptr, nullptr, out, bias, nullptr, nullptr, nullptr,
                     T, c_in, c_out, taps, 1, err, stride, T_out, trim};
    return launch_conv<kEpiStoreSnake>(passes, am, wm, a, batch, st);
}

extern "C" int lai_voc_final_f32(float *audio, const float *x, const float *exp_alpha,
                                 const float *inv_exp_beta, const float *w, const float *bias,
                                 int batch, int channels, int T, lai_stream_t stream) {
    using namespace lai;
    if (!audio || !x || !exp_alpha || !inv_exp_beta || !w || !bias || batch < 0 || T < 0 ||
        channels <= 0)
        return LAI_ERR_INVALID;
    if (batch == 0 || T == 0) return LAI_OK;
    if (batch > 65535) return LAI_ERR_RANGE;
    if (overlaps(audio, (size_t)batch * T * 4, x, (size_t)batch * T * channels * 4))
        return LAI_ERR_ALIAS;
    if (!aligned16(x)) return LAI_ERR_INVALID;
    const cudaStream_t st = as_stream(stream);
    switch (channels) {
        case 32: return launch_final<32>(audio, x, exp_alpha, inv_exp_beta, w, bias, batch, T, st);
        case 64: return launch_final<64>(audio, x, exp_alpha, inv_exp_beta, w, bias, batch, T, st);
        case 96: return launch_final<96>(audio, x, exp_alpha, inv_exp_beta, w, bias, batch, T, st);
        case 128: return launch_final<128>(audio, x, exp_alpha, inv_exp_beta, w, bias, batch, T, st);
        default: return LAI_ERR_INVALID;
    }
}

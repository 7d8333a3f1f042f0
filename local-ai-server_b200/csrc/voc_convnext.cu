// voc_convnext.cu - the vocoder's ConvNeXt block, FP32, channels-last, pointwise convs on
// tcgen05 tensor cores.
//
// Reference: run_convnext (src/tts_vocoder.c:463-533) on x [C, T], C = 1024 in both
// upsample stages (:658-670):
//   r = x; x = dwconv7(x) + dw_b (depthwise causal, voc_conv1d_causal groups == C,
//   src/tts_vocoder_ops.c:52-73); x = LayerNorm over channels per time step, eps 1e-6
//   (voc_layer_norm_channels, :311-336); h = gelu(W1 x + b1) (W1 [4C, C], voc_gelu exact
//   erf, :344-349); x = (W2 h + b2) * gamma + r (W2 [C, 4C]).
//
// Three launches per block:
//   dwconv_ln_kernel  one warp per time row: 7 taps from the row and the 6 before it
//                     (zero before t = 0), bias, then mean / variance across the row's C
//                     channels by warp shuffles, scale and shift; writes the LayerNorm
//                     output in the 3xTF32 hi/lo form the GEMM reads. The tap weights are
//                     transposed into shared memory once per CTA; each CTA walks a
//                     contiguous run of rows so the 7-fold row re-reads hit L1.
//   pw1 GEMM          voc_conv.cuh with M = time, N = 4C, K = C; epilogue: bias, exact GELU,
//                     hi/lo split of h [T, 4C].
//   pw2 GEMM          N = C, K = 4C; epilogue: (acc + b2) * gamma + x, in place on x.
// HBM traffic per element of x: dwconv+LN reads x 4 B, writes 8 B; pw1 reads 8 B, writes
// 32 B (h is 4C wide, hi/lo); pw2 reads 32 B + x 4 B, writes 4 B.
#include "voc_conv.cuh"

namespace lai {
namespace {

constexpr int kLnWarps = 8;
constexpr int kLnRowsPerWarp = 8;  // a CTA covers 64 consecutive time rows

// C = 128 * NV channels: lane owns channels 128 j + 4 lane .. + 3 for j < NV.
template <int NV, int PASSES>
__global__ void __launch_bounds__(kLnWarps * 32)
dwconv_ln_kernel(const float *__restrict__ x, const float *__restrict__ dw_w,
                 const float *__restrict__ dw_b, const float *__restrict__ nw,
                 const float *__restrict__ nb, float *hi, float *lo, int T, int64_t rows,
                 float eps) {
    constexpr int C = NV * 128;
    extern __shared__ float wt[];  // [7][C]: tap-major copy of dw_w [C, 1, 7]
    for (int i = threadIdx.x; i < 7 * C; i += blockDim.x) {
        const int c = i / 7, k = i - c * 7;
        wt[k * C + c] = dw_w[i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t row0 = (int64_t)blockIdx.x * kLnWarps * kLnRowsPerWarp;
    for (int r = 0; r < kLnRowsPerWarp; r++) {
        const int64_t row = row0 + (int64_t)r * kLnWarps + warp;
        if (row >= rows) break;
        const int t = (int)(row % T);
        float acc[NV][4];
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const float4 bb = *reinterpret_cast<const float4 *>(dw_b + 128 * j + 4 * lane);
            acc[j][0] = bb.x; acc[j][1] = bb.y; acc[j][2] = bb.z; acc[j][3] = bb.w;
        }
#pragma unroll
        for (int k = 0; k < 7; k++) {
            if (t - 6 + k < 0) continue;  // causal zero padding
            const float *xr = x + (row - 6 + k) * C;
#pragma unroll
            for (int j = 0; j < NV; j++) {
                const int c = 128 * j + 4 * lane;
                const float4 v = *reinterpret_cast<const float4 *>(xr + c);
                const float4 w = *reinterpret_cast<const float4 *>(wt + k * C + c);
                acc[j][0] = fmaf(w.x, v.x, acc[j][0]);
                acc[j][1] = fmaf(w.y, v.y, acc[j][1]);
                acc[j][2] = fmaf(w.z, v.z, acc[j][2]);
                acc[j][3] = fmaf(w.w, v.w, acc[j][3]);
            }
        }
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++) s += (acc[j][0] + acc[j][1]) + (acc[j][2] + acc[j][3]);
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        const float mean = s / (float)C;
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < NV; j++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float d = acc[j][e] - mean;
                q = fmaf(d, d, q);
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
        const float inv = 1.0f / sqrtf(q / (float)C + eps);
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const int c = 128 * j + 4 * lane;
            const float4 gw = *reinterpret_cast<const float4 *>(nw + c);
            const float4 gb = *reinterpret_cast<const float4 *>(nb + c);
            const float g[4] = {gw.x, gw.y, gw.z, gw.w}, bb[4] = {gb.x, gb.y, gb.z, gb.w};
            float y[4], h[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                y[e] = (acc[j][e] - mean) * inv * g[e] + bb[e];
                h[e] = umma::tf32_round(y[e]);
            }
            *reinterpret_cast<float4 *>(hi + row * C + c) = make_float4(h[0], h[1], h[2], h[3]);
            if (PASSES == 3)
                *reinterpret_cast<float4 *>(lo + row * C + c) =
                    make_float4(y[0] - h[0], y[1] - h[1], y[2] - h[2], y[3] - h[3]);
        }
    }
}

template <int NV, int PASSES>
int launch_dwconv_ln(const float *x, const lai_voc_convnext_t &p, float *hi, float *lo, int T,
                     int64_t rows, cudaStream_t st) {
    constexpr int C = NV * 128;
    const size_t smem = 7 * C * sizeof(float);
    auto kern = dwconv_ln_kernel<NV, PASSES>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
        return LAI_ERR_CUDA;
    const unsigned grid = grid_for(rows, kLnWarps * kLnRowsPerWarp);
    kern<<<grid, kLnWarps * 32, smem, st>>>(x, p.dw_w, p.dw_b, p.norm_w, p.norm_b, hi, lo, T, rows,
                                            1e-6f);
    return launch_status();
}

template <int PASSES>
int dwconv_ln(int C, const float *x, const lai_voc_convnext_t &p, float *hi, float *lo, int T,
              int64_t rows, cudaStream_t st) {
    switch (C) {
        case 128: return launch_dwconv_ln<1, PASSES>(x, p, hi, lo, T, rows, st);
        case 256: return launch_dwconv_ln<2, PASSES>(x, p, hi, lo, T, rows, st);
        case 512: return launch_dwconv_ln<4, PASSES>(x, p, hi, lo, T, rows, st);
        case 1024: return launch_dwconv_ln<8, PASSES>(x, p, hi, lo, T, rows, st);
        case 2048: return launch_dwconv_ln<16, PASSES>(x, p, hi, lo, T, rows, st);
        default: return LAI_ERR_INVALID;
    }
}

}  // namespace
}  // namespace lai

extern "C" int lai_voc_convnext_f32(float *x, float *scratch, const lai_voc_convnext_t *p,
                                    int batch, int channels, int T, int passes, int *err,
                                    lai_stream_t stream) {
    using namespace lai;
    if (!x || !scratch || !p || batch < 0 || T < 0 || (passes != 1 && passes != 3))
        return LAI_ERR_INVALID;
    if (batch == 0 || T == 0) return LAI_OK;
    if (channels != 128 && channels != 256 && channels != 512 && channels != 1024 &&
        channels != 2048)
        return LAI_ERR_INVALID;
    if (!p->dw_w || !p->dw_b || !p->norm_w || !p->norm_b || !p->pw1_w || !p->pw1_b || !p->pw2_w ||
        !p->pw2_b || !p->gamma || !aligned16(x) || !aligned16(scratch) || !aligned16(p->pw1_w) ||
        !aligned16(p->pw2_w) || !aligned16(p->dw_b) || !aligned16(p->norm_w) ||
        !aligned16(p->norm_b))
        return LAI_ERR_INVALID;
    if (batch > 65535) return LAI_ERR_RANGE;
    const size_t plane = (size_t)batch * T * channels;
    if (overlaps(x, plane * 4, scratch, 10 * plane * 4)) return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    float *s_hi = scratch, *s_lo = scratch + plane;
    float *h_hi = scratch + 2 * plane, *h_lo = scratch + 6 * plane;  // [B, T, 4C] each
    const cudaStream_t st = as_stream(stream);
    const int64_t rows = (int64_t)batch * T;
    int rc = passes == 3 ? dwconv_ln<3>(channels, x, *p, s_hi, s_lo, T, rows, st)
                         : dwconv_ln<1>(channels, x, *p, s_hi, s_lo, T, rows, st);
    if (rc != LAI_OK) return rc;
    const int C4 = 4 * channels;
    CUtensorMap s_map, h_map, w1, w2;
    if (!act_map(&s_map, s_hi, batch, T, channels) || !act_map(&h_map, h_hi, batch, T, C4) ||
        !weight_map(&w1, p->pw1_w, 1, C4, channels, pick_bn(C4)) ||
        !weight_map(&w2, p->pw2_w, 1, channels, C4, pick_bn(channels)))
        return LAI_ERR_INVALID;
    const ConvArgs a1{h_hi, h_lo, nullptr, p->pw1_b, nullptr, nullptr, nullptr,
                      T, channels, C4, 1, 1, err};
    rc = launch_conv<kEpiGelu>(passes, s_map, w1, a1, batch, st);
    if (rc != LAI_OK) return rc;
    const ConvArgs a2{nullptr, nullptr, x, p->pw2_b, nullptr, nullptr, p->gamma,
                      T, C4, channels, 1, 1, err};
    return launch_conv<kEpiScaleResidual>(passes, h_map, w2, a2, batch, st);
}

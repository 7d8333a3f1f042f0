// voc_resunit.cu - vocoder BigVGAN ResUnit on tcgen05 tensor cores, FP32 results.
//
// Reference: run_resunit (src/tts_vocoder.c:540-583) on x [C, T]:
//   r = x; x = snake1(x); h = conv1d_causal(x, w1 [C, C, 7], dilation d) + b1;
//   h = snake2(h); x = conv1d(h, w2 [C, C, 1]) + b2 + r
// with voc_conv1d_causal (src/tts_vocoder_ops.c:44-147: left zero padding of
// d * 6, im2col + SGEMM) and voc_snake_beta (:279-305). The three ResUnits of a
// BigVGAN block run back to back (src/tts_vocoder.c:725-728, dilations 1, 3, 9).
//
// The convolutions run on tensor cores as implicit GEMMs over channels-last activations
// [batch, T, C] (voc_conv.cuh: layout, 3xTF32 precision, pipeline).
//
// Fusion. SnakeBeta never runs as its own pass inside a block: conv1's epilogue
// applies bias + snake2 and writes h split; conv2's epilogue adds bias and the
// residual in place on x and applies the NEXT unit's snake1, writing its split input.
// Only the first unit's snake1 is a separate elementwise kernel (its input comes from
// outside). HBM traffic per unit and element: conv1 reads s (8 B) and writes h (8 B);
// conv2 reads h (8 B) and x (4 B), writes x (4 B) and s (8 B).
#include "voc_conv.cuh"

namespace lai {
namespace {

// s = snake(x) in split form (the first unit's input): x [rows, C] channels-last.
template <int PASSES>
__global__ void __launch_bounds__(256)
snake_split_kernel(const float *__restrict__ x, const float *__restrict__ ea,
                   const float *__restrict__ ieb, float *hi, float *lo, int64_t n4, int C) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        const int c = (int)((i * 4) % C);  // C % 4 == 0: the 4 lanes share a row
        // SnakeBeta two channels per instruction (snake2: same bits as snake1)
        const float2 lo2 = snake2(make_float2(v.x, v.y), make_float2(__ldg(ea + c), __ldg(ea + c + 1)),
                                  make_float2(__ldg(ieb + c), __ldg(ieb + c + 1)));
        const float2 hi2 = snake2(make_float2(v.z, v.w),
                                  make_float2(__ldg(ea + c + 2), __ldg(ea + c + 3)),
                                  make_float2(__ldg(ieb + c + 2), __ldg(ieb + c + 3)));
        float y[4] = {lo2.x, lo2.y, hi2.x, hi2.y}, h[4];
#pragma unroll
        for (int k = 0; k < 4; k++) h[k] = umma::tf32_round(y[k]);
        reinterpret_cast<float4 *>(hi)[i] = make_float4(h[0], h[1], h[2], h[3]);
        if (PASSES == 3)
            reinterpret_cast<float4 *>(lo)[i] =
                make_float4(y[0] - h[0], y[1] - h[1], y[2] - h[2], y[3] - h[3]);
    }
}

// Reference weight [c_out, c_in, taps] -> [2][taps][c_out][c_in] (hi plane, lo plane).
__global__ void pack_conv_kernel(float *dst, const float *__restrict__ w, int c_out, int c_in,
                                 int taps) {
    const int64_t per_plane = (int64_t)taps * c_out * c_in;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per_plane;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t k = i / ((int64_t)c_out * c_in);
        const int64_t oc = i - k * c_out * c_in;  // o * c_in + c
        const float v = w[oc * taps + k];
        const float h = umma::tf32_round(v);
        dst[i] = h;
        dst[per_plane + i] = v - h;
    }
}

// Batched transpose: dst[b][j][i] = src[b][i][j], src [batch][R][Ccols].
__global__ void transpose_kernel(float *dst, const float *__restrict__ src, int R, int Ccols) {
    __shared__ float tile[32][33];
    const int64_t base = (int64_t)blockIdx.z * R * Ccols;
    const int i0 = blockIdx.y * 32, j0 = blockIdx.x * 32;
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int i = i0 + k, j = j0 + threadIdx.x;
        if (i < R && j < Ccols) tile[k][threadIdx.x] = src[base + (int64_t)i * Ccols + j];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += 8) {
        const int j = j0 + k, i = i0 + threadIdx.x;
        if (i < R && j < Ccols) dst[base + (int64_t)j * R + i] = tile[threadIdx.x][k];
    }
}

}  // namespace
}  // namespace lai

extern "C" int lai_voc_pack_conv_f32(float *dst, const float *w, int c_out, int c_in, int kernel,
                                     lai_stream_t stream) {
    if (!dst || !w || c_out <= 0 || c_in <= 0 || kernel <= 0) return LAI_ERR_INVALID;
    const size_t n = (size_t)c_out * c_in * kernel;
    if (lai::overlaps(dst, 2 * n * sizeof(float), w, n * sizeof(float))) return LAI_ERR_ALIAS;
    const unsigned grid = lai::grid_for((int64_t)n, 256) < 148u * 8 ? lai::grid_for((int64_t)n, 256)
                                                                   : 148u * 8;
    lai::pack_conv_kernel<<<grid, 256, 0, lai::as_stream(stream)>>>(dst, w, c_out, c_in, kernel);
    return lai::launch_status();
}

extern "C" int lai_voc_transpose_f32(float *dst, const float *src, int batch, int rows, int cols,
                                     lai_stream_t stream) {
    if (!dst || !src || batch < 0 || rows < 0 || cols < 0) return LAI_ERR_INVALID;
    if (batch == 0 || rows == 0 || cols == 0) return LAI_OK;
    const size_t n = (size_t)batch * rows * cols * sizeof(float);
    if (lai::overlaps(dst, n, src, n)) return LAI_ERR_ALIAS;
    if (batch > 65535) return LAI_ERR_RANGE;
    const dim3 grid((unsigned)((cols + 31) / 32), (unsigned)((rows + 31) / 32), (unsigned)batch);
    if (grid.y > 65535) return LAI_ERR_RANGE;
    lai::transpose_kernel<<<grid, dim3(32, 8), 0, lai::as_stream(stream)>>>(dst, src, rows, cols);
    return lai::launch_status();
}

namespace lai {
namespace {

bool units_valid(const lai_voc_resunit_t *units, int n_units) {
    for (int u = 0; u < n_units; u++) {
        const lai_voc_resunit_t &p = units[u];
        if (!p.snake1_ea || !p.snake1_ieb || !p.conv1_w || !p.conv1_b || !p.snake2_ea ||
            !p.snake2_ieb || !p.conv2_w || !p.conv2_b || p.dilation <= 0 ||
            (int64_t)p.dilation * 6 > (int64_t)1 << 30 || !aligned16(p.conv1_w) ||
            !aligned16(p.conv2_w))
            return false;
    }
    return true;
}

// s = snake(x) split into scratch planes hi / lo ([rows, C] channels-last)
void launch_snake_split(const float *x, const float *ea, const float *ieb, float *hi, float *lo,
                        size_t n, int C, int passes, cudaStream_t st) {
    const int64_t n4 = (int64_t)n / 4;
    const unsigned g = grid_for(n4, 256) < 148u * 16 ? grid_for(n4, 256) : 148u * 16;
    if (passes == 3)
        snake_split_kernel<3><<<g, 256, 0, st>>>(x, ea, ieb, hi, lo, n4, C);
    else
        snake_split_kernel<1><<<g, 256, 0, st>>>(x, ea, ieb, hi, lo, n4, C);
}

// The ResUnit chain on x [batch, T, C]; scratch = [s hi, s lo, h hi, h lo] planes. With
// s_ready the first unit's split input is already in the s planes (written by the
// transposed conv's epilogue).
int run_resunits(float *x, float *scratch, const lai_voc_resunit_t *units, int n_units, int batch,
                 int channels, int T, int passes, int *err, cudaStream_t st, bool s_ready) {
    const size_t plane = (size_t)batch * T * channels;
    float *s_hi = scratch, *s_lo = scratch + plane, *h_hi = scratch + 2 * plane,
          *h_lo = scratch + 3 * plane;
    CUtensorMap s_map, h_map;
    if (!act_map(&s_map, s_hi, batch, T, channels) || !act_map(&h_map, h_hi, batch, T, channels))
        return LAI_ERR_INVALID;
    const int bn = pick_bn(channels);
    int rc = LAI_OK;
    if (!s_ready) {
        launch_snake_split(x, units[0].snake1_ea, units[0].snake1_ieb, s_hi, s_lo, plane, channels,
                           passes, st);
        rc = launch_status();
    }
    for (int u = 0; u < n_units && rc == LAI_OK; u++) {
        const lai_voc_resunit_t &p = units[u];
        CUtensorMap w1, w2;
        if (!weight_map(&w1, p.conv1_w, 7, channels, channels, bn) ||
            !weight_map(&w2, p.conv2_w, 1, channels, channels, bn))
            return LAI_ERR_INVALID;
        ConvArgs c1{h_hi, h_lo, nullptr, p.conv1_b, p.snake2_ea, p.snake2_ieb, nullptr,
                    T, channels, channels, 7, p.dilation, err, 1, T};
        rc = launch_conv<kEpiSnakeSplit>(passes, s_map, w1, c1, batch, st);
        if (rc != LAI_OK) break;
        const bool last = u + 1 == n_units;
        ConvArgs c2{last ? nullptr : s_hi, last ? nullptr : s_lo, x, p.conv2_b,
                    last ? nullptr : units[u + 1].snake1_ea,
                    last ? nullptr : units[u + 1].snake1_ieb, nullptr, T, channels, channels, 1,
                    1, err, 1, T};
        rc = launch_conv<kEpiResidual>(passes, h_map, w2, c2, batch, st);
    }
    return rc;
}

// Reference transposed-conv weight [c_in, c_out, kernel] -> [2][stride][taps][c_out][c_in],
// taps = kernel / stride: part (hi, lo), phase f, tap. kernel 2r: tap 0 = W[.., r + f]
// (applied to x[t - 1]), tap 1 = W[.., f] (applied to x[t]); kernel r: tap 0 = W[.., f].
__global__ void pack_tconv_kernel(float *dst, const float *__restrict__ w, int c_in, int c_out,
                                  int kernel, int stride) {
    const int taps = kernel / stride;
    const int64_t per_part = (int64_t)kernel * c_out * c_in;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < per_part;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t oc = i % ((int64_t)c_out * c_in);  // o * c_in + c
        const int64_t pk = i / ((int64_t)c_out * c_in);  // phase * taps + tap
        const int f = (int)(pk / taps), tap = (int)(pk % taps);
        const int64_t o = oc / c_in, c = oc % c_in;
        const int ki = taps == 2 && tap == 0 ? stride + f : f;
        const float v = w[(c * c_out + o) * kernel + ki];
        const float h = umma::tf32_round(v);
        dst[i] = h;
        dst[per_part + i] = v - h;
    }
}

}  // namespace
}  // namespace lai

extern "C" int lai_voc_resunits_f32(float *x, float *scratch, const lai_voc_resunit_t *units,
                                    int n_units, int batch, int channels, int T, int passes,
                                    int *err, lai_stream_t stream) {
    using namespace lai;
    if (!x || !scratch || !units || n_units < 0 || batch < 0 || channels <= 0 || T < 0 ||
        (passes != 1 && passes != 3))
        return LAI_ERR_INVALID;
    if (n_units == 0 || batch == 0 || T == 0) return LAI_OK;
    if (channels % 32 != 0 || !aligned16(x) || !aligned16(scratch)) return LAI_ERR_INVALID;
    if (batch > 65535) return LAI_ERR_RANGE;
    if (!units_valid(units, n_units)) return LAI_ERR_INVALID;
    const size_t plane = (size_t)batch * T * channels;
    if (overlaps(x, plane * 4, scratch, 4 * plane * 4)) return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    return run_resunits(x, scratch, units, n_units, batch, channels, T, passes, err,
                        as_stream(stream), false);
}

extern "C" int lai_voc_pack_tconv_f32(float *dst, const float *w, int c_in, int c_out, int kernel,
                                      int stride, lai_stream_t stream) {
    if (!dst || !w || c_in <= 0 || c_out <= 0 || stride <= 0 ||
        (kernel != stride && kernel != 2 * stride))
        return LAI_ERR_INVALID;
    const size_t n = (size_t)c_in * c_out * kernel;
    if (lai::overlaps(dst, 2 * n * sizeof(float), w, n * sizeof(float))) return LAI_ERR_ALIAS;
    const unsigned grid = lai::grid_for((int64_t)n, 256) < 148u * 8 ? lai::grid_for((int64_t)n, 256)
                                                                   : 148u * 8;
    lai::pack_tconv_kernel<<<grid, 256, 0, lai::as_stream(stream)>>>(dst, w, c_in, c_out, kernel,
                                                                     stride);
    return lai::launch_status();
}

extern "C" int lai_voc_bigvgan_block_f32(float *out, const float *x, float *scratch,
                                         const lai_voc_bigvgan_block_t *blk, int batch, int c_in,
                                         int c_out, int T, int passes, int *err,
                                         lai_stream_t stream) {
    using namespace lai;
    if (!out || !x || !scratch || !blk || batch < 0 || T < 0 || (passes != 1 && passes != 3))
        return LAI_ERR_INVALID;
    if (!blk->snake_ea || !blk->snake_ieb || !blk->tconv_w || !blk->tconv_b || blk->rate <= 0 ||
        blk->n_units < 0 || (blk->n_units > 0 && !blk->units))
        return LAI_ERR_INVALID;
    if (batch == 0 || T < 2) return batch == 0 ? LAI_OK : LAI_ERR_INVALID;
    if (c_in % 32 != 0 || c_out % 32 != 0 || !aligned16(out) || !aligned16(x) ||
        !aligned16(scratch) || !aligned16(blk->tconv_w))
        return LAI_ERR_INVALID;
    if ((int64_t)batch * blk->rate > 65535) return LAI_ERR_RANGE;
    if (!units_valid(blk->units, blk->n_units)) return LAI_ERR_INVALID;
    const int r = blk->rate;
    const int T_out = (T - 1) * r;  // (T + 1) r - 2r
    const size_t in_plane = (size_t)batch * T * c_in, out_plane = (size_t)batch * T_out * c_out;
    if (overlaps(out, out_plane * 4, x, in_plane * 4) ||
        overlaps(out, out_plane * 4, scratch, (2 * in_plane + 4 * out_plane) * 4) ||
        overlaps(x, in_plane * 4, scratch, (2 * in_plane + 4 * out_plane) * 4))
        return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    const cudaStream_t st = as_stream(stream);
    float *in_hi = scratch, *in_lo = scratch + in_plane;
    float *rs = scratch + 2 * in_plane;  // the ResUnits' scratch; its s planes come first
    // block snake -> split planes of the transposed conv's input
    launch_snake_split(x, blk->snake_ea, blk->snake_ieb, in_hi, in_lo, in_plane, c_in, passes, st);
    int rc = launch_status();
    if (rc != LAI_OK) return rc;
    CUtensorMap in_map, w_map;
    if (!act_map(&in_map, in_hi, batch, T, c_in) ||
        !weight_map(&w_map, blk->tconv_w, 2 * r, c_out, c_in, pick_bn(c_out)))
        return LAI_ERR_INVALID;
    const bool fuse = blk->n_units > 0;  // epilogue also writes the first unit's snake1 input
    const ConvArgs a{fuse ? rs : nullptr, fuse ? rs + out_plane : nullptr, out, blk->tconv_b,
                     fuse ? blk->units[0].snake1_ea : nullptr,
                     fuse ? blk->units[0].snake1_ieb : nullptr, nullptr, T, c_in, c_out, 2, 1,
                     err, r, T_out, 1};
    rc = launch_conv<kEpiStoreSnake>(passes, in_map, w_map, a, batch, st);
    if (rc != LAI_OK || !fuse) return rc;
    return run_resunits(out, rs, blk->units, blk->n_units, batch, c_out, T_out, passes, err, st,
                        true);
}

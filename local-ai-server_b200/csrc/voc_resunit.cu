// voc_resunit.cu - vocoder BigVGAN ResUnit on tcgen05 tensor cores, FP32 results.
//
// Reference: run_resunit (src/tts_vocoder.c:540-583) on x [C, T]:
//   r = x; x = snake1(x); h = conv1d_causal(x, w1 [C, C, 7], dilation d) + b1;
//   h = snake2(h); x = conv1d(h, w2 [C, C, 1]) + b2 + r
// with voc_conv1d_causal (src/tts_vocoder_ops.c:44-147: left zero padding of
// d * 6, im2col + SGEMM) and voc_snake_beta (:279-305). The three ResUnits of a
// BigVGAN block run back to back (src/tts_vocoder.c:725-728, dilations 1, 3, 9).
//
// Layout. Activations are channels-last, [batch, T, C] F32, so that a convolution
// tap is a shift along time = the OUTER coordinate of a TMA tile: tap k of output
// rows [t0, t0 + 128) reads input rows starting at t0 - (6 - k) * d, a negative
// start reads the tensor map's zero fill (the causal padding) and the inner (channel)
// coordinate stays a multiple of 16 floats. Each convolution is then an implicit
// GEMM  D[t, o] = sum_{k, c} S[t - (6-k) d, c] * W_k[o, c]  with M = time,
// N = output channels, K = taps x input channels; no im2col buffer exists.
//
// Precision (3 passes, the default). kind::tf32 multiplies 10-bit-mantissa inputs,
// so every operand is carried as a pair hi = tf32(v), lo = v - hi (both exact in
// F32) and each product is hi*hi + hi*lo + lo*hi: the dropped lo*lo term and the
// TF32 view of lo are ~2^-21 relative, below F32 round-off of the reference's own
// sums. passes = 1 uses hi*hi alone (plain TF32). Activation planes are written in
// this split form by the epilogue that produces them, weights by lai_voc_pack_conv_f32.
//
// Fusion. SnakeBeta never runs as its own pass inside a block: conv1's epilogue
// applies bias + snake2 and writes h split; conv2's epilogue adds bias and the
// residual in place on x and applies the NEXT unit's snake1, writing its split input.
// Only the first unit's snake1 is a separate elementwise kernel (its input comes from
// outside). HBM traffic per unit and element: conv1 reads s (8 B) and writes h (8 B);
// conv2 reads h (8 B) and x (4 B), writes x (4 B) and s (8 B).
//
// Kernel: one CTA per 128-row x BN-channel output tile, 320 threads. Warp 0 issues
// TMA loads into a STAGES-deep ring (64-byte-swizzled K-major tiles of 16 channels),
// warp 1 owns TMEM and issues tcgen05.mma from one thread, warps 2-9 drain finished
// K chunks from TMEM (lane quarter = warp % 4, half the columns each) into F32
// registers and finally apply bias / snake / residual and store to HBM.
// Every mbarrier wait is bounded (globaltimer); a timeout sets LAI_DEVERR_TIMEOUT in
// *err and the CTA still releases its TMEM before returning.
#include <mutex>

#include "lai_common.cuh"
#include "snake_math.cuh"
#include "umma.cuh"

namespace lai {
namespace {

constexpr int kBM = 128;        // output time rows per tile = UMMA M = TMEM lanes
constexpr int kBK = 16;         // input channels per K block: one 64-byte row of F32
constexpr int kUmmaK = 8;       // K of one kind::tf32 MMA (32 bytes)
constexpr int kEpiWarps = 8;    // two per TMEM lane quarter, each half of the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;  // warp 0 TMA, warp 1 MMA + TMEM, 2..9 drain
constexpr int kChunkBlocks = 2; // K blocks per TMEM accumulation chunk (32 input channels)
constexpr int kSmemTiles = 192 * 1024;
constexpr int kEpiPitch = 33;   // floats per row of a drain warp's 32 x 32 transpose buffer
constexpr uint32_t kEpiBytes = kEpiWarps * 32 * kEpiPitch * 4;
constexpr int kMaxStages = 8;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far beyond any healthy wait

enum Epi { kEpiSnakeSplit = 0, kEpiResidual = 1 };

struct ConvArgs {
    float *out_hi, *out_lo;  // split output planes (kEpiResidual: next unit's input, or null)
    float *x;                // kEpiResidual: residual stream, updated in place
    const float *bias;       // [c_out]
    const float *ea, *ieb;   // snake applied to the output (kEpiResidual: next snake1, or null)
    int T, c_in, c_out, taps, dilation;
    int *err;
};

template <int BN, int PASSES>
struct Tile {
    static constexpr uint32_t kA = kBM * kBK * 4;  // 8 KiB
    static constexpr uint32_t kB = BN * kBK * 4;
    static constexpr uint32_t kStage = (kA + kB) * (PASSES == 3 ? 2u : 1u);
    static constexpr int kStages =
        (int)(kSmemTiles / kStage) < kMaxStages ? (int)(kSmemTiles / kStage) : kMaxStages;
    // align slack + operand ring + the drain warps' transpose buffers + barriers
    static constexpr uint32_t kSmem = 1024 + kStages * kStage + kEpiBytes + 256;
    // two accumulator buffers: the MMAs fill one chunk while the other is drained
    static constexpr uint32_t kBufCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static constexpr uint32_t kTmemCols = 2 * kBufCols;
    static constexpr int kHalf = BN / 2;  // columns per drain warp
    static_assert(kA % 1024 == 0 && kB % 1024 == 0, "tiles must keep 1 KiB alignment");
    static_assert(kStages >= 2, "pipeline needs two stages");
    static_assert(kHalf % 16 == 0, "drain warps read 16-column groups");
};

__device__ __forceinline__ void store4(float *p, float a, float b, float c, float d) {
    *reinterpret_cast<float4 *>(p) = make_float4(a, b, c, d);
}

// Epilogue for 4 finished sums of output row `row` (global index), channels [c, c + 4):
// bias, then either snake + hi/lo split (conv1) or residual in place and the next unit's
// snake + split (conv2). `xr` holds x[row, c..c+3] for the residual, loaded earlier.
template <int PASSES, int EPI>
__device__ __forceinline__ void epilogue4(const ConvArgs &a, float (&v)[4], const float4 &xr,
                                          size_t row, int c) {
    const size_t off = row * (size_t)a.c_out + c;
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] += __ldg(a.bias + c + i);
    if (EPI == kEpiResidual) {
        v[0] += xr.x; v[1] += xr.y; v[2] += xr.z; v[3] += xr.w;
        store4(a.x + off, v[0], v[1], v[2], v[3]);
        if (a.ea == nullptr) return;
    }
    float hi[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        v[i] = snake1(v[i], __ldg(a.ea + c + i), __ldg(a.ieb + c + i));
        hi[i] = umma::tf32_round(v[i]);
    }
    store4(a.out_hi + off, hi[0], hi[1], hi[2], hi[3]);
    if (PASSES == 3)
        store4(a.out_lo + off, v[0] - hi[0], v[1] - hi[1], v[2] - hi[2], v[3] - hi[3]);
}

// Accumulation. The tensor core's F32 accumulation does not round to nearest: measured
// against double sums, its error grows linearly with the number of MMAs that update one
// accumulator and leans toward zero (biased), reaching ~2e-4 relative for a 7 x 768
// channel sum. Chunks of 2 blocks (6 MMAs per fresh accumulator with 3 passes) bring a
// 768-channel unit to ~3e-6 of the double-precision oracle; 4 blocks gave ~5e-6. So K is cut into chunks of kChunkBlocks blocks; each chunk starts a fresh
// TMEM accumulator (alternating between two buffers) and the drain warps add the
// finished chunk into F32 registers with round-to-nearest adds while the MMAs fill the
// other buffer. Chunk errors then carry each chunk's own sign and largely cancel.
//
// act_map: [2 planes][batch][T][c_in] (hi, lo); w_map: [2 * taps][c_out][c_in] (hi taps,
// then lo taps). Grid: (ceil(T / 128), c_out / BN, batch).
template <int BN, int PASSES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
conv_umma_kernel(const __grid_constant__ CUtensorMap act_map,
                 const __grid_constant__ CUtensorMap w_map, const ConvArgs a) {
    using L = Tile<BN, PASSES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *tiles = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    float *epi_buf = reinterpret_cast<float *>(tiles + L::kStages * L::kStage);
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + L::kStages * L::kStage + kEpiBytes);
    uint64_t *empty = full + L::kStages;
    uint64_t *acc_full = empty + L::kStages;  // [2]: chunk ready in buffer b
    uint64_t *acc_empty = acc_full + 2;       // [2]: buffer b drained
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int t0 = blockIdx.x * kBM, n0 = blockIdx.y * BN, b = blockIdx.z;
    const int kblocks = a.c_in / kBK;
    const int n_iter = a.taps * kblocks;
    const int n_chunks = (n_iter + kChunkBlocks - 1) / kChunkBlocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < L::kStages; s++) {
            bulk::mbar_init(&full[s], 1);
            bulk::mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; i++) {
            bulk::mbar_init(&acc_full[i], 1);
            bulk::mbar_init(&acc_empty[i], kEpiWarps);
        }
        bulk::fence_barrier_init();
        umma::prefetch_tensormap(&act_map);
        umma::prefetch_tensormap(&w_map);
    }
    if (warp == 1) {
        umma::tmem_alloc(tmem_slot, L::kTmemCols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tmem = *tmem_slot;

    bool ok = true;
    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            for (int it = 0; it < n_iter; it++) {
                const int s = it % L::kStages;
                if (it >= L::kStages &&
                    !bulk::mbar_wait_bounded(&empty[s], ((it / L::kStages) + 1) & 1, kWaitNs)) {
                    ok = false;
                    break;
                }
                const int tap = it / kblocks, kb = it - tap * kblocks;
                const int c = kb * kBK;
                const int row = t0 - (a.taps - 1 - tap) * a.dilation;
                uint8_t *st = tiles + s * L::kStage;
                bulk::mbar_arrive_expect_tx(&full[s], L::kStage);
                umma::tma_load_4d(st, &act_map, c, row, b, 0, &full[s]);
                umma::tma_load_3d(st + L::kA, &w_map, c, n0, tap, &full[s]);
                if (PASSES == 3) {
                    umma::tma_load_4d(st + L::kA + L::kB, &act_map, c, row, b, 1, &full[s]);
                    umma::tma_load_3d(st + 2 * L::kA + L::kB, &w_map, c, n0, a.taps + tap,
                                      &full[s]);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = umma::idesc_tf32<kBM, BN>();
            for (int it = 0; it < n_iter; it++) {
                const int s = it % L::kStages;
                const int j = it / kChunkBlocks;
                const bool first = it - j * kChunkBlocks == 0;
                if (first && j >= 2 &&
                    !bulk::mbar_wait_bounded(&acc_empty[j & 1], ((j >> 1) - 1) & 1, kWaitNs)) {
                    ok = false;
                    break;
                }
                if (!bulk::mbar_wait_bounded(&full[s], (it / L::kStages) & 1, kWaitNs)) {
                    ok = false;
                    break;
                }
                umma::fence_after_sync();
                const uint32_t d = tmem + (uint32_t)(j & 1) * L::kBufCols;
                const uint32_t st = umma::smem_addr(tiles + s * L::kStage);
#pragma unroll
                for (int k = 0; k < kBK / kUmmaK; k++) {
                    const uint32_t kofs = k * kUmmaK * 4;
                    const uint64_t ah = umma::desc_kmajor_sw64(st + kofs);
                    const uint64_t bh = umma::desc_kmajor_sw64(st + L::kA + kofs);
                    umma::mma_tf32(d, ah, bh, idesc, (first && k == 0) ? 0u : 1u);
                    if (PASSES == 3) {
                        const uint64_t al = umma::desc_kmajor_sw64(st + L::kA + L::kB + kofs);
                        const uint64_t bl =
                            umma::desc_kmajor_sw64(st + 2 * L::kA + L::kB + kofs);
                        umma::mma_tf32(d, ah, bl, idesc, 1);
                        umma::mma_tf32(d, al, bh, idesc, 1);
                    }
                }
                umma::commit(&empty[s]);  // frees the stage once these MMAs have read it
                if (it - j * kChunkBlocks == kChunkBlocks - 1 || it == n_iter - 1)
                    umma::commit(&acc_full[j & 1]);
            }
        }
        __syncwarp();
    } else {  // drain / epilogue warps 2..9
        const int q = warp & 3;                 // the TMEM lane quarter this warp may read
        const int half = (warp - 2) >> 2;       // which half of the BN columns
        const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
        float sum[L::kHalf];
#pragma unroll
        for (int i = 0; i < L::kHalf; i++) sum[i] = 0.0f;
        for (int j = 0; j < n_chunks; j++) {
            if (!bulk::mbar_wait_bounded(&acc_full[j & 1], (j >> 1) & 1, kWaitNs)) {
                ok = false;
                break;
            }
            umma::fence_after_sync();
            const uint32_t base = tmem + lane_addr + (uint32_t)(j & 1) * L::kBufCols +
                                  (uint32_t)(half * L::kHalf);
#pragma unroll
            for (int g = 0; g < L::kHalf / 16; g++) {
                uint32_t r[16];
                umma::tmem_ld_32x32b_x16(base + g * 16, r);
                umma::tmem_wait_ld();
#pragma unroll
                for (int i = 0; i < 16; i++) sum[g * 16 + i] += __uint_as_float(r[i]);
            }
            umma::fence_before_sync();
            __syncwarp();
            if (lane == 0) bulk::mbar_arrive(&acc_empty[j & 1]);
        }
        if (ok) {
            // Coalesced epilogue: the warp's 32 rows x GW columns of sums go through a
            // padded shared-memory buffer (row per lane in, conflict-free) and come back
            // as GW/4 lanes per row, 4 consecutive channels each, so every global load and
            // store covers whole 32-byte sectors (a 128-byte line per row when GW = 32).
            constexpr int GW = L::kHalf % 32 == 0 ? 32 : 16;
            constexpr int LPR = GW / 4;    // lanes per row
            constexpr int RPP = 32 / LPR;  // rows per pass
            constexpr int NP = 32 / RPP;   // passes over the 32 rows
            float *buf = epi_buf + (warp - 2) * 32 * kEpiPitch;
            const int r_off = lane / LPR, c4 = (lane % LPR) * 4;
            const int row0 = t0 + q * 32;
#pragma unroll
            for (int g = 0; g < L::kHalf / GW; g++) {
                const int c = n0 + half * L::kHalf + g * GW + c4;
#pragma unroll
                for (int i = 0; i < GW; i++) buf[lane * kEpiPitch + i] = sum[g * GW + i];
                __syncwarp();
                constexpr int PB = NP < 4 ? NP : 4;  // passes whose residual loads fly together
#pragma unroll
                for (int p0 = 0; p0 < NP; p0 += PB) {
                    float4 xr[PB];
                    if (EPI == kEpiResidual) {
#pragma unroll
                        for (int p = 0; p < PB; p++) {
                            const int t = row0 + (p0 + p) * RPP + r_off;
                            xr[p] = t < a.T ? *reinterpret_cast<const float4 *>(
                                                  a.x + ((size_t)b * a.T + t) * a.c_out + c)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int p = 0; p < PB; p++) {
                        const int r = (p0 + p) * RPP + r_off;
                        float v[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) v[i] = buf[r * kEpiPitch + c4 + i];
                        const int t = row0 + r;
                        if (t < a.T)
                            epilogue4<PASSES, EPI>(a, v, EPI == kEpiResidual ? xr[p] : xr[0],
                                                   (size_t)b * a.T + t, c);
                    }
                }
                __syncwarp();
            }
        }
    }
    if (!ok && a.err) atomicOr(a.err, LAI_DEVERR_TIMEOUT);
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tmem, L::kTmemCols);
    }
}

// s = snake(x) in split form (the first unit's input): x [rows, C] channels-last.
template <int PASSES>
__global__ void __launch_bounds__(256)
snake_split_kernel(const float *__restrict__ x, const float *__restrict__ ea,
                   const float *__restrict__ ieb, float *hi, float *lo, int64_t n4, int C) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4 *>(x)[i];
        const int c = (int)((i * 4) % C);  // C % 4 == 0: the 4 lanes share a row
        float y[4] = {v.x, v.y, v.z, v.w}, h[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            y[k] = snake1(y[k], __ldg(ea + c + k), __ldg(ieb + c + k));
            h[k] = umma::tf32_round(y[k]);
        }
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

// ---- host side ----------------------------------------------------------------

using EncodeTiled = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                 const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                 const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiled>(p);
    });
    return fn;
}

// [2][batch][T][C] split activation planes, box 16 channels x 128 rows.
bool act_map(CUtensorMap *m, const float *planes, int batch, int T, int C) {
    const cuuint64_t dims[4] = {(cuuint64_t)C, (cuuint64_t)T, (cuuint64_t)batch, 2};
    const cuuint64_t strides[3] = {(cuuint64_t)C * 4, (cuuint64_t)T * C * 4,
                                   (cuuint64_t)batch * T * C * 4};
    const cuuint32_t box[4] = {kBK, kBM, 1, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float *>(planes), dims,
                       strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// [2 * taps][c_out][c_in] packed weights, box 16 channels x bn rows.
bool weight_map(CUtensorMap *m, const float *w, int taps, int c_out, int c_in, int bn) {
    const cuuint64_t dims[3] = {(cuuint64_t)c_in, (cuuint64_t)c_out, (cuuint64_t)2 * taps};
    const cuuint64_t strides[2] = {(cuuint64_t)c_in * 4, (cuuint64_t)c_out * c_in * 4};
    const cuuint32_t box[3] = {kBK, (cuuint32_t)bn, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(w), dims,
                       strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int pick_bn(int c_out) {
    for (int bn : {256, 192, 128, 96, 64, 32})
        if (c_out % bn == 0) return bn;
    return 0;
}

template <int BN, int PASSES, int EPI>
int launch_conv_t(const CUtensorMap &am, const CUtensorMap &wm, const ConvArgs &a, int batch,
                  cudaStream_t st) {
    using L = Tile<BN, PASSES>;
    auto kern = conv_umma_kernel<BN, PASSES, EPI>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmem) !=
        cudaSuccess)
        return LAI_ERR_CUDA;
    const dim3 grid((unsigned)((a.T + kBM - 1) / kBM), (unsigned)(a.c_out / BN), (unsigned)batch);
    kern<<<grid, kThreads, L::kSmem, st>>>(am, wm, a);
    return launch_status();
}

template <int PASSES, int EPI>
int launch_conv_p(int bn, const CUtensorMap &am, const CUtensorMap &wm, const ConvArgs &a,
                  int batch, cudaStream_t st) {
    switch (bn) {
        case 256: return launch_conv_t<256, PASSES, EPI>(am, wm, a, batch, st);
        case 192: return launch_conv_t<192, PASSES, EPI>(am, wm, a, batch, st);
        case 128: return launch_conv_t<128, PASSES, EPI>(am, wm, a, batch, st);
        case 96: return launch_conv_t<96, PASSES, EPI>(am, wm, a, batch, st);
        case 64: return launch_conv_t<64, PASSES, EPI>(am, wm, a, batch, st);
        case 32: return launch_conv_t<32, PASSES, EPI>(am, wm, a, batch, st);
        default: return LAI_ERR_INVALID;
    }
}

int launch_conv(int passes, int epi, const CUtensorMap &am, const CUtensorMap &wm,
                const ConvArgs &a, int batch, cudaStream_t st) {
    const int bn = pick_bn(a.c_out);
    if (passes == 3)
        return epi == kEpiSnakeSplit ? launch_conv_p<3, kEpiSnakeSplit>(bn, am, wm, a, batch, st)
                                     : launch_conv_p<3, kEpiResidual>(bn, am, wm, a, batch, st);
    return epi == kEpiSnakeSplit ? launch_conv_p<1, kEpiSnakeSplit>(bn, am, wm, a, batch, st)
                                 : launch_conv_p<1, kEpiResidual>(bn, am, wm, a, batch, st);
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
    for (int u = 0; u < n_units; u++) {
        const lai_voc_resunit_t &p = units[u];
        if (!p.snake1_ea || !p.snake1_ieb || !p.conv1_w || !p.conv1_b || !p.snake2_ea ||
            !p.snake2_ieb || !p.conv2_w || !p.conv2_b || p.dilation <= 0 ||
            (int64_t)p.dilation * 6 > (int64_t)1 << 30 || !aligned16(p.conv1_w) ||
            !aligned16(p.conv2_w))
            return LAI_ERR_INVALID;
    }
    const size_t plane = (size_t)batch * T * channels;
    if (overlaps(x, plane * 4, scratch, 4 * plane * 4)) return LAI_ERR_ALIAS;
    if (!encode_fn()) return LAI_ERR_CUDA;
    float *s_hi = scratch, *s_lo = scratch + plane, *h_hi = scratch + 2 * plane,
          *h_lo = scratch + 3 * plane;
    CUtensorMap s_map, h_map;
    if (!act_map(&s_map, s_hi, batch, T, channels) || !act_map(&h_map, h_hi, batch, T, channels))
        return LAI_ERR_INVALID;
    const cudaStream_t st = as_stream(stream);
    const int bn = pick_bn(channels);

    const int64_t n4 = (int64_t)plane / 4;
    const unsigned g = grid_for(n4, 256) < 148u * 16 ? grid_for(n4, 256) : 148u * 16;
    if (passes == 3)
        snake_split_kernel<3><<<g, 256, 0, st>>>(x, units[0].snake1_ea, units[0].snake1_ieb, s_hi,
                                                s_lo, n4, channels);
    else
        snake_split_kernel<1><<<g, 256, 0, st>>>(x, units[0].snake1_ea, units[0].snake1_ieb, s_hi,
                                                s_lo, n4, channels);
    int rc = launch_status();
    for (int u = 0; u < n_units && rc == LAI_OK; u++) {
        const lai_voc_resunit_t &p = units[u];
        CUtensorMap w1, w2;
        if (!weight_map(&w1, p.conv1_w, 7, channels, channels, bn) ||
            !weight_map(&w2, p.conv2_w, 1, channels, channels, bn))
            return LAI_ERR_INVALID;
        ConvArgs c1{h_hi, h_lo, nullptr, p.conv1_b, p.snake2_ea, p.snake2_ieb,
                    T, channels, channels, 7, p.dilation, err};
        rc = launch_conv(passes, kEpiSnakeSplit, s_map, w1, c1, batch, st);
        if (rc != LAI_OK) break;
        const bool last = u + 1 == n_units;
        ConvArgs c2{last ? nullptr : s_hi, last ? nullptr : s_lo, x, p.conv2_b,
                    last ? nullptr : units[u + 1].snake1_ea,
                    last ? nullptr : units[u + 1].snake1_ieb, T, channels, channels, 1, 1, err};
        rc = launch_conv(passes, kEpiResidual, h_map, w2, c2, batch, st);
    }
    return rc;
}

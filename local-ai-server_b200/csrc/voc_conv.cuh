// voc_conv.cuh - causal conv1d / pointwise conv as an implicit GEMM on tcgen05 tensor cores
// (kind::tf32, F32 results), shared by the vocoder's ResUnit (voc_resunit.cu) and ConvNeXt
// (voc_convnext.cu) blocks. Each including file instantiates the epilogues it uses.
//
// Layout. Activations are channels-last, [batch, T, C] F32, so that a convolution
// tap is a shift along time = the OUTER coordinate of a TMA tile: tap k of output
// rows [t0, t0 + 128) reads input rows starting at t0 - (taps-1-k) * d; a negative
// start reads the tensor map's zero fill (the causal padding) and the inner (channel)
// coordinate stays a multiple of 16 floats. A convolution is then the implicit GEMM
// D[t, o] = sum_{k, c} S[t - (taps-1-k) d, c] * W_k[o, c] with M = time, N = output
// channels, K = taps x input channels; no im2col buffer exists (the reference's
// voc_conv1d_causal, src/tts_vocoder_ops.c:44-147, pads, builds im2col and calls SGEMM).
//
// Precision (3 passes, the default). kind::tf32 multiplies 10-bit-mantissa inputs,
// so every operand is carried as a pair hi = tf32(v), lo = v - hi (both exact in
// F32) and each product is hi*hi + hi*lo + lo*hi: the dropped lo*lo term and the
// TF32 view of lo are ~2^-21 relative, below F32 round-off of the reference's own
// sums. passes = 1 uses hi*hi alone (plain TF32). Activation planes are written in
// this split form by the epilogue that produces them, weights by lai_voc_pack_conv_f32.
//
// Kernel: one CTA per 128-row x BN-channel output tile, 320 threads (two CTAs per SM when
// BN <= 128). Warp 0 issues
// TMA loads into a STAGES-deep ring (64-byte-swizzled K-major tiles of 16 channels),
// warp 1 owns TMEM and issues tcgen05.mma from one thread, warps 2-9 drain finished
// K chunks from TMEM (lane quarter = warp % 4, half the columns each) into F32
// registers and finally run the epilogue and store to HBM through a per-warp
// shared-memory transpose (coalesced). Every mbarrier wait is bounded (globaltimer);
// a timeout sets LAI_DEVERR_TIMEOUT in *err and the CTA still releases its TMEM.
#pragma once

#include <cooperative_groups.h>

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
constexpr int kSmemTiles = 227 * 1024;  // the per-CTA maximum when one CTA runs per SM
constexpr int kBarBytes = 256;          // mbarriers + the TMEM address slot
constexpr int kEpiPitch = 33;   // floats per row of a drain warp's 32 x 32 transpose buffer
constexpr uint32_t kEpiBytes = kEpiWarps * 32 * kEpiPitch * 4;
constexpr int kMaxStages = 8;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far beyond any healthy wait

// Epilogues: conv1 of a ResUnit (bias, snake2, split store); conv2 of a ResUnit (bias,
// residual in place, then the next unit's snake1 + split store when ea != null);
// ConvNeXt pw1 (bias, exact GELU, split store); ConvNeXt pw2 (bias, * gamma, residual);
// transposed conv of a BigVGAN block (bias, store x, then the first ResUnit's snake1 +
// split store when ea != null).
enum Epi { kEpiSnakeSplit = 0, kEpiResidual = 1, kEpiGelu = 2, kEpiScaleResidual = 3,
           kEpiStoreSnake = 4 };

struct ConvArgs {
    float *out_hi, *out_lo;  // split output planes (kEpiResidual: next unit's input, or null)
    float *x;                // kEpiResidual: residual stream, updated in place
    const float *bias;       // [c_out]
    const float *ea, *ieb;   // snake applied to the output (kEpiResidual: next snake1, or null)
    const float *gamma;      // kEpiScaleResidual: per-channel layer scale
    int T, c_in, c_out, taps, dilation;
    int *err;
    // Phased output (a transposed conv as `phases` interleaved convs of taps taps): GEMM row
    // t >= row_trim of phase f goes to output row (t - row_trim) * phases + f of a T_out-row
    // sequence (kernel 2r: 2 taps, row_trim 1; kernel r: 1 tap, row_trim 0). phases 0 or 1:
    // an ordinary conv, row t to row t.
    int phases, T_out, row_trim;
};

template <int BN, int PASSES>
struct Tile {
    static constexpr uint32_t kA = kBM * kBK * 4;  // 8 KiB
    static constexpr uint32_t kB = BN * kBK * 4;
    static constexpr uint32_t kStage = (kA + kB) * (PASSES == 3 ? 2u : 1u);
    // Narrow tiles (BN <= 128: at most 2 x 128 TMEM columns) run two CTAs per SM with half
    // the shared memory each, so one CTA's fill, drain and epilogue overlap the other's MMAs
    // (measured: the 96/192/384-channel vocoder stages 24-30% faster than one CTA per SM).
    static constexpr int kMinBlocks = BN <= 128 ? 2 : 1;
    // An SM has 228 KiB of shared memory and reserves 1 KiB per resident CTA; the ring
    // takes what is left after the barriers. The drain warps' transpose buffers reuse the
    // ring once the last MMA has completed, so they cost no pipeline depth: the operand
    // bytes in flight per CTA (all stages but the one the MMAs read) set the rate at
    // which L2 can feed the tensor core.
    static constexpr int kBudget = (kMinBlocks == 2 ? 113 * 1024 : kSmemTiles) - kBarBytes;
    static constexpr int kStages =
        (int)(kBudget / kStage) < kMaxStages ? (int)(kBudget / kStage) : kMaxStages;
    static constexpr uint32_t kRing = kStages * kStage > kEpiBytes ? kStages * kStage : kEpiBytes;
    // operand ring (1 KiB-aligned dynamic shared memory) + barriers
    static constexpr uint32_t kSmem = kRing + kBarBytes;
    // two accumulator buffers: the MMAs fill one chunk while the other is drained
    static constexpr uint32_t kBufCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
    static constexpr uint32_t kTmemCols = 2 * kBufCols;
    static constexpr int kHalf = BN / 2;  // columns per drain warp
    static constexpr int kChunk = kChunkBlocks;
    static_assert(kA % 1024 == 0 && kB % 1024 == 0, "tiles must keep 1 KiB alignment");
    static_assert(kStages >= 2, "pipeline needs two stages");
    static_assert(kMinBlocks == 1 ? kSmem <= 227 * 1024 : 2 * (kSmem + 1024) <= 228 * 1024,
                  "shared memory beyond the SM's capacity for kMinBlocks CTAs");
    static_assert(2 * kStages + 4 <= kBarBytes / 8 - 1, "barrier area too small");
    static_assert(kHalf % 16 == 0, "drain warps read 16-column groups");
    // split-K partial tile [128][BN + 4] in the ring (float4 rows, conflict-free by rows)
    static constexpr int kPartPitch = BN + 4;
    static_assert(kRing >= (uint32_t)kBM * kPartPitch * 4, "partial tile must fit the ring");
};

__device__ __forceinline__ void store4(float *p, float a, float b, float c, float d) {
    *reinterpret_cast<float4 *>(p) = make_float4(a, b, c, d);
}

// Per-channel epilogue parameters of channels [c, c + 4), loaded once per channel group and
// reused for every row the lane finishes (scalar loads: the caller's arrays need only
// 4-byte alignment).
struct EpiParams {
    float bias[4], p1[4], p2[4];  // p1, p2: snake ea, ieb; or gamma (kEpiScaleResidual) in p1
};

template <int EPI>
__device__ __forceinline__ EpiParams epi_params(const ConvArgs &a, int c) {
    EpiParams q;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        q.bias[i] = __ldg(a.bias + c + i);
        q.p1[i] = q.p2[i] = 0.0f;
        if (EPI == kEpiScaleResidual) {
            q.p1[i] = __ldg(a.gamma + c + i);
        } else if (EPI != kEpiGelu && a.ea != nullptr) {
            q.p1[i] = __ldg(a.ea + c + i);
            q.p2[i] = __ldg(a.ieb + c + i);
        }
    }
    return q;
}

// Epilogue for 4 finished sums of output row `row` (global index), channels [c, c + 4).
// `xr` holds x[row, c..c+3] for the residual epilogues, loaded earlier.
// PACK: SnakeBeta two channels per instruction (snake2, same bits as snake1). Used by the
// narrow tiles (BN <= 128, two CTAs per SM), where a shorter epilogue leaves the SM's other
// CTA its shared-memory-bound mainloop alone for longer (the 96/128/192-channel blocks 2-3%
// faster, the final step 14%); the one-CTA-per-SM BN = 256 tiles were 11% slower with it.
template <int PASSES, int EPI, bool PACK>
__device__ __forceinline__ void epilogue4(const ConvArgs &a, const EpiParams &q, float (&v)[4],
                                          const float4 &xr, size_t row, int c) {
    const size_t off = row * (size_t)a.c_out + c;
    if (PACK) {  // two-wide FP32 adds: the same per-lane additions
        const float2 b01 = __fadd2_rn(make_float2(v[0], v[1]), make_float2(q.bias[0], q.bias[1]));
        const float2 b23 = __fadd2_rn(make_float2(v[2], v[3]), make_float2(q.bias[2], q.bias[3]));
        v[0] = b01.x; v[1] = b01.y; v[2] = b23.x; v[3] = b23.y;
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] += q.bias[i];
    }
    if (EPI == kEpiScaleResidual) {  // x = (W h + b) * gamma + x  (run_convnext order)
        const float r[4] = {xr.x, xr.y, xr.z, xr.w};
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = v[i] * q.p1[i] + r[i];
        store4(a.x + off, v[0], v[1], v[2], v[3]);
        return;
    }
    if (EPI == kEpiResidual) {
        if (PACK) {
            const float2 r01 = __fadd2_rn(make_float2(v[0], v[1]), make_float2(xr.x, xr.y));
            const float2 r23 = __fadd2_rn(make_float2(v[2], v[3]), make_float2(xr.z, xr.w));
            v[0] = r01.x; v[1] = r01.y; v[2] = r23.x; v[3] = r23.y;
        } else {
            v[0] += xr.x; v[1] += xr.y; v[2] += xr.z; v[3] += xr.w;
        }
        store4(a.x + off, v[0], v[1], v[2], v[3]);
        if (a.ea == nullptr) return;
    }
    if (EPI == kEpiStoreSnake) {
        store4(a.x + off, v[0], v[1], v[2], v[3]);
        if (a.ea == nullptr) return;
    }
    float hi[4];
    if (PACK && EPI != kEpiGelu) {
#pragma unroll
        for (int i = 0; i < 4; i += 2) {
            const float2 r = snake2(make_float2(v[i], v[i + 1]), make_float2(q.p1[i], q.p1[i + 1]),
                                    make_float2(q.p2[i], q.p2[i + 1]));
            v[i] = r.x;
            v[i + 1] = r.y;
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        if (EPI == kEpiGelu)
            v[i] = 0.5f * v[i] * (1.0f + erff(v[i] * 0.7071067811865475f));  // voc_gelu
        else if (!PACK)
            v[i] = snake1(v[i], q.p1[i], q.p2[i]);
        hi[i] = umma::tf32_round(v[i]);
    }
    store4(a.out_hi + off, hi[0], hi[1], hi[2], hi[3]);
    if (PASSES == 3)
        if (PACK) {
            const float2 l01 = __fadd2_rn(make_float2(v[0], v[1]), make_float2(-hi[0], -hi[1]));
            const float2 l23 = __fadd2_rn(make_float2(v[2], v[3]), make_float2(-hi[2], -hi[3]));
            store4(a.out_lo + off, l01.x, l01.y, l23.x, l23.y);
        } else {
            store4(a.out_lo + off, v[0] - hi[0], v[1] - hi[1], v[2] - hi[2], v[3] - hi[3]);
        }
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
// then lo taps). Grid: ceil(T / 128) x (c_out / BN) x phases x batch tiles, one dimension,
// times `splits` when a GEMM has too few tiles to fill the SMs (a short sequence: the
// pre-transformer's 500-row linears make 8-48 tiles). Split-K runs the `splits` CTAs of a
// tile as one cluster, each over a contiguous 1/splits of the K chunks; each writes its F32
// partial tile into its own (then idle) operand ring, and after a cluster barrier the CTA
// of rank r sums rows/columns unit r of every CTA's partial through distributed shared
// memory in rank order 0..splits-1 (deterministic, no global workspace, no waits on
// flags) and runs the epilogue for them.
template <int BN, int PASSES, int EPI, bool SPLITK>
__global__ void __launch_bounds__(kThreads, (BN <= 128 ? 2 : 1))
conv_umma_kernel(const __grid_constant__ CUtensorMap act_map,
                 const __grid_constant__ CUtensorMap w_map, const ConvArgs a) {
    using L = Tile<BN, PASSES>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 64-byte swizzled tiles need 512-byte alignment; the declaration asks for 1 KiB. A base
    // that is not aligned makes the CTA report LAI_DEVERR_SMEM_ALIGN and do nothing.
    if (reinterpret_cast<uintptr_t>(smem_raw) & 1023) {
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, LAI_DEVERR_SMEM_ALIGN);
        return;
    }
    uint8_t *tiles = smem_raw;
    float *epi_buf = reinterpret_cast<float *>(tiles);  // reused after the last MMA
    uint64_t *full = reinterpret_cast<uint64_t *>(tiles + L::kRing);
    uint64_t *empty = full + L::kStages;
    uint64_t *acc_full = empty + L::kStages;  // [2]: chunk ready in buffer b
    uint64_t *acc_empty = acc_full + 2;       // [2]: buffer b drained
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    // split-K: the cluster's CTAs share one tile; S = cluster size, split = rank in it
    const int S = SPLITK ? (int)cooperative_groups::this_cluster().num_blocks() : 1;
    const int split = SPLITK ? (int)cooperative_groups::this_cluster().block_rank() : 0;
    // Tile order (fastest first): output-channel tile, phase, time tile, batch. The CTAs
    // that read the same input rows (every channel tile and phase of one time tile) run
    // side by side, so an input larger than L2 comes from HBM once, not once per channel
    // tile or phase.
    const int P = a.phases > 1 ? a.phases : 1;
    const int n_nt = a.c_out / BN, n_tt = (a.T + kBM - 1) / kBM;
    int rest = SPLITK ? (int)(blockIdx.x / (unsigned)S) : (int)blockIdx.x;
    const int nt = rest % n_nt;
    rest /= n_nt;
    const int phase = rest % P;
    rest /= P;
    const int t0 = (rest % n_tt) * kBM, n0 = nt * BN;
    const int b = rest / n_tt;
    // global output row of GEMM row t, or -1 when it has none
    auto out_row = [&](int t) -> int64_t {
        if (t >= a.T) return -1;
        if (P == 1) return (int64_t)b * a.T + t;
        if (t < a.row_trim) return -1;
        return (int64_t)b * a.T_out + (int64_t)(t - a.row_trim) * P + phase;
    };
    const int kblocks = a.c_in / kBK;
    const int n_iter_all = a.taps * kblocks;
    const int n_chunks_all = (n_iter_all + L::kChunk - 1) / L::kChunk;
    // this CTA's contiguous share of the K chunks: iterations [it0, it0 + n_iter)
    const int c_lo = SPLITK ? (int)((int64_t)split * n_chunks_all / S) : 0;
    const int c_hi = SPLITK ? (int)((int64_t)(split + 1) * n_chunks_all / S) : n_chunks_all;
    const int it0 = SPLITK ? c_lo * L::kChunk : 0;
    const int n_iter = SPLITK ? min(n_iter_all, c_hi * L::kChunk) - it0 : n_iter_all;
    const int n_chunks = SPLITK ? c_hi - c_lo : n_chunks_all;

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
                const int tap = (it0 + it) / kblocks, kb = (it0 + it) - tap * kblocks;
                const int c = kb * kBK;
                const int row = t0 - (a.taps - 1 - tap) * a.dilation;
                uint8_t *st = tiles + s * L::kStage;
                bulk::mbar_arrive_expect_tx(&full[s], L::kStage);
                umma::tma_load_4d(st, &act_map, c, row, b, 0, &full[s]);
                umma::tma_load_3d(st + L::kA, &w_map, c, n0, phase * a.taps + tap, &full[s]);
                if (PASSES == 3) {
                    umma::tma_load_4d(st + L::kA + L::kB, &act_map, c, row, b, 1, &full[s]);
                    umma::tma_load_3d(st + 2 * L::kA + L::kB, &w_map, c, n0,
                                      (P + phase) * a.taps + tap,
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
                const int j = it / L::kChunk;
                const bool first = it - j * L::kChunk == 0;
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
                if (it - j * L::kChunk == L::kChunk - 1 || it == n_iter - 1)
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
        // Split-K: every CTA of the cluster writes its partial tile into its own ring; then
        // rank r finishes rows [r * 128 / S, (r + 1) * 128 / S) of the tile with all 256
        // drain threads (float4 items, partials summed in rank order 0..S-1, the same
        // epilogue4 per item) and skips the per-warp epilogue below.
        bool mine = true;
        if (SPLITK) {
            namespace cg = cooperative_groups;
            cg::cluster_group cluster = cg::this_cluster();
            float *part = reinterpret_cast<float *>(tiles);  // the ring: every MMA has completed
            if (ok) {
                const int row = q * 32 + lane;
#pragma unroll
                for (int i = 0; i < L::kHalf; i += 4)
                    *reinterpret_cast<float4 *>(part + row * L::kPartPitch + half * L::kHalf +
                                                i) = make_float4(sum[i], sum[i + 1], sum[i + 2],
                                                                 sum[i + 3]);
            }
            cluster.sync();  // every partial written (release / acquire across the cluster)
            mine = false;
            const int rows_per = kBM / S, n4 = rows_per * (BN / 4);
            const int row_lo = split * rows_per;
            for (int i = (int)threadIdx.x - 64; ok && i < n4; i += 32 * kEpiWarps) {
                const int rr = i / (BN / 4), c4 = (i - rr * (BN / 4)) * 4;
                const int row = row_lo + rr;
                const int64_t orow = out_row(t0 + row);
                float v[4] = {0.f, 0.f, 0.f, 0.f};
                for (int r = 0; r < S; r++) {
                    const float4 pv = *reinterpret_cast<const float4 *>(
                        cluster.map_shared_rank(part, r) + row * L::kPartPitch + c4);
                    v[0] += pv.x;
                    v[1] += pv.y;
                    v[2] += pv.z;
                    v[3] += pv.w;
                }
                if (orow < 0) continue;
                const int c = n0 + c4;
                const EpiParams prm = epi_params<EPI>(a, c);
                float4 xr = make_float4(0.f, 0.f, 0.f, 0.f);
                if (EPI == kEpiResidual || EPI == kEpiScaleResidual)
                    xr = *reinterpret_cast<const float4 *>(a.x + (size_t)orow * a.c_out + c);
                epilogue4<PASSES, EPI, (BN <= 128)>(a, prm, v, xr, (size_t)orow, c);
            }
            cluster.sync();  // no CTA exits while its partial is still being read
        }
        if (ok && mine) {
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
                const EpiParams prm = epi_params<EPI>(a, c);
#pragma unroll
                for (int i = 0; i < GW; i++) buf[lane * kEpiPitch + i] = sum[g * GW + i];
                __syncwarp();
                constexpr int PB = NP < 4 ? NP : 4;  // passes whose residual loads fly together
#pragma unroll
                for (int p0 = 0; p0 < NP; p0 += PB) {
                    float4 xr[PB];
                    if (EPI == kEpiResidual || EPI == kEpiScaleResidual) {
#pragma unroll
                        for (int p = 0; p < PB; p++) {
                            const int64_t orow = out_row(row0 + (p0 + p) * RPP + r_off);
                            xr[p] = orow >= 0 ? *reinterpret_cast<const float4 *>(
                                                    a.x + (size_t)orow * a.c_out + c)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                        }
                    }
#pragma unroll
                    for (int p = 0; p < PB; p++) {
                        const int r = (p0 + p) * RPP + r_off;
                        float v[4];
#pragma unroll
                        for (int i = 0; i < 4; i++) v[i] = buf[r * kEpiPitch + c4 + i];
                        const int64_t orow = out_row(row0 + r);
                        if (orow >= 0)
                            epilogue4<PASSES, EPI, (BN <= 128)>(
                                a, prm, v,
                                EPI == kEpiResidual || EPI == kEpiScaleResidual ? xr[p] : xr[0],
                                (size_t)orow, c);
                    }
                }
                __syncwarp();
            }
        }
    }
    if (SPLITK && warp < 2) {  // the producer and MMA warps join the drain warps' two barriers
        cooperative_groups::this_cluster().sync();
        cooperative_groups::this_cluster().sync();
    }
    if (!ok && a.err) atomicOr(a.err, LAI_DEVERR_TIMEOUT);
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tmem, L::kTmemCols);
    }
}

// ---- host side: tensor maps and launches ------------------------------------------

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

// SMs of the current device (cached per device; 148 on B200).
int sm_count() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) ==
                                  cudaSuccess && n > 0
                          ? n
                          : 148;
    }
    return cached[dev];
}

int pick_bn(int c_out) {
    if (c_out <= 384) {  // narrow outputs: tiles that fit two CTAs per SM
        for (int bn : {128, 96, 64, 32})
            if (c_out % bn == 0) return bn;
    }
    for (int bn : {256, 192, 128, 96, 64, 32})
        if (c_out % bn == 0) return bn;
    return 0;
}

template <int BN, int PASSES, int EPI>
int launch_conv_t(const CUtensorMap &am, const CUtensorMap &wm, const ConvArgs &a, int batch,
                  cudaStream_t st) {
    using L = Tile<BN, PASSES>;
    auto kern = conv_umma_kernel<BN, PASSES, EPI, false>;
    auto kern_split = conv_umma_kernel<BN, PASSES, EPI, true>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L::kSmem) !=
        cudaSuccess)
        return LAI_ERR_CUDA;
    const unsigned phases = a.phases > 1 ? (unsigned)a.phases : 1u;
    const long long tiles = (long long)((a.T + kBM - 1) / kBM) * (a.c_out / BN) * phases * batch;
    if (tiles > 0x7fffffffLL) return LAI_ERR_TOOBIG;
    // Split-K while the grid stays within one wave of resident CTAs and every split keeps
    // at least two K chunks (64 input channels).
    const int chunks = (a.taps * (a.c_in / kBK) + L::kChunk - 1) / L::kChunk;
    const long long slots = (long long)L::kMinBlocks * sm_count();
    int S = 1;
    while (S < 8 && tiles * 2 * S <= slots && chunks / (2 * S) >= 2) S *= 2;
    if (S == 1) {
        kern<<<(unsigned)tiles, kThreads, L::kSmem, st>>>(am, wm, a);
        return launch_status();
    }
    if (cudaFuncSetAttribute(kern_split, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)L::kSmem) != cudaSuccess)
        return LAI_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(tiles * S));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = L::kSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern_split, am, wm, a) != cudaSuccess) return LAI_ERR_CUDA;
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

template <int EPI>
int launch_conv(int passes, const CUtensorMap &am, const CUtensorMap &wm, const ConvArgs &a,
                int batch, cudaStream_t st) {
    const int bn = pick_bn(a.c_out);
    return passes == 3 ? launch_conv_p<3, EPI>(bn, am, wm, a, batch, st)
                       : launch_conv_p<1, EPI>(bn, am, wm, a, batch, st);
}

}  // namespace
}  // namespace lai

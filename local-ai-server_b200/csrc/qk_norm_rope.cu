// qk_norm_rope.cu - fused per-head q/k RMSNorm + NeoX RoPE, and the RoPE table.
//
// Reference semantics: qwen_rms_norm_per_head(q|k, w, seq, heads, hd, eps) then
// qwen_apply_rope_neox(q|k, cos, sin, seq, heads, hd), as talker_prefill calls them
// (src/tts_native.c:562-568); RoPE formula tools/verify_xfmr.py:49-53; table rows
// hold cos/sin with duplicated halves (src/tts_native.c:402-412).
//
// Roofline: HBM. Algorithmic bytes per token: 2 * (n_q + n_kv) * hd * s (q and k
// read once, written once in place); the [hd] weights and the table rows are
// shared (L1/L2-resident) and not counted.
//
// Kernels. BF16 with hd=128 and the Qwen3 head layout (16 q / 8 kv heads, every Qwen3
// decoder shape) runs qk_reg_kernel: one warp per token, the token's rows held in
// registers; other head counts run qk_stream_kernel, a persistent kernel whose warps
// each stream single tokens through their own shared-memory stages filled by bulk
// async copies. Both share the per-head arithmetic and are used for every batch size,
// so a token's result never depends on the batch it arrives in. FP32 and hd=64/256 run
// qk_warp_kernel: one warp owns one (token, q-or-k) segment; a head of hd elements
// spans LPH = hd*s/16 lanes, each lane one 16-byte vector, all of the segment's
// loads issued before any arithmetic; the per-head sum of squares is an xor-shuffle
// tree over the LPH lanes and the RoPE partner (d <-> d + hd/2) sits in lane ^ LPH/2.
// The FP32 path uses separately rounded products (no contraction), so with
// identical inputs it reproduces the reference's scalar C RoPE bit for bit.
// Anything else (odd head counts per warp, unaligned rows) runs qk_generic_kernel.
#include "bulk_copy.cuh"
#include "lai_common.cuh"

#include <math.h>

namespace lai {
namespace {

constexpr int kItemsPerCta = 8;  // warps per CTA, one (token, segment) each
constexpr int kMaxSlots = 8;     // 16-byte loads in flight per lane per pass

__device__ __forceinline__ float rope_first(float own, float partner, float c, float s) {
    return __fsub_rn(__fmul_rn(own, c), __fmul_rn(partner, s));  // x1*c - x2*s
}
__device__ __forceinline__ float rope_second(float own, float partner, float c, float s) {
    return __fadd_rn(__fmul_rn(partner, s), __fmul_rn(own, c));  // x1*s + x2*c
}

template <typename T, int HD>
__global__ void __launch_bounds__(kItemsPerCta * 32)
qk_warp_kernel(T *q, T *k, const float *__restrict__ wq, const float *__restrict__ wk,
               const float *__restrict__ cos_t, const float *__restrict__ sin_t,
               const int32_t *__restrict__ pos, int64_t table_rows, int64_t rows, int nq,
               int nkv, float eps, int *err) {
    constexpr int E = Elt<T>::N;
    constexpr int LPH = HD * (int)sizeof(T) / 16;  // lanes per head
    constexpr int HL = LPH / 2;
    static_assert(LPH >= 2 && LPH <= 32 && (32 % LPH) == 0, "head must span 2..32 lanes");

    const int lane = threadIdx.x & 31;
    const int nseg = k ? 2 : 1;
    const int64_t item = (int64_t)blockIdx.x * kItemsPerCta + (threadIdx.x >> 5);
    if (item >= rows * nseg) return;
    const int64_t row = nseg == 2 ? (item >> 1) : item;
    const int seg = nseg == 2 ? (int)(item & 1) : 0;

    const int heads = seg == 0 ? nq : nkv;
    T *base = seg == 0 ? q + (size_t)row * nq * HD : k + (size_t)row * nkv * HD;
    const float *w = seg == 0 ? wq : wk;
    const bool rope = cos_t != nullptr;

    int64_t p = pos ? (int64_t)pos[row] : row;
    if (rope && (p < 0 || p >= table_rows)) {
        if (lane == 0 && err && seg == 0) atomicOr(err, LAI_DEVERR_POSITION);
        return;
    }

    const int hl = lane % LPH;
    const int c0 = hl * E;  // first column of this lane within its head
    const bool first = hl < HL;
    float wv[E], cs[E], sn[E];
    if (w) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            float4 t = ld_f4(w + c0 + e);
            wv[e] = t.x; wv[e + 1] = t.y; wv[e + 2] = t.z; wv[e + 3] = t.w;
        }
    }
    if (rope) {
#pragma unroll
        for (int e = 0; e < E; e += 4) {
            float4 a = ld_f4(cos_t + (size_t)p * HD + c0 + e);
            float4 b = ld_f4(sin_t + (size_t)p * HD + c0 + e);
            cs[e] = a.x; cs[e + 1] = a.y; cs[e + 2] = a.z; cs[e + 3] = a.w;
            sn[e] = b.x; sn[e + 1] = b.y; sn[e + 2] = b.z; sn[e + 3] = b.w;
        }
    }

    const int slots = heads * LPH / 32;
    for (int s0 = 0; s0 < slots; s0 += kMaxSlots) {
        uint4 v[kMaxSlots];
#pragma unroll
        for (int j = 0; j < kMaxSlots; j++)
            if (s0 + j < slots) v[j] = ld_stream(base + ((size_t)(s0 + j) * 32 + lane) * E);
#pragma unroll
        for (int j = 0; j < kMaxSlots; j++) {
            if (s0 + j >= slots) break;  // warp-uniform
            float a[E];
            unpack<T>(v[j], a);
            if (w) {
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < E; e++) ss = fmaf(a[e], a[e], ss);
                ss = group_sum<LPH>(ss);
                const float inv = 1.0f / sqrtf(ss / (float)HD + eps);
#pragma unroll
                for (int e = 0; e < E; e++) a[e] = __fmul_rn(__fmul_rn(a[e], inv), wv[e]);
            }
            if (rope) {
#pragma unroll
                for (int e = 0; e < E; e++) {
                    const float pa = __shfl_xor_sync(0xffffffffu, a[e], HL);
                    a[e] = first ? rope_first(a[e], pa, cs[e], sn[e])
                                 : rope_second(a[e], pa, cs[e], sn[e]);
                }
            }
            st_vec(base + ((size_t)(s0 + j) * 32 + lane) * E, pack<T>(a));
        }
    }
}

// ---- BF16 hd=128 kernels: shared per-head arithmetic -----------------------------
//
// A quarter-warp (8 lanes) holds one head; a lane owns elements d0..d0+7 of the first
// half (d0 = 8 * (lane % 8)) and their RoPE partners 64+d0..64+d0+7, one 16-byte access
// each, so the rotation needs no shuffle and the sum of squares is a 3-step xor tree.
// Arithmetic runs on packed two-wide FP32 (FMUL2 / FFMA2). qk_stream_kernel (large
// batches) and qk_reg_kernel (small batches) share head_math, so a token's bits do not
// depend on which of them ran or on the batch it arrived in.
__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t w) { return make_float2(bf16_lo(w), bf16_hi(w)); }
__device__ __forceinline__ uint32_t f2_to_bf16x2(float2 v) { return pack_bf16x2(v.x, v.y); }

struct RopeRow {
    float2 cl[4], ch[4], sl[4], sh[4];  // cos / sin of d0..d0+7 and 64+d0..64+d0+7
};

// All eight lanes of every quarter-warp must call it (3 xor shuffles).
__device__ __forceinline__ void head_math(uint4 &lo, uint4 &hi, const float2 (&w)[8], bool norm,
                                          bool rope, const RopeRow &t, float eps) {
    float2 a[4] = {bf16x2_to_f2(lo.x), bf16x2_to_f2(lo.y), bf16x2_to_f2(lo.z), bf16x2_to_f2(lo.w)};
    float2 b[4] = {bf16x2_to_f2(hi.x), bf16x2_to_f2(hi.y), bf16x2_to_f2(hi.z), bf16x2_to_f2(hi.w)};
    if (norm) {
        float2 s0 = __fmul2_rn(a[0], a[0]), s1 = __fmul2_rn(b[0], b[0]);
#pragma unroll
        for (int e = 1; e < 4; e++) {
            s0 = __ffma2_rn(a[e], a[e], s0);
            s1 = __ffma2_rn(b[e], b[e], s1);
        }
        float ss = (s0.x + s0.y) + (s1.x + s1.y);
        ss += __shfl_xor_sync(0xffffffffu, ss, 4);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        // BF16 output keeps 8 significant bits, so the approximate reciprocal square
        // root and the packed products (ulp-level departures from the separately
        // rounded reference form) cannot show in the result.
        const float inv = rsqrtf(ss * (1.0f / 128) + eps);
        const float2 inv2 = make_float2(inv, inv);
#pragma unroll
        for (int e = 0; e < 4; e++) {
            a[e] = __fmul2_rn(__fmul2_rn(a[e], inv2), w[e]);
            b[e] = __fmul2_rn(__fmul2_rn(b[e], inv2), w[4 + e]);
        }
    }
    if (rope) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float2 x1 = a[e], x2 = b[e];
            const float2 nx2 = make_float2(-x2.x, -x2.y);
            a[e] = __ffma2_rn(nx2, t.sl[e], __fmul2_rn(x1, t.cl[e]));  // x1*c - x2*s
            b[e] = __ffma2_rn(x1, t.sh[e], __fmul2_rn(x2, t.ch[e]));   // x1*s + x2*c
        }
    }
    lo = make_uint4(f2_to_bf16x2(a[0]), f2_to_bf16x2(a[1]), f2_to_bf16x2(a[2]), f2_to_bf16x2(a[3]));
    hi = make_uint4(f2_to_bf16x2(b[0]), f2_to_bf16x2(b[1]), f2_to_bf16x2(b[2]), f2_to_bf16x2(b[3]));
}

// A lane's cos / sin values from a table row (shared or global memory).
__device__ __forceinline__ void load_rope_row(RopeRow &t, const float *c, const float *s, int d0) {
    const float4 c0 = *reinterpret_cast<const float4 *>(c + d0);
    const float4 c1 = *reinterpret_cast<const float4 *>(c + d0 + 4);
    const float4 c2 = *reinterpret_cast<const float4 *>(c + 64 + d0);
    const float4 c3 = *reinterpret_cast<const float4 *>(c + 64 + d0 + 4);
    const float4 s0 = *reinterpret_cast<const float4 *>(s + d0);
    const float4 s1 = *reinterpret_cast<const float4 *>(s + d0 + 4);
    const float4 s2 = *reinterpret_cast<const float4 *>(s + 64 + d0);
    const float4 s3 = *reinterpret_cast<const float4 *>(s + 64 + d0 + 4);
    t.cl[0] = make_float2(c0.x, c0.y); t.cl[1] = make_float2(c0.z, c0.w);
    t.cl[2] = make_float2(c1.x, c1.y); t.cl[3] = make_float2(c1.z, c1.w);
    t.ch[0] = make_float2(c2.x, c2.y); t.ch[1] = make_float2(c2.z, c2.w);
    t.ch[2] = make_float2(c3.x, c3.y); t.ch[3] = make_float2(c3.z, c3.w);
    t.sl[0] = make_float2(s0.x, s0.y); t.sl[1] = make_float2(s0.z, s0.w);
    t.sl[2] = make_float2(s1.x, s1.y); t.sl[3] = make_float2(s1.z, s1.w);
    t.sh[0] = make_float2(s2.x, s2.y); t.sh[1] = make_float2(s2.z, s2.w);
    t.sh[2] = make_float2(s3.x, s3.y); t.sh[3] = make_float2(s3.z, s3.w);
}

// A lane's weights: w[0..3] = pairs of d0..d0+7, w[4..7] = pairs of 64+d0..64+d0+7.
__device__ __forceinline__ void load_head_weights(float2 (&w)[8], const float *src, int d0) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
        w[e] = src ? make_float2(src[d0 + 2 * e], src[d0 + 2 * e + 1]) : make_float2(1.f, 1.f);
        w[4 + e] = src ? make_float2(src[64 + d0 + 2 * e], src[64 + d0 + 2 * e + 1])
                       : make_float2(1.f, 1.f);
    }
}

// One token's heads (q or k) in shared memory: 4 heads per pass.
// P > 0: the pass count is known at compile time (fully unrolled); P == 0: any count.
template <int P>
__device__ __forceinline__ void stream_heads(unsigned char *base, int nheads, int hsub, int d0,
                                             const float2 (&w)[8], bool norm, bool rope,
                                             const RopeRow &t, float eps) {
    const int passes = P > 0 ? P : (nheads + 3) / 4;
#pragma unroll
    for (int j = 0; j < (P > 0 ? P : passes); j++) {
        const int h = hsub + 4 * j;
        const bool hv = P > 0 || h < nheads;
        uint16_t *hp = reinterpret_cast<uint16_t *>(base) + (size_t)h * 128;
        uint4 lo = hv ? *reinterpret_cast<const uint4 *>(hp + d0) : make_uint4(0, 0, 0, 0);
        uint4 hi = hv ? *reinterpret_cast<const uint4 *>(hp + 64 + d0) : make_uint4(0, 0, 0, 0);
        head_math(lo, hi, w, norm, rope, t, eps);
        if (hv) {
            *reinterpret_cast<uint4 *>(hp + d0) = lo;
            *reinterpret_cast<uint4 *>(hp + 64 + d0) = hi;
        }
    }
}

// ---- streaming kernel: an independent bulk-copy pipeline per warp -------------------
//
// Any head count (qk_reg_kernel covers the Qwen3 layout, whose rows fit in registers).
// One CTA per SM, up to kStreamWarps warps, no CTA-wide barrier after set-up: every
// warp runs its own pipeline over kStreamStages single-token stages. A stage holds the
// token's q row, its k row and (with RoPE) its cos and sin table rows, fetched by bulk
// async copies that complete on the stage's mbarrier; the warp normalises and rotates
// the heads in place in shared memory and writes the q and k rows back with two bulk
// stores. Warp w of the grid takes tokens w, w + W_total, ... After issuing token i's
// stores the warp refills the stage of token i - 1 (whose stores have been read out by
// then) with token i - 1 + S, so a token's stores drain while the next token loads and
// the warp never waits for a store. Memory parallelism comes from the 16 independent
// warps per SM (16 x 2 stages x 7 KB fill the shared memory): refilling a stage as soon
// as its own store has been read out (waiting on it) measured 15% slower, and 3-stage
// pipelines at 8-10 warps 5-10% slower. Positions are fetched 32 tokens at a time (lane
// j holds the position of the warp's token 32b + j) one block ahead, so the issuing
// lane never waits on them.
constexpr int kStreamWarps = 16;
constexpr int kStreamStages = 2;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any real copy

// Shared memory of qk_stream_kernel: per warp S mbarriers and S validity words, then
// per warp S stages of one token's q and k rows (+ its cos / sin rows with RoPE).
__host__ __device__ inline size_t stream_header_bytes(int warps) {
    return ((size_t)warps * kStreamStages * 12 + 127) / 128 * 128;
}
__host__ __device__ inline size_t stream_stage_bytes(int nq, int nkv, bool rope) {
    return (size_t)(nq + nkv) * 256 + (rope ? 1024 : 0);
}

template <int QP, int KP>  // QP / KP: q / k passes of 4 heads (0: runtime count)
__global__ void __launch_bounds__(kStreamWarps * 32, 1)
qk_stream_kernel(uint16_t *q, uint16_t *k, const float *__restrict__ wq,
                 const float *__restrict__ wk, const float *__restrict__ cos_t,
                 const float *__restrict__ sin_t, const int32_t *__restrict__ pos,
                 int64_t table_rows, int64_t rows, int nq, int nkv, float eps, int *err) {
    constexpr int S = kStreamStages;
    extern __shared__ __align__(128) unsigned char smem[];
    const int W = blockDim.x >> 5;  // warps of this launch (fewer for wide head layouts)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool rope = cos_t != nullptr;
    const uint32_t q_tok = (uint32_t)nq * 256u, k_tok = (uint32_t)nkv * 256u;
    const uint32_t stage_bytes = (uint32_t)stream_stage_bytes(nq, nkv, rope);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem) + warp * S;
    int *valid_slot = reinterpret_cast<int *>(smem + W * S * 8) + warp * S;
    unsigned char *ring = smem + stream_header_bytes(W) + (size_t)warp * S * stage_bytes;

    const int64_t wg = (int64_t)blockIdx.x * W + warp, nw = (int64_t)gridDim.x * W;
    const int64_t my_n = wg < rows ? (rows - 1 - wg) / nw + 1 : 0;
    if (my_n == 0) return;  // the whole warp; nothing below synchronises across warps
    if (lane == 0) {
        for (int s = 0; s < S; s++) bulk::mbar_init(&full[s], 1);
        bulk::fence_barrier_init();
    }
    __syncwarp();

    // positions of the warp's items, 32 per register block, one block ahead
    auto load_pos_block = [&](int64_t b) -> int64_t {
        const int64_t i = b * 32 + lane;
        if (i >= my_n) return 0;
        const int64_t r = wg + i * nw;
        return pos ? (int64_t)pos[r] : r;
    };
    int64_t pblk = load_pos_block(0), pnxt = load_pos_block(1), cur_b = 0;
    auto pos_of = [&](int64_t i) -> int64_t {  // warp-collective; i never decreases
        while (cur_b < (i >> 5)) {
            pblk = pnxt;
            cur_b++;
            pnxt = load_pos_block(cur_b + 1);
        }
        return __shfl_sync(0xffffffffu, pblk, (int)(i & 31));
    };
    auto issue = [&](int64_t i, int64_t p) {  // lane 0: item i into stage i % S
        const int s = (int)(i % S);
        const int64_t r = wg + i * nw;
        unsigned char *st = ring + (size_t)s * stage_bytes;
        const bool ok = !rope || (p >= 0 && p < table_rows);
        valid_slot[s] = ok ? 1 : 0;  // read by the warp after the stage's barrier completes
        bulk::mbar_arrive_expect_tx(&full[s], stage_bytes);
        bulk::load(st, q + (size_t)r * nq * 128, q_tok, &full[s]);
        if (k_tok) bulk::load(st + q_tok, k + (size_t)r * nkv * 128, k_tok, &full[s]);
        if (rope) {
            const int64_t pr = ok ? p : 0;  // an out-of-range row loads row 0 and is skipped
            bulk::load(st + q_tok + k_tok, cos_t + (size_t)pr * 128, 512, &full[s]);
            bulk::load(st + q_tok + k_tok + 512, sin_t + (size_t)pr * 128, 512, &full[s]);
        }
    };

    int64_t issued = 0;
    for (; issued < S && issued < my_n; issued++) {
        const int64_t p = pos_of(issued);
        if (lane == 0) issue(issued, p);
    }

    const int hsub = lane >> 3;     // head within a pass of 4
    const int d0 = (lane & 7) * 8;  // elements d0..d0+7 and 64+d0..64+d0+7
    float2 wq2[8], wk2[8];
    load_head_weights(wq2, wq, d0);
    load_head_weights(wk2, wk, d0);

    bool stopped = false;
    int64_t i = 0;
    for (; i < my_n; i++) {
        const int s = (int)(i % S);
        const uint32_t parity = (uint32_t)((i / S) & 1);
        unsigned char *st = ring + (size_t)s * stage_bytes;
        if (!__all_sync(0xffffffffu, bulk::mbar_wait_bounded(&full[s], parity, kWaitLimitNs))) {
            stopped = true;
            break;
        }
        if (valid_slot[s]) {
            RopeRow t = {};
            if (rope) {
                const float *ct = reinterpret_cast<const float *>(st + q_tok + k_tok);
                load_rope_row(t, ct, ct + 128, d0);
            }
            stream_heads<QP>(st, nq, hsub, d0, wq2, wq != nullptr, rope, t, eps);
            if (k_tok) stream_heads<KP>(st + q_tok, nkv, hsub, d0, wk2, wk != nullptr, rope, t, eps);
        } else if (lane == 0 && err) {
            atomicOr(err, LAI_DEVERR_POSITION);  // row left as it was (stored back unchanged)
        }
        bulk::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            const int64_t r = wg + i * nw;
            bulk::store(q + (size_t)r * nq * 128, st, q_tok);
            if (k_tok) bulk::store(k + (size_t)r * nkv * 128, st + q_tok, k_tok);
            bulk::commit();
        }
        // refill the previous item's stage: its store was committed one iteration ago
        if (i >= 1 && issued < my_n) {
            const int64_t p = pos_of(issued);
            if (lane == 0) {
                bulk::wait_read<1>();
                issue(issued, p);
            }
            issued++;
        }
    }
    if (lane == 0) {
        bulk::wait_all();
        if (stopped) {
            if (err) atomicOr(err, LAI_DEVERR_TIMEOUT);
            // drain loads still in flight into this warp's stages, each bounded
            for (int64_t j = i; j < issued; j++)
                bulk::mbar_wait_bounded(&full[j % S], (uint32_t)((j / S) & 1), kWaitLimitNs);
        }
    }
}

// ---- Qwen3 head layout: one warp per token straight from global memory -------------
// Every q / k load of the token (12 x 16 bytes per lane for 16 + 8 heads) is issued
// before the position's table row is needed, so a warp keeps 6 KB in flight and the
// ~16 resident warps per SM (126 registers each) keep ~100 KB per SM in flight. Same
// lane mapping and head_math as qk_stream_kernel. Measured against it (same bits, B200,
// 16 q / 8 kv heads): 125 vs 135 us at 65536 tokens (0.98 vs 0.91 of the measured copy
// bandwidth), 3.82 vs 3.97 ms at 2M tokens, 16.5 vs 22.6 us at 8192 and 5.1 vs 5.0 us
// at 512: the shared-memory staging of the stream kernel buys nothing when the whole
// token fits in a warp's registers.
constexpr int kRegWarps = 4;

template <int QP, int KP>  // q / k passes of 4 heads; the token's rows held in registers
__global__ void __launch_bounds__(kRegWarps * 32)
qk_reg_kernel(uint16_t *q, uint16_t *k, const float *__restrict__ wq, const float *__restrict__ wk,
              const float *__restrict__ cos_t, const float *__restrict__ sin_t,
              const int32_t *__restrict__ pos, int64_t table_rows, int64_t rows, float eps,
              int *err) {
    constexpr int NQ = 4 * QP, NKV = 4 * KP;
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)blockIdx.x * kRegWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    pdl_wait_prior();  // launched with programmatic dependent launch: inputs after this
    const bool rope = cos_t != nullptr;
    const int hsub = lane >> 3, d0 = (lane & 7) * 8;
    uint16_t *qr = q + (size_t)row * NQ * 128;
    uint16_t *kr = KP ? k + (size_t)row * NKV * 128 : nullptr;
    uint4 lo[QP + KP], hi[QP + KP];
#pragma unroll
    for (int j = 0; j < QP + KP; j++) {
        const uint16_t *hp = (j < QP ? qr + (size_t)(hsub + 4 * j) * 128
                                     : kr + (size_t)(hsub + 4 * (j - QP)) * 128);
        lo[j] = *reinterpret_cast<const uint4 *>(hp + d0);
        hi[j] = *reinterpret_cast<const uint4 *>(hp + 64 + d0);
    }
    const int64_t p = pos ? (int64_t)pos[row] : row;
    if (rope && (p < 0 || p >= table_rows)) {
        if (lane == 0 && err) atomicOr(err, LAI_DEVERR_POSITION);
        return;  // row left as it was
    }
    RopeRow t = {};
    if (rope) load_rope_row(t, cos_t + (size_t)p * 128, sin_t + (size_t)p * 128, d0);
    float2 w2[8];
    load_head_weights(w2, wq, d0);
#pragma unroll
    for (int j = 0; j < QP; j++) head_math(lo[j], hi[j], w2, wq != nullptr, rope, t, eps);
    if (KP) {
        load_head_weights(w2, wk, d0);
#pragma unroll
        for (int j = QP; j < QP + KP; j++) head_math(lo[j], hi[j], w2, wk != nullptr, rope, t, eps);
    }
#pragma unroll
    for (int j = 0; j < QP + KP; j++) {
        uint16_t *hp = (j < QP ? qr + (size_t)(hsub + 4 * j) * 128
                               : kr + (size_t)(hsub + 4 * (j - QP)) * 128);
        *reinterpret_cast<uint4 *>(hp + d0) = lo[j];
        *reinterpret_cast<uint4 *>(hp + 64 + d0) = hi[j];
    }
    pdl_launch_dependents();
}

// Any even head_dim / alignment / head count: one warp per (token, head).
template <typename T>
__global__ void __launch_bounds__(256)
qk_generic_kernel(T *q, T *k, const float *wq, const float *wk, const float *cos_t,
                  const float *sin_t, const int32_t *pos, int64_t table_rows, int64_t rows,
                  int nq, int nkv, int hd, float eps, int *err) {
    const int lane = threadIdx.x & 31;
    const int nh = nq + (k ? nkv : 0);
    const int64_t item = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= rows * nh) return;
    const int64_t row = item / nh;
    const int h = (int)(item % nh);
    T *xh = h < nq ? q + ((size_t)row * nq + h) * hd : k + ((size_t)row * nkv + (h - nq)) * hd;
    const float *w = h < nq ? wq : wk;
    const bool rope = cos_t != nullptr;
    int64_t p = pos ? (int64_t)pos[row] : row;
    if (rope && (p < 0 || p >= table_rows)) {
        if (lane == 0 && err && h == 0) atomicOr(err, LAI_DEVERR_POSITION);
        return;
    }
    float inv = 1.f;
    if (w) {
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) {
            float a = to_f(xh[d]);
            ss = fmaf(a, a, ss);
        }
        ss = group_sum<32>(ss);
        inv = 1.0f / sqrtf(ss / (float)hd + eps);
    }
    const int half = hd / 2;
    const float *c = rope ? cos_t + (size_t)p * hd : nullptr;
    const float *s = rope ? sin_t + (size_t)p * hd : nullptr;
    for (int d = lane; d < half; d += 32) {
        float x1 = to_f(xh[d]), x2 = to_f(xh[d + half]);
        if (w) {
            x1 = __fmul_rn(__fmul_rn(x1, inv), w[d]);
            x2 = __fmul_rn(__fmul_rn(x2, inv), w[d + half]);
        }
        if (rope) {
            const float r1 = rope_first(x1, x2, c[d], s[d]);
            const float r2 = rope_second(x2, x1, c[d + half], s[d + half]);
            x1 = r1;
            x2 = r2;
        }
        xh[d] = from_f<T>(x1);
        xh[d + half] = from_f<T>(x2);
    }
}

// ---- FP32, hd = 128: one warp per (token, q-or-k) straight from global memory ----------
// The FP32 drop-ins' type. A quarter-warp (8 lanes) per head, lane owns elements d0..d0+7
// (d0 = 8 * (lane % 8)) and their RoPE partners 64+d0..64+d0+7 (four 16-byte loads per head),
// every load of the segment issued before the position's table row is needed. The
// arithmetic is the reference's: the sum of squares in FP32, inv = 1 / sqrtf(ss / hd + eps),
// x * inv * w, and the rotation's products and sums rounded separately (scalar __fmul_rn /
// __fadd_rn, which the compiler never contracts into FMAs), so RoPE alone is bit-exact with
// the reference's scalar C.
// At 65 536 tokens of Qwen3-1.7B shapes: 239 us (1.03 of measured HBM) against 319 us (0.77)
// for qk_warp_kernel (a warp per head, the partner by shuffle). Packed FMUL2 / FADD2 for the
// rotation did not reproduce the reference's bits; the scalar forms below do.
template <int QP, int KP>  // passes of 4 heads for q and k
__global__ void __launch_bounds__(kRegWarps * 32)
qk_reg_f32_kernel(float *q, float *k, const float *__restrict__ wq, const float *__restrict__ wk,
                  const float *__restrict__ cos_t, const float *__restrict__ sin_t,
                  const int32_t *__restrict__ pos, int64_t table_rows, int64_t rows, float eps,
                  int *err) {
    constexpr int PMAX = QP > KP ? QP : KP;
    const int lane = threadIdx.x & 31;
    const int nseg = KP ? 2 : 1;
    const int64_t item = (int64_t)blockIdx.x * kRegWarps + (threadIdx.x >> 5);
    if (item >= rows * nseg) return;
    pdl_wait_prior();  // launched with programmatic dependent launch: inputs after this
    const int64_t row = nseg == 2 ? item >> 1 : item;
    const int seg = nseg == 2 ? (int)(item & 1) : 0;
    const int passes = seg ? KP : QP;
    float *base = seg ? k + (size_t)row * (4 * KP) * 128 : q + (size_t)row * (4 * QP) * 128;
    const float *w = seg ? wk : wq;
    const bool rope = cos_t != nullptr;
    const int hsub = lane >> 3, d0 = (lane & 7) * 8;
    float4 v[PMAX][4];  // per pass: first half d0..d0+3, d0+4..d0+7, partners 64+d0.., 68+d0..
#pragma unroll
    for (int j = 0; j < PMAX; j++) {
        if (j >= passes) break;
        const float *hp = base + (size_t)(hsub + 4 * j) * 128;
        v[j][0] = *reinterpret_cast<const float4 *>(hp + d0);
        v[j][1] = *reinterpret_cast<const float4 *>(hp + d0 + 4);
        v[j][2] = *reinterpret_cast<const float4 *>(hp + 64 + d0);
        v[j][3] = *reinterpret_cast<const float4 *>(hp + 64 + d0 + 4);
    }
    const int64_t p = pos ? (int64_t)pos[row] : row;
    if (rope && (p < 0 || p >= table_rows)) {
        if (lane == 0 && err && seg == 0) atomicOr(err, LAI_DEVERR_POSITION);
        return;  // row left as it was
    }
    RopeRow t = {};
    if (rope) load_rope_row(t, cos_t + (size_t)p * 128, sin_t + (size_t)p * 128, d0);
    float2 w2[8];
    load_head_weights(w2, w, d0);
#pragma unroll
    for (int j = 0; j < PMAX; j++) {
        if (j >= passes) break;  // warp-uniform
        float2 a[4] = {make_float2(v[j][0].x, v[j][0].y), make_float2(v[j][0].z, v[j][0].w),
                       make_float2(v[j][1].x, v[j][1].y), make_float2(v[j][1].z, v[j][1].w)};
        float2 b[4] = {make_float2(v[j][2].x, v[j][2].y), make_float2(v[j][2].z, v[j][2].w),
                       make_float2(v[j][3].x, v[j][3].y), make_float2(v[j][3].z, v[j][3].w)};
        if (w) {
            float2 s0 = __fmul2_rn(a[0], a[0]), s1 = __fmul2_rn(b[0], b[0]);
#pragma unroll
            for (int e = 1; e < 4; e++) {
                s0 = __ffma2_rn(a[e], a[e], s0);
                s1 = __ffma2_rn(b[e], b[e], s1);
            }
            float ss = (s0.x + s0.y) + (s1.x + s1.y);
            ss += __shfl_xor_sync(0xffffffffu, ss, 4);
            ss += __shfl_xor_sync(0xffffffffu, ss, 2);
            ss += __shfl_xor_sync(0xffffffffu, ss, 1);
            const float inv = 1.0f / sqrtf(ss / 128.0f + eps);
            const float2 inv2 = make_float2(inv, inv);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                a[e] = __fmul2_rn(__fmul2_rn(a[e], inv2), w2[e]);
                b[e] = __fmul2_rn(__fmul2_rn(b[e], inv2), w2[4 + e]);
            }
        }
        if (rope) {  // scalar, separately rounded (never contracted): the reference's bits
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float2 x1 = a[e], x2 = b[e];
                a[e] = make_float2(rope_first(x1.x, x2.x, t.cl[e].x, t.sl[e].x),
                                   rope_first(x1.y, x2.y, t.cl[e].y, t.sl[e].y));
                b[e] = make_float2(rope_second(x2.x, x1.x, t.ch[e].x, t.sh[e].x),
                                   rope_second(x2.y, x1.y, t.ch[e].y, t.sh[e].y));
            }
        }
        float *hp = base + (size_t)(hsub + 4 * j) * 128;
        *reinterpret_cast<float4 *>(hp + d0) = make_float4(a[0].x, a[0].y, a[1].x, a[1].y);
        *reinterpret_cast<float4 *>(hp + d0 + 4) = make_float4(a[2].x, a[2].y, a[3].x, a[3].y);
        *reinterpret_cast<float4 *>(hp + 64 + d0) = make_float4(b[0].x, b[0].y, b[1].x, b[1].y);
        *reinterpret_cast<float4 *>(hp + 64 + d0 + 4) = make_float4(b[2].x, b[2].y, b[3].x, b[3].y);
    }
    pdl_launch_dependents();
}

template <typename T, int HD>
bool try_fast(T *q, T *k, const float *wq, const float *wk, const float *cos_t,
              const float *sin_t, const int32_t *pos, int64_t table_rows, int64_t rows, int nq,
              int nkv, float eps, int *err, cudaStream_t s) {
    constexpr int LPH = HD * (int)sizeof(T) / 16;
    if constexpr (LPH > 32) {
        return false;  // a head wider than one warp-wide load: generic kernel
    } else {
        if ((nq * LPH) % 32 != 0 || (k && (nkv * LPH) % 32 != 0)) return false;
        if (!aligned16(q) || (k && !aligned16(k)) || (wq && !aligned16(wq)) ||
            (k && wk && !aligned16(wk)) || (cos_t && (!aligned16(cos_t) || !aligned16(sin_t))))
            return false;
        const int64_t items = rows * (k ? 2 : 1);
        qk_warp_kernel<T, HD><<<grid_for(items, kItemsPerCta), kItemsPerCta * 32, 0, s>>>(
            q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err);
        return true;
    }
}

struct DeviceInfo {
    int sms = 0;
    bool attr_set = false;
};

// BF16, hd = 128: qk_reg_kernel for the Qwen3 head layout (16 q / 8 or 0 kv heads),
// qk_stream_kernel for any other head count (the same per-head bits either way).
// false when neither applies.
bool try_bf16_hd128(uint16_t *q, uint16_t *k, const float *wq, const float *wk,
                    const float *cos_t, const float *sin_t, const int32_t *pos, int64_t table_rows,
                    int64_t rows, int nq, int nkv, float eps, int *err, cudaStream_t s) {
    constexpr size_t kMaxSmem = 227 * 1024;
    const bool rope = cos_t != nullptr;
    if (!aligned16(q) || (k && !aligned16(k)) || (rope && (!aligned16(cos_t) || !aligned16(sin_t))))
        return false;
    const bool qwen = nq == 16 && (nkv == 8 || nkv == 0);
    if (qwen) {
        auto kern = nkv ? qk_reg_kernel<4, 2> : qk_reg_kernel<4, 0>;
        launch_pdl(kern, dim3(grid_for(rows, kRegWarps)), dim3(kRegWarps * 32), 0, s, q, k, wq, wk,
                   cos_t, sin_t, pos, table_rows, rows, eps, err);
        return true;
    }
    // as many warps (up to kStreamWarps per SM) as fit their stages in shared memory
    const size_t per_warp = (size_t)kStreamStages * stream_stage_bytes(nq, nkv, rope);
    int warps = kStreamWarps;
    while (warps > 0 && stream_header_bytes(warps) + warps * per_warp > kMaxSmem) warps--;
    if (warps == 0) return false;
    const size_t smem = stream_header_bytes(warps) + warps * per_warp;
    static DeviceInfo info[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    DeviceInfo &d = info[dev];
    auto kern = qk_stream_kernel<0, 0>;
    if (!d.attr_set) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)kMaxSmem) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        d.attr_set = true;
    }
    const int64_t ctas = (rows + warps - 1) / warps;
    const int64_t cap = (int64_t)d.sms;
    const int64_t grid = ctas < cap ? ctas : cap;
    kern<<<(unsigned)grid, warps * 32, smem, s>>>(q, k, wq, wk, cos_t, sin_t, pos, table_rows,
                                                  rows, nq, nkv, eps, err);
    return true;
}

template <typename T>
int run(T *q, T *k, const float *wq, const float *wk, const float *cos_t, const float *sin_t,
        const int32_t *pos, int64_t table_rows, int64_t rows, int nq, int nkv, int hd, float eps,
        int *err, lai_stream_t stream) {
    if (!q || rows < 0 || nq <= 0 || hd <= 0 || (hd & 1) || (k && nkv <= 0)) return LAI_ERR_INVALID;
    if (cos_t && (!sin_t || table_rows <= 0)) return LAI_ERR_INVALID;
    if (!cos_t && !wq && !wk) return LAI_ERR_INVALID;  // nothing to do is a caller bug
    if (rows == 0) return LAI_OK;
    if (k && overlaps(q, (size_t)rows * nq * hd * sizeof(T), k, (size_t)rows * nkv * hd * sizeof(T)))
        return LAI_ERR_ALIAS;
    cudaStream_t s = as_stream(stream);
    bool done = false;
    if constexpr (sizeof(T) == 2) {
        if (hd == 128) done = try_bf16_hd128(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows,
                                             nq, k ? nkv : 0, eps, err, s);
    }
    if constexpr (sizeof(T) == 4) {
        if (hd == 128 && nq == 16 && (!k || nkv == 8) && aligned16(q) && (!k || aligned16(k)) &&
            (!wq || aligned16(wq)) && (!k || !wk || aligned16(wk)) &&
            (!cos_t || (aligned16(cos_t) && aligned16(sin_t)))) {
            auto kern = k ? qk_reg_f32_kernel<4, 2> : qk_reg_f32_kernel<4, 0>;
            const int64_t items = rows * (k ? 2 : 1);
            launch_pdl(kern, dim3(grid_for(items, kRegWarps)), dim3(kRegWarps * 32), 0, s,
                       reinterpret_cast<float *>(q), reinterpret_cast<float *>(k), wq, wk, cos_t,
                       sin_t, pos, table_rows, rows, eps, err);
            done = true;
        }
    }
    if (!done) switch (hd) {
        case 64: done = try_fast<T, 64>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err, s); break;
        case 128: done = try_fast<T, 128>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err, s); break;
        case 256: done = try_fast<T, 256>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq, nkv, eps, err, s); break;
        default: break;
    }
    if (!done) {
        const int64_t items = rows * (nq + (k ? nkv : 0));
        qk_generic_kernel<T><<<grid_for(items, 8), 256, 0, s>>>(q, k, wq, wk, cos_t, sin_t, pos,
                                                               table_rows, rows, nq, nkv, hd, eps, err);
    }
    return launch_status();
}

// ---- RoPE table -----------------------------------------------------------------
struct InvFreq {
    float f[256];
};

__global__ void __launch_bounds__(256)
rope_table_kernel(float *cos_t, float *sin_t, const int32_t *pos, int64_t n, int hd, InvFreq inv) {
    const int half = hd / 2;
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n * half) return;
    const int64_t i = idx / half;
    const int d = (int)(idx % half);
    const int p = pos ? pos[i] : (int)i;
    const float angle = __fmul_rn((float)p, inv.f[d]);
    const float c = cosf(angle), s = sinf(angle);
    cos_t[i * hd + d] = c;
    cos_t[i * hd + half + d] = c;
    sin_t[i * hd + d] = s;
    sin_t[i * hd + half + d] = s;
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_qk_norm_rope_bf16(lai_bf16 *q, lai_bf16 *k, const float *wq, const float *wk,
                          const float *cos_t, const float *sin_t, const int32_t *pos,
                          int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                          int head_dim, float eps, int *err, lai_stream_t stream) {
    return lai::run<uint16_t>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, n_q_heads,
                              n_kv_heads, head_dim, eps, err, stream);
}

int lai_qk_norm_rope_f32(float *q, float *k, const float *wq, const float *wk,
                         const float *cos_t, const float *sin_t, const int32_t *pos,
                         int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                         int head_dim, float eps, int *err, lai_stream_t stream) {
    return lai::run<float>(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, n_q_heads,
                           n_kv_heads, head_dim, eps, err, stream);
}

int lai_rope_table_f32(float *cos_t, float *sin_t, const int32_t *pos, int64_t n, int head_dim,
                       float theta, lai_stream_t stream) {
    if (!cos_t || !sin_t || n < 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 512)
        return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    lai::InvFreq inv;
    // Host-side, with the host libm, exactly as ensure_rope_cache computes it
    // (src/tts_native.c:383-388), so the device table sees identical frequencies.
    for (int d = 0; d < head_dim / 2; d++)
        inv.f[d] = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
    const int64_t work = n * (head_dim / 2);
    lai::rope_table_kernel<<<lai::grid_for(work, 256), 256, 0, lai::as_stream(stream)>>>(
        cos_t, sin_t, pos, n, head_dim, inv);
    return lai::launch_status();
}

}  // extern "C"

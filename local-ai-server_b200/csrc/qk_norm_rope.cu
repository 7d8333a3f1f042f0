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
// Kernels. BF16 with hd=128 (every Qwen3 decoder shape) runs qk_pipe_kernel: a
// persistent kernel that streams token tiles through a shared-memory ring filled
// by bulk async copies (described at the kernel), used for every batch size so a
// token's result never depends on the batch it arrives in. FP32 and hd=64/256 run
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

// ---- pipelined BF16 hd=128 kernel: bulk async copies through a shared-memory ring ----
//
// Persistent CTAs (2 per SM). A tile is kTileTok consecutive tokens: their q rows
// and their k rows are each one contiguous range, fetched by two bulk copies into
// one of kStages shared-memory stages (completion counted on the stage's mbarrier),
// computed in place in shared memory and written back by two bulk stores; a stage is
// refilled only after its stores have finished reading it. Memory parallelism
// therefore comes from the copy engine, not from registers.
//
// Each CTA runs as two independent groups of 4 warps that take alternate tiles (group g:
// tiles g, g+2, ...; stages g and g+2), each with its own named barrier and its own
// leader thread issuing its loads and stores. One group's barrier, stores and refill then
// overlap the other group's arithmetic; with one CTA-wide barrier per tile (the previous
// form) the whole CTA stalled at every tile boundary and the kernel reached 0.79 of the
// measured copy bandwidth against 0.855 now (same bits out). Work split within a group:
// 8 half-warps, 8/kTileTok per token, a half-warp per head (pipe_heads).
__device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

constexpr int kTileTok = 4;
constexpr int kStages = 4;
constexpr int kPipeThreads = 256;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: far beyond any real copy

// One token's heads (q or k) in shared memory, BF16 hd=128: a half-warp per head,
// lane owns elements d0..d0+3 (first half) and their RoPE partners 64+d0..64+d0+3,
// so the rotation needs no shuffle; the sum of squares is a 4-step xor tree. The
// trip count is the same in every half-warp (shuffles need the whole warp); `valid`
// and h < nheads predicate the shared-memory traffic.
template <int HW, int TRIPS>
__device__ __forceinline__ void pipe_heads(uint16_t *base, int nheads, int sub, int d0, bool valid,
                                           const float (&w)[8], bool norm, bool rope,
                                           const float (&cs)[8], const float (&sn)[8], float eps) {
    // TRIPS > 0: the trip count is known at compile time, the loop unrolls fully and
    // independent heads interleave; TRIPS == 0: any head count.
    const int trips = TRIPS > 0 ? TRIPS : (nheads + HW - 1) / HW;
#pragma unroll
    for (int j = 0; j < (TRIPS > 0 ? TRIPS : trips); j++) {
        const int h = sub + j * HW;
        const bool hv = valid && h < nheads;
        uint16_t *hp = base + (size_t)h * 128;
        const uint2 lo = hv ? *reinterpret_cast<const uint2 *>(hp + d0) : make_uint2(0, 0);
        const uint2 hi = hv ? *reinterpret_cast<const uint2 *>(hp + 64 + d0) : make_uint2(0, 0);
        float a[8] = {bf16_lo(lo.x), bf16_hi(lo.x), bf16_lo(lo.y), bf16_hi(lo.y),
                      bf16_lo(hi.x), bf16_hi(hi.x), bf16_lo(hi.y), bf16_hi(hi.y)};
        // pairwise tree: 3 dependent levels instead of 8
        float ss = ((a[0] * a[0] + a[1] * a[1]) + (a[2] * a[2] + a[3] * a[3])) +
                   ((a[4] * a[4] + a[5] * a[5]) + (a[6] * a[6] + a[7] * a[7]));
        ss = group_sum<16>(ss);
        // BF16 output keeps 8 significant bits, so the approximate reciprocal square
        // root and the fused multiply-adds (FP32 ulp-level departures from the
        // separately rounded reference form) cannot show in the result.
        if (norm) {
            const float inv = rsqrtf(ss * (1.0f / 128) + eps);
#pragma unroll
            for (int e = 0; e < 8; e++) a[e] = a[e] * inv * w[e];
        }
        if (rope) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float x1 = a[e], x2 = a[4 + e];
                a[e] = fmaf(-x2, sn[e], x1 * cs[e]);         // x1*c - x2*s
                a[4 + e] = fmaf(x1, sn[4 + e], x2 * cs[4 + e]);  // x1*s + x2*c
            }
        }
        if (hv) {
            *reinterpret_cast<uint2 *>(hp + d0) = make_uint2(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]));
            *reinterpret_cast<uint2 *>(hp + 64 + d0) =
                make_uint2(pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
        }
    }
}

template <int QT, int KT>  // head trips per half-warp for q and k (0: runtime)
__global__ void __launch_bounds__(kPipeThreads, 2)
qk_pipe_kernel(uint16_t *q, uint16_t *k, const float *__restrict__ wq,
               const float *__restrict__ wk, const float *__restrict__ cos_t,
               const float *__restrict__ sin_t, const int32_t *__restrict__ pos,
               int64_t table_rows, int64_t rows, int nq, int nkv, float eps, int *err) {
    constexpr int HD = 128;
    constexpr int kGroupThreads = kPipeThreads / 2;
    constexpr int HWT = (kGroupThreads / 16) / kTileTok;  // half-warps per token in a group
    static_assert(kStages % 2 == 0, "the two groups own alternate stages");
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);
    int *stop_flag = reinterpret_cast<int *>(smem + 64);  // [2]: a group lost a copy
    unsigned char *ring = smem + 128;
    const uint32_t q_tok = (uint32_t)nq * HD * 2, k_tok = (uint32_t)nkv * HD * 2;
    const uint32_t stage_bytes = kTileTok * (q_tok + k_tok);
    const int64_t ntiles = (rows + kTileTok - 1) / kTileTok;
    const int64_t my_n = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int tid = threadIdx.x, lane = tid & 31;
    const int g = tid / kGroupThreads, gtid = tid % kGroupThreads;
    const bool leader = gtid == 0;

    if (tid == 0) {
        for (int s = 0; s < kStages; s++) bulk::mbar_init(&full[s], 1);
        stop_flag[0] = stop_flag[1] = 0;
        bulk::fence_barrier_init();
    }
    __syncthreads();

    auto issue = [&](int64_t i) {  // tile i of this CTA into stage i % kStages (a leader)
        const int64_t r0 = (blockIdx.x + i * gridDim.x) * kTileTok;
        const uint32_t gt = (uint32_t)imin64((int64_t)kTileTok, rows - r0);
        unsigned char *st = ring + (size_t)(i % kStages) * stage_bytes;
        uint64_t *bar = &full[i % kStages];
        bulk::mbar_arrive_expect_tx(bar, gt * (q_tok + k_tok));
        bulk::load(st, q + (size_t)r0 * nq * HD, gt * q_tok, bar);
        if (k_tok) bulk::load(st + kTileTok * q_tok, k + (size_t)r0 * nkv * HD, gt * k_tok, bar);
    };
    int64_t issued = g;  // the group's next tile to issue
    if (leader)
        for (int n = 0; n < kStages / 2 && issued < my_n; n++, issued += 2) issue(issued);

    const int hw = gtid >> 4;   // half-warp 0..7 of the group
    const int tok = hw / HWT;   // token within the tile
    const int sub = hw % HWT;   // this half-warp's share of the token's heads
    const int d0 = (lane & 15) * 4;  // lane owns elements d0..d0+3 and 64+d0..64+d0+3
    const bool rope = cos_t != nullptr;
    float wqv[8], wkv[8];  // [0..3] first half, [4..7] second half
#pragma unroll
    for (int e = 0; e < 4; e++) {
        wqv[e] = wq ? wq[d0 + e] : 1.f;
        wqv[4 + e] = wq ? wq[64 + d0 + e] : 1.f;
        wkv[e] = wk ? wk[d0 + e] : 1.f;
        wkv[4 + e] = wk ? wk[64 + d0 + e] : 1.f;
    }
    // Table position of this half-warp's token in tile t (-1 when there is no token).
    auto tile_pos = [&](int64_t t) -> int64_t {
        if (t >= my_n) return -1;
        const int64_t row = (blockIdx.x + t * gridDim.x) * kTileTok + tok;
        if (row >= rows) return -1;
        return pos ? (int64_t)pos[row] : row;
    };
    auto load_table = [&](int64_t p, float (&c)[8], float (&sgn)[8]) {
        if (!rope || p < 0 || p >= table_rows) return;
        const float *cr = cos_t + (size_t)p * HD, *sr = sin_t + (size_t)p * HD;
        const float4 c1 = ld_f4(cr + d0), c2 = ld_f4(cr + 64 + d0);
        const float4 s1 = ld_f4(sr + d0), s2 = ld_f4(sr + 64 + d0);
        c[0] = c1.x; c[1] = c1.y; c[2] = c1.z; c[3] = c1.w;
        c[4] = c2.x; c[5] = c2.y; c[6] = c2.z; c[7] = c2.w;
        sgn[0] = s1.x; sgn[1] = s1.y; sgn[2] = s1.z; sgn[3] = s1.w;
        sgn[4] = s2.x; sgn[5] = s2.y; sgn[6] = s2.z; sgn[7] = s2.w;
    };
    // positions run two of the group's tiles ahead and table rows one ahead of the
    // compute, so their global-load latency overlaps the wait for the tile's copy
    int64_t p_cur = tile_pos(g), p_nxt = tile_pos(g + 2);
    float cs[8] = {}, sn[8] = {}, csn[8] = {}, snn[8] = {};
    load_table(p_cur, cs, sn);

    bool stopped = false;
    int64_t i = g;
    for (; i < my_n; i += 2) {
        const int s = (int)(i % kStages);
        const uint32_t parity = (uint32_t)((i / kStages) & 1);
        const int64_t r0 = (blockIdx.x + i * gridDim.x) * kTileTok;
        const int gt = (int)imin64((int64_t)kTileTok, rows - r0);
        unsigned char *st = ring + (size_t)s * stage_bytes;
        load_table(p_nxt, csn, snn);
        const int64_t p_far = tile_pos(i + 4);
        const bool ok = bulk::mbar_wait_bounded(&full[s], parity, kWaitLimitNs);
        if (!ok) atomicOr(&stop_flag[g], 1);
        if (ok) {
            bool valid = tok < gt;
            if (rope && valid && (p_cur < 0 || p_cur >= table_rows)) {
                valid = false;
                if (sub == 0 && (lane & 15) == 0 && err) atomicOr(err, LAI_DEVERR_POSITION);
            }
            uint16_t *qb = reinterpret_cast<uint16_t *>(st + (size_t)tok * q_tok);
            uint16_t *kb = reinterpret_cast<uint16_t *>(st + (size_t)kTileTok * q_tok + (size_t)tok * k_tok);
            pipe_heads<HWT, QT>(qb, nq, sub, d0, valid, wqv, wq != nullptr, rope, cs, sn, eps);
            pipe_heads<HWT, KT>(kb, nkv, sub, d0, valid, wkv, wk != nullptr, rope, cs, sn, eps);
        }
        p_cur = p_nxt;
        p_nxt = p_far;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            cs[e] = csn[e];
            sn[e] = snn[e];
        }
        bulk::fence_proxy_async_smem();
        // the group's barrier (ids 1 and 2; 0 is __syncthreads); a lost copy in any of the
        // group's threads ends the group's work, uniformly
        asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(kGroupThreads) : "memory");
        if (*reinterpret_cast<volatile int *>(&stop_flag[g])) {
            stopped = true;
            break;
        }
        if (leader) {
            bulk::store(q + (size_t)r0 * nq * HD, st, (uint32_t)gt * q_tok);
            if (k_tok)
                bulk::store(k + (size_t)r0 * nkv * HD, st + kTileTok * q_tok, (uint32_t)gt * k_tok);
            bulk::commit();
            if (issued < my_n) {
                bulk::wait_read<0>();  // this stage has been read out by its stores
                issue(issued);
                issued += 2;
            }
        }
    }
    if (leader) {
        bulk::wait_all();
        if (stopped) {
            if (err) atomicOr(err, LAI_DEVERR_TIMEOUT);
            // drain loads still in flight into this group's stages, each bounded
            for (int64_t j = i; j < issued; j += 2)
                bulk::mbar_wait_bounded(&full[j % kStages], (uint32_t)((j / kStages) & 1), kWaitLimitNs);
        }
    }
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

// Shared memory of the pipelined kernel, and whether it fits two CTAs per SM.
inline size_t pipe_smem_bytes(int nq, int nkv) {
    return 128 + (size_t)kStages * kTileTok * (size_t)(nq + nkv) * 128 * 2;
}

struct DeviceInfo {
    int sms = 0;
    bool attr_set = false;
};

bool try_pipe(uint16_t *q, uint16_t *k, const float *wq, const float *wk, const float *cos_t,
              const float *sin_t, const int32_t *pos, int64_t table_rows, int64_t rows, int nq,
              int nkv, float eps, int *err, cudaStream_t s) {
    constexpr size_t kMaxSmem = 110 * 1024;  // two CTAs per SM
    const size_t smem = pipe_smem_bytes(nq, nkv);
    if (smem > kMaxSmem || !aligned16(q) || (k && !aligned16(k)) ||
        (cos_t && (!aligned16(cos_t) || !aligned16(sin_t))))
        return false;
    static DeviceInfo info[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    DeviceInfo &d = info[dev];
    // Qwen3's 16 q / 8 kv heads get fully unrolled head loops; other counts the generic one.
    constexpr int HW = 8 / kTileTok;  // half-warps per token within a warp group
    const bool qwen = nq == 8 * HW && (nkv == 4 * HW || nkv == 0);
    auto kern = qwen ? (nkv ? qk_pipe_kernel<8, 4> : qk_pipe_kernel<8, 0>) : qk_pipe_kernel<0, 0>;
    if (!d.attr_set) {
        if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        for (auto f : {qk_pipe_kernel<8, 4>, qk_pipe_kernel<8, 0>, qk_pipe_kernel<0, 0>}) {
            if (cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)kMaxSmem) != cudaSuccess ||
                // the largest carveout, so that two CTAs' rings are resident per SM
                cudaFuncSetAttribute(f, cudaFuncAttributePreferredSharedMemoryCarveout, 100) !=
                    cudaSuccess) {
                cudaGetLastError();
                return false;
            }
        }
        d.attr_set = true;
    }
    const int64_t ntiles = (rows + kTileTok - 1) / kTileTok;
    const int64_t grid = ntiles < 2 * (int64_t)d.sms ? ntiles : 2 * (int64_t)d.sms;
    kern<<<(unsigned)grid, kPipeThreads, smem, s>>>(q, k, wq, wk, cos_t, sin_t, pos, table_rows,
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
        if (hd == 128) done = try_pipe(q, k, wq, wk, cos_t, sin_t, pos, table_rows, rows, nq,
                                       k ? nkv : 0, eps, err, s);
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

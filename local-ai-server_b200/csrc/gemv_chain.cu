// gemv_chain.cu - a decode step's whole chain of fused M = 1 GEMVs in one persistent kernel.
//
// Reference: the per-layer decode sequence of talker_forward (src/tts_native.c:637-668):
//   qwen_rms_norm -> q/k/v linear_bf16                  (:637-642)
//   o_proj linear_bf16 -> qwen_add_inplace              (:658-659)
//   qwen_rms_norm -> gate_up linear_bf16 -> qwen_swiglu_multiply (:661-665)
//   down_proj linear_bf16 -> qwen_add_inplace           (:666-668)
// with linear_bf16(out, in, W, 1, K, N) = W[N,K] . in[K], BF16 weights, FP32 activations
// (src/tts_native.c:66-79). Each op of a chain is one of these fused GEMVs (store, residual
// add or SwiGLU over interleaved gate/up rows, each with an optional RMSNorm of its input),
// and op j reads what op j-1 wrote, as the reference's sequence does.
//
// Why one kernel: at M = 1 a projection streams 2-50 MB of weights, a few microseconds at
// HBM speed, so a chain of one launch per GEMV is bound by the dependency between launches,
// not by HBM. The weights depend on nothing, though. Here every CTA (one per SM, all resident:
// cooperative launch) owns a fixed contiguous slice of rows of every matrix, and a producer
// warp streams the CTA's slices of op j, j+1, ... into a ring of shared-memory stages with
// bulk async copies as fast as the consumer warps free stages - across op boundaries,
// independent of the activations. The consumer warps wait for the grid-wide completion of op
// j-1 (a counter in global memory: one release-add per CTA, an acquire poll), read op j's
// input vector from L2 (the norm weights and the residual rows are requested before it, the
// norm weights before the barrier), normalise it, run the dot products on weights already in
// shared memory and write the op's outputs.
//
// What bounds it (measured with %globaltimer stamps per op and CTA): each op's critical path
// is ~1.5-2 us from the last CTA's stores of op j-1 to op j's staged input (barrier plus one
// L2 round trip), then the dot products over the CTA's rows from shared memory (~0.4 us per
// 12 KiB stage for a warp), then the stores. The per-launch GEMVs (gemv.cu) hold their
// weights in registers before they wait and so spend less after the dependency. Measured on
// B200 (28 layers, CUDA graph): the 0.6B talker's step 454 us here against 410 us as one
// launch per projection, the 1.7B step (2.8 GB of weights) 792 us against 860 us.
//
// Layout in shared memory: kStages stages of 12 KiB (whole weight rows: 6 rows of K = 1024, 3
// of 2048, 2 of 3072, 1 of 6144), the input vector split in two float4 arrays (elements 8v..8v+3
// and 8v+4..8v+7 of 16-byte weight vector v, so both reads of a lane's vector are contiguous
// across the warp), the CTA's row results and the stage mbarriers. Consumer warp w computes
// the op-local rows r = w (mod kConsumerWarps), a whole row per warp (one shuffle tree a row).
//
// Every wait is bounded (1 s): a wait that runs out sets *err, marks the CTA aborted (the
// consumer threads act on it together, at a barrier that ORs the flag), and the producer waits
// (bounded) for its copies in flight before the CTA exits; the other CTAs' next grid waits then
// run out in turn. The grid counter is zeroed before every launch.
#include "lai_common.cuh"
#include "bulk_copy.cuh"

#include <math.h>
#include <new>

namespace lai {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kChainThreads = kConsumers + 32;  // + one producer warp
constexpr int kStages = 16;
constexpr int kStageBytes = 12 * 1024;
constexpr int kMaxK = kStageBytes / 2;           // at least one BF16 row per stage
constexpr int kGroups = kMaxK / 8 / kConsumers;  // 8-element input groups per consumer thread
constexpr int kMaxRowsPerCta = 512;
constexpr int kResPerThread = kMaxRowsPerCta / kConsumers;
constexpr uint64_t kWaitLimitNs = 1000000000ull;
static_assert(kGroups * 8 * kConsumers == kMaxK, "input groups must tile the largest row");

enum Epi { kStore = 0, kResidual = 1, kSwiglu = 2 };

struct ChainSmem {
    uint8_t ring[kStages][kStageBytes];
    float4 xlo[kMaxK / 8], xhi[kMaxK / 8];
    float dot[kMaxRowsPerCta];
    float red[kConsumerWarps];
    uint64_t full[kStages], empty[kStages];
    int abort;
};

// op-local rows of CTA c of G: contiguous, SwiGLU slices in whole gate/up pairs
__host__ __device__ __forceinline__ void rows_of(int n, int epi, int c, int G, int &r0, int &R) {
    if (epi == kSwiglu) {
        const int64_t P = n / 2, p0 = P * c / G, p1 = P * (c + 1) / G;
        r0 = (int)(2 * p0);
        R = (int)(2 * (p1 - p0));
    } else {
        const int64_t a = (int64_t)n * c / G, b = (int64_t)n * (c + 1) / G;
        r0 = (int)a;
        R = (int)(b - a);
    }
}
__host__ __device__ __forceinline__ int rows_per_stage(int k) { return kStageBytes / (k * 2); }

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}
// Consumer barrier that also ORs `v` over the consumer threads: every one gets the same
// answer, so an abort flag the producer warp may set at any moment is acted on uniformly
// (a thread that returned while others wait at the next barrier would leave them waiting).
__device__ __forceinline__ bool consumer_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kConsumers)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Release-add: the consumer barrier before it orders the CTA's stores ahead of the count.
__device__ __forceinline__ void red_release_add(unsigned *p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ bool aborted(const ChainSmem &sm) {
    return *reinterpret_cast<const volatile int *>(&sm.abort) != 0;
}
__device__ __forceinline__ void set_abort(ChainSmem &sm, int *err) {
    *reinterpret_cast<volatile int *>(&sm.abort) = 1;
    atomicOr(err, 1);
}

// Wait until every CTA has finished op j-1 (the counter holds G per finished op).
__device__ bool grid_wait(const unsigned *sync, unsigned target) {
    if (ld_acquire(sync) >= target) return true;
    const uint64_t t0 = bulk::globaltimer_ns();
    for (uint32_t n = 1;; n++) {
        if (ld_acquire(sync) >= target) return true;
        if ((n & 63u) == 0 && bulk::globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// mbarrier phase wait that also gives up when the CTA has aborted
__device__ bool stage_wait(uint64_t *bar, uint32_t parity, const ChainSmem &sm) {
    if (bulk::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = bulk::globaltimer_ns();
    for (uint32_t n = 1;; n++) {
        if (bulk::mbar_try_wait(bar, parity)) return true;
        if ((n & 63u) == 0 && (aborted(sm) || bulk::globaltimer_ns() - t0 > kWaitLimitNs))
            return false;
    }
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float sig = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g)));
    return __fmul_rn(__fmul_rn(g, sig), u);
}

__device__ __forceinline__ float2 bf16_pair(uint32_t w) { return make_float2(bf16_lo(w), bf16_hi(w)); }

// One lane of the producer warp: the CTA's weight slices of every op, in op order, into the
// ring. A stage is refilled once all consumer warps have released its previous contents.
__device__ void produce(const lai_gemv_chain_op_t *ops, int n_ops, ChainSmem &sm, int c, int G,
                        int *err) {
    uint32_t f = 0;  // fills issued
    bool ok = true;
    for (int j = 0; j < n_ops && ok; j++) {
        const lai_gemv_chain_op_t op = ops[j];
        int r0, R;
        rows_of(op.n, op.epilogue, c, G, r0, R);
        const int rps = rows_per_stage(op.k);
        const size_t row_bytes = (size_t)op.k * 2;
        const uint8_t *src = reinterpret_cast<const uint8_t *>(op.w) + (size_t)r0 * row_bytes;
        for (int s0 = 0; s0 < R; s0 += rps, f++) {
            const int q = (int)(f % kStages);
            const uint32_t n = f / kStages;
            if (n > 0 && !stage_wait(&sm.empty[q], (n - 1) & 1u, sm)) {
                if (!aborted(sm)) set_abort(sm, err);
                ok = false;
                break;
            }
            const uint32_t bytes = (uint32_t)((R - s0 < rps ? R - s0 : rps) * row_bytes);
            bulk::mbar_arrive_expect_tx(&sm.full[q], bytes);
            bulk::load(sm.ring[q], src + (size_t)s0 * row_bytes, bytes, &sm.full[q]);
        }
    }
    // the copies still in flight land before this warp (and so the CTA) exits, whether the
    // consumers take them or have aborted
    const uint32_t first = f > (uint32_t)kStages ? f - kStages : 0u;
    for (uint32_t g = first; g < f; g++)
        bulk::mbar_wait_bounded(&sm.full[g % kStages], (g / kStages) & 1u, kWaitLimitNs);
}

// The input vector into shared memory (split layout), RMSNorm-scaled by this thread's
// norm-weight groups (loaded before the grid barrier) when `norm`.
__device__ void stage_input(const lai_gemv_chain_op_t &op, bool norm, const float4 (&nlo)[kGroups],
                            const float4 (&nhi)[kGroups], ChainSmem &sm) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nv = op.k / 8;
    const float4 *in4 = reinterpret_cast<const float4 *>(op.in);
    float4 lo[kGroups], hi[kGroups];
#pragma unroll
    for (int i = 0; i < kGroups; i++) {
        const int v = tid + i * kConsumers;
        if (v < nv) {
            lo[i] = __ldcg(in4 + 2 * v);
            hi[i] = __ldcg(in4 + 2 * v + 1);
        }
    }
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kGroups; i++) {
            if (tid + i * kConsumers >= nv) continue;
            ss = fmaf(lo[i].x, lo[i].x, ss);
            ss = fmaf(lo[i].y, lo[i].y, ss);
            ss = fmaf(lo[i].z, lo[i].z, ss);
            ss = fmaf(lo[i].w, lo[i].w, ss);
            ss = fmaf(hi[i].x, hi[i].x, ss);
            ss = fmaf(hi[i].y, hi[i].y, ss);
            ss = fmaf(hi[i].z, hi[i].z, ss);
            ss = fmaf(hi[i].w, hi[i].w, ss);
        }
        ss = group_sum<32>(ss);
        if (lane == 0) sm.red[warp] = ss;
        consumer_sync();
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; w++) t += sm.red[w];
        const float inv = 1.0f / sqrtf(t / (float)op.k + op.eps);
#pragma unroll
        for (int i = 0; i < kGroups; i++) {
            if (tid + i * kConsumers >= nv) continue;
            const float4 a = nlo[i], b = nhi[i];
            lo[i] = make_float4(__fmul_rn(__fmul_rn(lo[i].x, inv), a.x), __fmul_rn(__fmul_rn(lo[i].y, inv), a.y),
                                __fmul_rn(__fmul_rn(lo[i].z, inv), a.z), __fmul_rn(__fmul_rn(lo[i].w, inv), a.w));
            hi[i] = make_float4(__fmul_rn(__fmul_rn(hi[i].x, inv), b.x), __fmul_rn(__fmul_rn(hi[i].y, inv), b.y),
                                __fmul_rn(__fmul_rn(hi[i].z, inv), b.z), __fmul_rn(__fmul_rn(hi[i].w, inv), b.w));
        }
    }
#pragma unroll
    for (int i = 0; i < kGroups; i++) {
        const int v = tid + i * kConsumers;
        if (v < nv) {
            sm.xlo[v] = lo[i];
            sm.xhi[v] = hi[i];
        }
    }
    consumer_sync();
}

// dot of one BF16 weight row in shared memory with the staged input; every lane gets the total
__device__ __forceinline__ float row_dot(const uint4 *wrow, const ChainSmem &sm, int vpr, int lane) {
    float2 a0 = make_float2(0.f, 0.f), a1 = a0;
#pragma unroll 4
    for (int v = lane; v < vpr; v += 32) {
        const uint4 w = wrow[v];
        const float4 x0 = sm.xlo[v], x1 = sm.xhi[v];
        a0 = __ffma2_rn(bf16_pair(w.x), make_float2(x0.x, x0.y), a0);
        a1 = __ffma2_rn(bf16_pair(w.y), make_float2(x0.z, x0.w), a1);
        a0 = __ffma2_rn(bf16_pair(w.z), make_float2(x1.x, x1.y), a0);
        a1 = __ffma2_rn(bf16_pair(w.w), make_float2(x1.z, x1.w), a1);
    }
    return group_sum<32>((a0.x + a0.y) + (a1.x + a1.y));
}

__device__ void consume(const lai_gemv_chain_op_t *ops, int n_ops, ChainSmem &sm, int c, int G,
                        unsigned *sync, int *err) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t f = 0;  // fills consumed
    for (int j = 0; j < n_ops; j++) {
        const lai_gemv_chain_op_t op = ops[j];
        int r0, R;
        rows_of(op.n, op.epilogue, c, G, r0, R);
        const int rps = rows_per_stage(op.k), vpr = op.k / 8;
        const bool norm = op.norm_w != nullptr;
        // the norm weights depend on nothing: requested before the barrier
        float4 nlo[kGroups], nhi[kGroups];
        if (norm) {
            const float4 *w4 = reinterpret_cast<const float4 *>(op.norm_w);
#pragma unroll
            for (int i = 0; i < kGroups; i++) {
                const int v = tid + i * kConsumers;
                if (v < vpr) {
                    nlo[i] = __ldg(w4 + 2 * v);
                    nhi[i] = __ldg(w4 + 2 * v + 1);
                }
            }
        }
        if (j > 0) {  // op j-1 finished on every CTA: its outputs are this op's inputs
            if (tid == 0 && !grid_wait(sync, (unsigned)j * (unsigned)G)) set_abort(sm, err);
            if (consumer_sync_any(aborted(sm))) return;
        }
        // the residual rows this thread adds into, in flight with the input vector
        float res[kResPerThread];
        if (op.epilogue == kResidual) {
#pragma unroll
            for (int i = 0; i < kResPerThread; i++) {
                const int t = tid + i * kConsumers;
                res[i] = t < R ? __ldcg(op.out + r0 + t) : 0.f;
            }
        }
        stage_input(op, norm, nlo, nhi, sm);
        for (int s0 = 0; s0 < R; s0 += rps, f++) {
            const int q = (int)(f % kStages);
            if (!__all_sync(0xffffffffu, stage_wait(&sm.full[q], (f / kStages) & 1u, sm))) {
                if (lane == 0 && !aborted(sm)) set_abort(sm, err);
                break;
            }
            const int s1 = R - s0 < rps ? R : s0 + rps;
            const int first = s0 + ((warp - s0) % kConsumerWarps + kConsumerWarps) % kConsumerWarps;
            for (int lr = first; lr < s1; lr += kConsumerWarps) {
                const uint4 *wrow =
                    reinterpret_cast<const uint4 *>(sm.ring[q] + (size_t)(lr - s0) * op.k * 2);
                const float d = row_dot(wrow, sm, vpr, lane);
                if (lane == 0) sm.dot[lr] = d;
            }
            __syncwarp();
            if (lane == 0) bulk::mbar_arrive(&sm.empty[q]);
        }
        if (consumer_sync_any(aborted(sm))) return;
        if (op.epilogue == kSwiglu) {
            for (int t = tid; t < R / 2; t += kConsumers)
                op.out[r0 / 2 + t] = silu_mul(sm.dot[2 * t], sm.dot[2 * t + 1]);
        } else if (op.epilogue == kResidual) {
#pragma unroll
            for (int i = 0; i < kResPerThread; i++) {
                const int t = tid + i * kConsumers;
                if (t < R) op.out[r0 + t] = res[i] + sm.dot[t];
            }
        } else {
            for (int t = tid; t < R; t += kConsumers) op.out[r0 + t] = sm.dot[t];
        }
        consumer_sync();
        if (tid == 0) red_release_add(sync, 1u);
    }
}

__global__ void __launch_bounds__(kChainThreads, 1)
gemv_chain_kernel(const lai_gemv_chain_op_t *ops, int n_ops, unsigned *sync, int *err) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    ChainSmem &sm = *reinterpret_cast<ChainSmem *>(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) {
            bulk::mbar_init(&sm.full[s], 1);
            bulk::mbar_init(&sm.empty[s], kConsumerWarps);
        }
        sm.abort = 0;
        bulk::fence_barrier_init();
    }
    __syncthreads();
    if (warp == kConsumerWarps) {
        if (lane == 0) produce(ops, n_ops, sm, blockIdx.x, gridDim.x, err);
        return;
    }
    consume(ops, n_ops, sm, blockIdx.x, gridDim.x, sync, err);
}

}  // namespace
}  // namespace lai

struct lai_gemv_chain {
    lai_gemv_chain_op_t *ops;  // device copy of the op table
    unsigned *sync;            // device grid counter
    int n_ops;
    int grid;
};

extern "C" int lai_gemv_chain_create(lai_gemv_chain_t **chain, const lai_gemv_chain_op_t *ops,
                                     int n_ops) {
    using namespace lai;
    if (!chain || n_ops < 0 || (n_ops > 0 && !ops)) return LAI_ERR_INVALID;
    *chain = nullptr;
    for (int j = 0; j < n_ops; j++) {  // checks that need no device first
        const lai_gemv_chain_op_t &op = ops[j];
        if (!op.w || !op.in || !op.out || op.n <= 0 || op.k <= 0 || op.k % 256 != 0 ||
            op.epilogue < kStore || op.epilogue > kSwiglu || !aligned16(op.w) || !aligned16(op.in) ||
            (op.norm_w && !aligned16(op.norm_w)) || !(op.eps >= 0.f) ||
            (op.epilogue == kSwiglu && op.n % 2 != 0))
            return LAI_ERR_INVALID;
        if (op.k > kMaxK) return LAI_ERR_TOOBIG;
        const size_t out_n = op.epilogue == kSwiglu ? (size_t)op.n / 2 : (size_t)op.n;
        if (overlaps(op.out, out_n * 4, op.in, (size_t)op.k * 4)) return LAI_ERR_ALIAS;
    }
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return LAI_ERR_CUDA;
    const size_t smem = sizeof(ChainSmem);
    if (cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem) != cudaSuccess)
        return LAI_ERR_CUDA;
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemv_chain_kernel, kChainThreads,
                                                      smem) != cudaSuccess ||
        per_sm < 1)
        return LAI_ERR_CUDA;
    const int G = sms;  // one CTA per SM: the whole grid is resident
    for (int j = 0; j < n_ops; j++) {  // the rows one CTA holds results for
        const lai_gemv_chain_op_t &op = ops[j];
        const int most = op.epilogue == kSwiglu ? 2 * ((op.n / 2 + G - 1) / G) : (op.n + G - 1) / G;
        if (most > kMaxRowsPerCta) return LAI_ERR_TOOBIG;
    }
    lai_gemv_chain *c = new (std::nothrow) lai_gemv_chain{};
    if (!c) return LAI_ERR_NOMEM;
    c->n_ops = n_ops;
    c->grid = G;
    const size_t tb = sizeof(lai_gemv_chain_op_t) * (size_t)(n_ops > 0 ? n_ops : 1);
    if (cudaMalloc(&c->ops, tb) != cudaSuccess) {
        delete c;
        return LAI_ERR_NOMEM;
    }
    if (cudaMalloc(&c->sync, sizeof(unsigned)) != cudaSuccess) {
        cudaFree(c->ops);
        delete c;
        return LAI_ERR_NOMEM;
    }
    if ((n_ops > 0 && cudaMemcpy(c->ops, ops, sizeof(lai_gemv_chain_op_t) * n_ops,
                                 cudaMemcpyHostToDevice) != cudaSuccess) ||
        cudaMemset(c->sync, 0, sizeof(unsigned)) != cudaSuccess) {
        cudaFree(c->ops);
        cudaFree(c->sync);
        delete c;
        return LAI_ERR_CUDA;
    }
    *chain = c;
    return LAI_OK;
}

extern "C" int lai_gemv_chain_run(const lai_gemv_chain_t *chain, int *err, lai_stream_t stream) {
    using namespace lai;
    if (!chain || !err) return LAI_ERR_INVALID;
    if (chain->n_ops == 0) return LAI_OK;
    cudaStream_t st = as_stream(stream);
    if (cudaMemsetAsync(chain->sync, 0, sizeof(unsigned), st) != cudaSuccess) return LAI_ERR_CUDA;
    const lai_gemv_chain_op_t *ops = chain->ops;
    int n = chain->n_ops;
    unsigned *sync = chain->sync;
    void *args[] = {(void *)&ops, (void *)&n, (void *)&sync, (void *)&err};
    if (cudaLaunchCooperativeKernel((const void *)gemv_chain_kernel, dim3(chain->grid),
                                    dim3(kChainThreads), args, sizeof(ChainSmem), st) != cudaSuccess)
        return LAI_ERR_CUDA;
    return launch_status();
}

extern "C" int lai_gemv_chain_grid(const lai_gemv_chain_t *chain) { return chain ? chain->grid : 0; }

extern "C" void lai_gemv_chain_destroy(lai_gemv_chain_t *chain) {
    if (!chain) return;
    cudaFree(chain->ops);
    cudaFree(chain->sync);
    delete chain;
}

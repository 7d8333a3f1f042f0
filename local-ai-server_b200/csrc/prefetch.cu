// prefetch.cu - L2 prefetch of a weight range, for the decode GEMV chain.
//
// At decode (M = 1) each of a layer's four projections is a 2-50 MB weight stream whose
// kernel starts only after the previous one has produced its input vector
// (src/tts_native.c:637-668): launched one after another, every GEMV pays the DRAM
// latency and ramp of its own stream and HBM idles between them. Weights depend on
// nothing, so the next GEMV's matrix can be brought into L2 while the current one
// runs: lai_prefetch_l2 issues bulk L2 prefetches (cp.async.bulk.prefetch.L2, the TMA
// engine, no data into the SM) for [p, p + bytes) from up to one CTA per SM, each lane
// 8 KB at a time. It is launched with programmatic dependent launch: it lets the next
// kernel on the stream start launching at once, issues its prefetches alongside the
// previous kernel, and ends only after that kernel has (griddepcontrol.wait), so a
// kernel that waits on this one also waits on the one before it.
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kPrefetchThreads = 32;
constexpr uint32_t kPrefetchChunk = 8u << 10;  // bytes per bulk prefetch

__global__ void __launch_bounds__(kPrefetchThreads)
l2_prefetch_kernel(const unsigned char *p, uint64_t bytes) {
    pdl_launch_dependents();
    const uint64_t step = (uint64_t)gridDim.x * kPrefetchThreads * kPrefetchChunk;
    for (uint64_t off = ((uint64_t)blockIdx.x * kPrefetchThreads + threadIdx.x) * kPrefetchChunk;
         off < bytes; off += step) {
        const uint64_t left = bytes - off;
        const uint32_t n = (uint32_t)(left < kPrefetchChunk ? left : kPrefetchChunk) & ~15u;
        if (n)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + off), "r"(n)
                         : "memory");
    }
    pdl_wait_prior();  // complete only after the previous kernel on the stream
}

}  // namespace
}  // namespace lai

extern "C" int lai_prefetch_l2(const void *p, int64_t bytes, lai_stream_t stream) {
    if (!p || bytes < 0) return LAI_ERR_INVALID;
    if (!lai::aligned16(p)) return LAI_ERR_INVALID;
    if (bytes == 0) return LAI_OK;
    static int sms[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return LAI_ERR_CUDA;
    if (!sms[dev] && cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev) !=
                         cudaSuccess) {
        cudaGetLastError();
        return LAI_ERR_CUDA;
    }
    const int64_t per_cta = (int64_t)lai::kPrefetchThreads * lai::kPrefetchChunk;
    const int64_t want = (bytes + per_cta - 1) / per_cta;
    const unsigned grid = (unsigned)(want < sms[dev] ? want : sms[dev]);
    if (lai::launch_pdl(lai::l2_prefetch_kernel, dim3(grid), dim3(lai::kPrefetchThreads), 0,
                        lai::as_stream(stream), static_cast<const unsigned char *>(p),
                        (uint64_t)bytes) != cudaSuccess) {
        cudaGetLastError();
        return LAI_ERR_CUDA;
    }
    return LAI_OK;
}

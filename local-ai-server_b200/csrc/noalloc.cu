// noalloc.cu - host-buffer RMSNorm that allocates no device memory.
//
// qwen_rms_norm on host buffers stages rows through device buffers that the
// library allocates with cudaMalloc on first use. Some callers cannot let a
// library allocate: a process whose device memory is all handed to its own pool
// allocator (a framework's caching allocator, a fixed arena sized at start-up),
// or a latency-critical loop that must never hit cudaMalloc / cudaFree, which
// can synchronise the whole device. lai_rmsnorm_f32_host_noalloc serves them:
// it stages through one fixed array compiled into this library.
//
// The array below lives in the memory of every GPU that loads this library's
// device code, from that load until process exit (kNoAllocScratchBytes per GPU).
// With CUDA's default lazy module loading the load happens at the first use of
// the module on a device -- in practice inside this entry point's first
// cudaGetSymbolAddress -- so the first call on a device is the one that claims
// the 8 MiB. A caller whose pool reserves (nearly) all device memory must make
// one call (or run with CUDA_MODULE_LOADING=EAGER) before the pool reserves it,
// and before any stream capture begins.
//
// Host code may not use the array's name as an address (that is a host-side
// stand-in; a kernel given it would fault, or silently touch host memory where
// the GPU can reach it): every call looks up the device address with
// cudaGetSymbolAddress on the current device. That look-up is cheap once the
// module is loaded, and it stays correct after the caller resets the device.
//
// Every call on a device uses the same array and it keeps the last call's bytes.
// Nothing in it must start at zero: each call writes the weights and rows it
// reads before reading them. Calls whose GPU work overlaps (two host threads, or
// two streams, on one device at once) race on the array; a call synchronises
// its stream before returning -- on its error paths too, once anything was
// queued -- so calls made one after another are safe.
#include "../../include/lai_qwen_dropin.h"
#include "lai_common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device.
int scratch_address(void **out) {
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) {
        cudaGetLastError();
        return LAI_ERR_CUDA;
    }
    *out = p;
    return LAI_OK;
}

inline size_t round256(size_t n) { return (n + 255) & ~size_t(255); }

// Ends a call whose work was (partly) queued on s: waits for it, so that no copy
// into the shared array is still running when the call returns, and returns the
// status that ended the call.
int drain(cudaStream_t s, int st) {
    cudaStreamSynchronize(s);
    cudaGetLastError();
    return st;
}

}  // namespace

extern "C" int lai_rmsnorm_f32_host_noalloc(float *out, const float *x, const float *w, int seq,
                                            int dim, float eps, lai_stream_t stream) {
    if (!out || !x || !w || seq < 0 || dim <= 0) return LAI_ERR_INVALID;
    if (seq == 0) return LAI_OK;
    const size_t row_bytes = (size_t)seq * dim * sizeof(float);
    const size_t w_bytes = (size_t)dim * sizeof(float);
    if (round256(w_bytes) + round256(row_bytes) > kNoAllocScratchBytes) return LAI_ERR_TOOBIG;
    void *base = nullptr;
    int st = scratch_address(&base);
    if (st != LAI_OK) return st;
    float *sw = static_cast<float *>(base);
    float *sx = reinterpret_cast<float *>(static_cast<char *>(base) + round256(w_bytes));
    cudaStream_t s = lai::as_stream(stream);
    // cudaMemcpyDefault: host (pageable or pinned) or device pointers alike.
    if (cudaMemcpyAsync(sw, w, w_bytes, cudaMemcpyDefault, s) != cudaSuccess)
        return drain(s, LAI_ERR_CUDA);
    if (cudaMemcpyAsync(sx, x, row_bytes, cudaMemcpyDefault, s) != cudaSuccess)
        return drain(s, LAI_ERR_CUDA);
    st = lai_rmsnorm_f32(sx, sx, sw, seq, dim, eps, stream);  // in place in the scratch rows
    if (st != LAI_OK) return drain(s, st);
    if (cudaMemcpyAsync(out, sx, row_bytes, cudaMemcpyDefault, s) != cudaSuccess)
        return drain(s, LAI_ERR_CUDA);
    if (cudaStreamSynchronize(s) != cudaSuccess) {
        cudaGetLastError();
        return LAI_ERR_CUDA;
    }
    return LAI_OK;
}

// elementwise.cu - residual add (x += y) and the BF16 token-embedding gather.
//
// Residual add: qwen_add_inplace(x, y, n) (src/tts_native.c:582, 591, 1142).
//   Roofline: HBM, 3*s bytes per element (read x, y; write x).
// Gather: embed_lookup_bf16 / bf16_to_f32_row (src/tts_native.c:35-40, 473-476):
//   out row r = table row ids[r]; widening is the exact bit shift.
//   Roofline: HBM (or L2 for small hot tables), per row 2*D read + 4 B id +
//   2*D (BF16 out) or 4*D (F32 out) written. One warp per row, 16-byte vectors.
#include "lai_common.cuh"

namespace lai {
namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kGatherVec = 8;  // gather: 16-byte vectors per lane in flight (2048 BF16 per warp)

template <typename T>
__global__ void __launch_bounds__(kThreads)
add_vec_kernel(T *x, const T *y, int64_t nvec) {
    constexpr int E = Elt<T>::N;
    const int64_t base = (int64_t)blockIdx.x * (kThreads * kUnroll) + threadIdx.x;
    uint4 a[kUnroll], b[kUnroll];
#pragma unroll
    for (int i = 0; i < kUnroll; i++) {
        const int64_t k = base + (int64_t)i * kThreads;
        if (k < nvec) {
            a[i] = ld_rw(x + k * E);
            b[i] = ld_stream(y + k * E);
        }
    }
#pragma unroll
    for (int i = 0; i < kUnroll; i++) {
        const int64_t k = base + (int64_t)i * kThreads;
        if (k < nvec) {
            float fa[E], fb[E];
            unpack<T>(a[i], fa);
            unpack<T>(b[i], fb);
#pragma unroll
            for (int e = 0; e < E; e++) fa[e] = __fadd_rn(fa[e], fb[e]);
            st_vec(x + k * E, pack<T>(fa));
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) add_scalar_kernel(T *x, const T *y, int64_t k0, int64_t n) {
    const int64_t k = k0 + (int64_t)blockIdx.x * kThreads + threadIdx.x;
    if (k < n) x[k] = from_f<T>(__fadd_rn(to_f(x[k]), to_f(y[k])));
}

template <typename T>
int run_add(T *x, const T *y, int64_t n, lai_stream_t stream) {
    if (!x || !y || n < 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    const size_t b = (size_t)n * sizeof(T);
    if (x != y && overlaps(x, b, y, b)) return LAI_ERR_ALIAS;
    cudaStream_t s = as_stream(stream);
    constexpr int E = Elt<T>::N;
    int64_t done = 0;
    if (aligned16(x) && aligned16(y)) {
        const int64_t nvec = n / E;
        if (nvec > 0)
            add_vec_kernel<T><<<grid_for(nvec, kThreads * kUnroll), kThreads, 0, s>>>(x, y, nvec);
        done = nvec * E;
    }
    if (done < n) add_scalar_kernel<T><<<grid_for(n - done, kThreads), kThreads, 0, s>>>(x, y, done, n);
    return launch_status();
}

// ---- gather ----------------------------------------------------------------------
// OUT_F32: widen to F32 (bit shift), else copy BF16. VEC: 16-byte path.
template <bool OUT_F32, bool VEC>
__global__ void __launch_bounds__(256)
gather_kernel(void *out, const uint16_t *__restrict__ table, const int32_t *__restrict__ ids,
              int64_t n, int dim, int64_t vocab, int *err) {
    const int lane = threadIdx.x & 31;
    const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= n) return;
    pdl_wait_prior();  // launched with programmatic dependent launch: inputs after this
    const int64_t id = ids[r];
    const bool ok = id >= 0 && id < vocab;
    if (!ok && lane == 0 && err) atomicOr(err, LAI_DEVERR_TOKEN_ID);
    const uint16_t *src = table + (size_t)(ok ? id : 0) * dim;
    if constexpr (VEC) {
        // up to kGatherVec 16-byte vectors per lane (a 2048-wide row) loaded before any store,
        // so a warp has its whole row in flight
        const int nv = dim / 8;
        for (int v0 = 0; v0 < nv; v0 += 32 * kGatherVec) {
            uint4 t[kGatherVec];
#pragma unroll
            for (int i = 0; i < kGatherVec; i++) {
                const int v = v0 + i * 32 + lane;
                t[i] = ok && v < nv ? ld_stream(src + (size_t)v * 8) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < kGatherVec; i++) {
                const int v = v0 + i * 32 + lane;
                if (v >= nv) break;
                if constexpr (OUT_F32) {
                    uint4 *o = reinterpret_cast<uint4 *>(static_cast<float *>(out) + (size_t)r * dim) + 2 * v;
                    o[0] = make_uint4(t[i].x << 16, t[i].x & 0xffff0000u, t[i].y << 16, t[i].y & 0xffff0000u);
                    o[1] = make_uint4(t[i].z << 16, t[i].z & 0xffff0000u, t[i].w << 16, t[i].w & 0xffff0000u);
                } else {
                    st_vec(static_cast<uint16_t *>(out) + (size_t)r * dim + (size_t)v * 8, t[i]);
                }
            }
        }
    } else {
        for (int i = lane; i < dim; i += 32) {
            const uint16_t h = ok ? src[i] : 0;
            if constexpr (OUT_F32)
                static_cast<uint32_t *>(out)[(size_t)r * dim + i] = ((uint32_t)h) << 16;
            else
                static_cast<uint16_t *>(out)[(size_t)r * dim + i] = h;
        }
    }
    pdl_launch_dependents();
}

template <bool OUT_F32>
int run_gather(void *out, const uint16_t *table, const int32_t *ids, int64_t n, int dim,
               int64_t vocab, int *err, lai_stream_t stream) {
    if (!out || !table || !ids || n < 0 || dim <= 0 || vocab <= 0) return LAI_ERR_INVALID;
    if (n == 0) return LAI_OK;
    cudaStream_t s = as_stream(stream);
    const bool vec = dim % 8 == 0 && aligned16(out) && aligned16(table);
    if (vec)
        launch_pdl(gather_kernel<OUT_F32, true>, dim3(grid_for(n, 8)), dim3(256), 0, s, out, table,
                   ids, n, dim, vocab, err);
    else
        launch_pdl(gather_kernel<OUT_F32, false>, dim3(grid_for(n, 8)), dim3(256), 0, s, out, table,
                   ids, n, dim, vocab, err);
    return launch_status();
}

}  // namespace
}  // namespace lai

extern "C" {

int lai_add_bf16(lai_bf16 *x, const lai_bf16 *y, int64_t n, lai_stream_t stream) {
    return lai::run_add<uint16_t>(x, y, n, stream);
}
int lai_add_f32(float *x, const float *y, int64_t n, lai_stream_t stream) {
    return lai::run_add<float>(x, y, n, stream);
}

int lai_embed_gather_bf16(lai_bf16 *out, const lai_bf16 *table, const int32_t *ids, int64_t n,
                          int dim, int64_t vocab, int *err, lai_stream_t stream) {
    return lai::run_gather<false>(out, table, ids, n, dim, vocab, err, stream);
}
int lai_embed_gather_bf16_to_f32(float *out, const lai_bf16 *table, const int32_t *ids,
                                 int64_t n, int dim, int64_t vocab, int *err,
                                 lai_stream_t stream) {
    return lai::run_gather<true>(out, table, ids, n, dim, vocab, err, stream);
}

}  // extern "C"

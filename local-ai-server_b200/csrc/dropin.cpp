// dropin.cpp - the reference's qwen_* / voc_snake_beta names over the B200 kernels.
//
// Each drop-in call is described as a list of arguments (pointer, bytes per row
// or whole size, in/out) plus a launcher that runs one lai_* kernel on a row
// range. If every pointer is device-accessible the launcher runs once on the
// drop-in stream. Otherwise host rows are staged: rows are cut into chunks of
// about kChunkBytes host bytes that cycle through kSlots device slots, and three
// streams carry them: copy-in (all host-to-device copies, in chunk order), kernel
// and copy-out (all device-to-host copies). Chunk c's kernel waits for its copy-in,
// its copy-out for its kernel, and the copy-in of chunk c + kSlots for that copy-out
// (the slot is free again), so both copy directions stay busy back to back. When a
// host output aliases a host input with another row size (SwiGLU compaction,
// out == gate_up), the copy-out of chunk c overwrites input bytes of chunks <= c
// only, all copied in before chunk c's own copy-in on the in-order copy-in stream:
// no further ordering is needed.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <functional>
#include <unordered_map>
#include <vector>

#include "../../include/lai_kernels.h"
#include "../../include/lai_qwen_dropin.h"

namespace {

constexpr int kSlots = 4;
constexpr size_t kChunkBytes = 16u << 20;
enum { kIn = 0, kKernel = 1, kOut = 2, kStreams = 3 };

struct Ctx {
    int device = -1;
    cudaStream_t pipe[kStreams] = {};  // copy-in, kernel, copy-out
    void *slot[kSlots] = {};
    size_t slot_cap[kSlots] = {};
    void *whole = nullptr;
    size_t whole_cap = 0;
    int *derr = nullptr;        // device error word of staged calls
    int *derr_direct = nullptr; // device error word of device-pointer calls
    int32_t *zero_id = nullptr; // a device int holding 0 (single-row gathers)
    cudaEvent_t in_done[kSlots] = {}, k_done[kSlots] = {}, out_done[kSlots] = {};
    cudaEvent_t start_ev = nullptr;
};

thread_local std::unordered_map<int, Ctx> t_ctx;
thread_local int t_last_error = LAI_OK;
thread_local cudaStream_t t_stream = nullptr;

int fail(const char *fn, int status, const char *what) {
    t_last_error = status;
    std::fprintf(stderr, "lai: %s: %s (%s)\n", fn, lai_status_string(status), what ? what : "");
    return status;
}

int cuda_fail(const char *fn, cudaError_t e) {
    return fail(fn, LAI_ERR_CUDA, cudaGetErrorString(e));
}

Ctx *get_ctx(const char *fn) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        cuda_fail(fn, e);
        return nullptr;
    }
    Ctx &c = t_ctx[dev];
    if (c.device < 0) {
        c.device = dev;
        for (int i = 0; i < kStreams; i++)
            if ((e = cudaStreamCreateWithFlags(&c.pipe[i], cudaStreamNonBlocking)) != cudaSuccess) break;
        for (int i = 0; i < kSlots && e == cudaSuccess; i++)
            for (cudaEvent_t *ev : {&c.in_done[i], &c.k_done[i], &c.out_done[i]})
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaMalloc(&c.derr, 4 * sizeof(int));
        if (e == cudaSuccess) e = cudaMemset(c.derr, 0, 4 * sizeof(int));
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c.start_ev, cudaEventDisableTiming);
        if (e != cudaSuccess) {
            cuda_fail(fn, e);
            t_ctx.erase(dev);
            return nullptr;
        }
        c.derr_direct = c.derr + 1;
        c.zero_id = reinterpret_cast<int32_t *>(c.derr + 2);
    }
    return &c;
}

bool grow(void **p, size_t *cap, size_t need) {
    if (need <= *cap) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t n = need + need / 4;
    if (cudaMalloc(p, n) != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        return false;
    }
    *cap = n;
    return true;
}

bool device_accessible(const void *p) {
    if (!p) return true;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// Host memory registered (pinned and mapped): the device address to read it with.
const void *mapped_device_ptr(const void *p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) return p;
    if (a.type == cudaMemoryTypeHost) return a.devicePointer;
    return nullptr;
}

struct Arg {
    const void *ptr;  // user pointer (may be NULL for optional args)
    size_t row_bytes; // > 0: chunked by rows; 0: whole argument of whole_bytes
    size_t whole_bytes;
    bool in, out;
    // filled by the engine
    bool host = false;
    size_t whole_off = 0;
    size_t slot_off = 0;
};

// launcher(stream, row0, nrows, device pointers per arg, err word) -> LAI status
using Launcher = std::function<int(cudaStream_t, int64_t, int64_t, void **, int *)>;

int run_op(const char *fn, std::vector<Arg> &args, int64_t rows, const Launcher &launch) {
    Ctx *c = get_ctx(fn);
    if (!c) return LAI_ERR_CUDA;
    if (rows <= 0) return LAI_OK;
    std::vector<void *> dptr(args.size());
    bool all_dev = true;
    for (auto &a : args) {
        a.host = a.ptr && !device_accessible(a.ptr);
        all_dev = all_dev && !a.host;
    }
    if (all_dev) {
        for (size_t i = 0; i < args.size(); i++) dptr[i] = const_cast<void *>(args[i].ptr);
        int st = launch(t_stream, 0, rows, dptr.data(), c->derr_direct);
        return st == LAI_OK ? LAI_OK : fail(fn, st, "launch");
    }

    // ---- staged path ----
    cudaError_t e;
    size_t whole = 0, per_row = 0;
    for (auto &a : args) {
        if (!a.host) continue;
        if (a.row_bytes == 0) {
            a.whole_off = whole;
            whole += (a.whole_bytes + 255) & ~size_t(255);
        } else {
            per_row += a.row_bytes;
        }
    }
    int64_t chunk = per_row ? (int64_t)(kChunkBytes / per_row) : rows;
    if (chunk < 1) chunk = 1;
    if (chunk > rows) chunk = rows;
    size_t off = 0;
    for (auto &a : args)
        if (a.host && a.row_bytes) {
            a.slot_off = off;
            off += ((size_t)chunk * a.row_bytes + 255) & ~size_t(255);
        }
    for (int s = 0; s < kSlots; s++)
        if (off && !grow(&c->slot[s], &c->slot_cap[s], off)) return fail(fn, LAI_ERR_NOMEM, "staging");
    if (whole && !grow(&c->whole, &c->whole_cap, whole)) return fail(fn, LAI_ERR_NOMEM, "staging");

    // order after prior work on the drop-in stream (device-pointer args)
    if ((e = cudaEventRecord(c->start_ev, t_stream)) != cudaSuccess) return cuda_fail(fn, e);
    for (int s = 0; s < kStreams; s++) cudaStreamWaitEvent(c->pipe[s], c->start_ev, 0);
    cudaStream_t sin = c->pipe[kIn], sk = c->pipe[kKernel], sout = c->pipe[kOut];
    cudaMemsetAsync(c->derr, 0, sizeof(int), sin);
    for (auto &a : args)
        if (a.host && a.row_bytes == 0 && a.in)
            cudaMemcpyAsync(static_cast<char *>(c->whole) + a.whole_off, a.ptr, a.whole_bytes,
                            cudaMemcpyHostToDevice, sin);

    // An aliased host output may only be a compaction of its input (rows no longer than the
    // input's, as SwiGLU's): then chunk c's copy-out overwrites input bytes of chunks <= c
    // only, all already copied in on the in-order copy-in stream (see the top of this file).
    for (auto &o : args)
        for (auto &i : args)
            if (&o != &i && o.host && i.host && o.out && i.in && o.ptr == i.ptr &&
                o.row_bytes > i.row_bytes) {
                for (int s2 = 0; s2 < kStreams; s2++) cudaStreamSynchronize(c->pipe[s2]);
                return fail(fn, LAI_ERR_ALIAS, "output rows longer than the input rows they alias");
            }

    const int64_t nchunks = (rows + chunk - 1) / chunk;
    int status = LAI_OK;
    for (int64_t ci = 0; ci < nchunks && status == LAI_OK; ci++) {
        const int64_t r0 = ci * chunk, nr = (r0 + chunk <= rows) ? chunk : rows - r0;
        const int s = (int)(ci % kSlots);
        if (ci >= kSlots) cudaStreamWaitEvent(sin, c->out_done[s], 0);  // slot read out
        for (size_t i = 0; i < args.size(); i++) {
            Arg &a = args[i];
            if (!a.ptr) { dptr[i] = nullptr; continue; }
            if (!a.host) {
                dptr[i] = const_cast<char *>(static_cast<const char *>(a.ptr)) +
                          (a.row_bytes ? (size_t)r0 * a.row_bytes : 0);
                continue;
            }
            if (a.row_bytes == 0) {
                dptr[i] = static_cast<char *>(c->whole) + a.whole_off;
                continue;
            }
            dptr[i] = static_cast<char *>(c->slot[s]) + a.slot_off;
            if (a.in)
                cudaMemcpyAsync(dptr[i], static_cast<const char *>(a.ptr) + (size_t)r0 * a.row_bytes,
                                (size_t)nr * a.row_bytes, cudaMemcpyHostToDevice, sin);
        }
        cudaEventRecord(c->in_done[s], sin);
        cudaStreamWaitEvent(sk, c->in_done[s], 0);
        status = launch(sk, r0, nr, dptr.data(), c->derr);
        cudaEventRecord(c->k_done[s], sk);
        cudaStreamWaitEvent(sout, c->k_done[s], 0);
        for (size_t i = 0; i < args.size() && status == LAI_OK; i++) {
            Arg &a = args[i];
            if (!a.ptr || !a.host || !a.out || a.row_bytes == 0) continue;
            char *hdst = const_cast<char *>(static_cast<const char *>(a.ptr)) + (size_t)r0 * a.row_bytes;
            cudaMemcpyAsync(hdst, dptr[i], (size_t)nr * a.row_bytes, cudaMemcpyDeviceToHost, sout);
        }
        cudaEventRecord(c->out_done[s], sout);
    }
    cudaError_t sync_err = cudaSuccess;
    for (int s = 0; s < kStreams; s++) {
        cudaError_t es = cudaStreamSynchronize(c->pipe[s]);
        if (es != cudaSuccess && sync_err == cudaSuccess) sync_err = es;
    }
    const cudaError_t last = cudaGetLastError();
    if (sync_err != cudaSuccess) return cuda_fail(fn, sync_err);
    if (last != cudaSuccess) return cuda_fail(fn, last);
    int flags = 0;
    if ((e = cudaMemcpy(&flags, c->derr, sizeof(int), cudaMemcpyDeviceToHost)) != cudaSuccess)
        return cuda_fail(fn, e);
    if (status != LAI_OK) return fail(fn, status, "launch");
    if (flags) return fail(fn, LAI_ERR_RANGE, "index out of range");
    return LAI_OK;
}

template <typename T> T *P(void **d, int i) { return static_cast<T *>(d[i]); }

}  // namespace

extern "C" {

void qwen_rms_norm(float *out, const float *x, const float *w, int seq, int dim, float eps) {
    const char *fn = "qwen_rms_norm";
    if (!out || !x || !w || seq < 0 || dim <= 0) { fail(fn, LAI_ERR_INVALID, "arguments"); return; }
    std::vector<Arg> a = {{out, (size_t)dim * 4, 0, false, true},
                          {x, (size_t)dim * 4, 0, true, false},
                          {w, 0, (size_t)dim * 4, true, false}};
    run_op(fn, a, seq, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *) {
        return lai_rmsnorm_f32(P<float>(d, 0), P<float>(d, 1), P<float>(d, 2), n, dim, eps, s);
    });
}

void qwen_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim,
                            float eps) {
    const char *fn = "qwen_rms_norm_per_head";
    if (!x || !w || seq < 0 || n_heads <= 0 || head_dim <= 0 || (head_dim & 1)) {
        fail(fn, LAI_ERR_INVALID, "arguments");
        return;
    }
    std::vector<Arg> a = {{x, (size_t)n_heads * head_dim * 4, 0, true, true},
                          {w, 0, (size_t)head_dim * 4, true, false}};
    run_op(fn, a, seq, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *err) {
        return lai_qk_norm_rope_f32(P<float>(d, 0), nullptr, P<float>(d, 1), nullptr, nullptr,
                                    nullptr, nullptr, 0, n, n_heads, 0, head_dim, eps, err, s);
    });
}

void qwen_apply_rope_neox(float *x, const float *cos, const float *sin, int seq, int n_heads,
                          int head_dim) {
    const char *fn = "qwen_apply_rope_neox";
    if (!x || !cos || !sin || seq < 0 || n_heads <= 0 || head_dim <= 0 || (head_dim & 1)) {
        fail(fn, LAI_ERR_INVALID, "arguments");
        return;
    }
    const size_t hb = (size_t)head_dim * 4;
    std::vector<Arg> a = {{x, (size_t)n_heads * hb, 0, true, true},
                          {cos, hb, 0, true, false},
                          {sin, hb, 0, true, false}};
    run_op(fn, a, seq, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *err) {
        return lai_qk_norm_rope_f32(P<float>(d, 0), nullptr, nullptr, nullptr, P<float>(d, 1),
                                    P<float>(d, 2), nullptr, n, n, n_heads, 0, head_dim, 0.f,
                                    err, s);
    });
}

void qwen_compute_rope_neox(float *cos, float *sin, const int *pos, int n, int head_dim,
                            float theta) {
    const char *fn = "qwen_compute_rope_neox";
    if (!cos || !sin || !pos || n < 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 512) {
        fail(fn, LAI_ERR_INVALID, "arguments");
        return;
    }
    const size_t hb = (size_t)head_dim * 4;
    std::vector<Arg> a = {{cos, hb, 0, false, true}, {sin, hb, 0, false, true},
                          {pos, 4, 0, true, false}};
    run_op(fn, a, n, [&](cudaStream_t s, int64_t, int64_t m, void **d, int *) {
        return lai_rope_table_f32(P<float>(d, 0), P<float>(d, 1), P<int32_t>(d, 2), m, head_dim,
                                  theta, s);
    });
}

void qwen_swiglu_multiply(float *out, const float *gate_up, int seq, int inter) {
    const char *fn = "qwen_swiglu_multiply";
    if (!out || !gate_up || seq < 0 || inter <= 0) { fail(fn, LAI_ERR_INVALID, "arguments"); return; }
    std::vector<Arg> a = {{out, (size_t)inter * 4, 0, false, true},
                          {gate_up, (size_t)inter * 8, 0, true, false}};
    run_op(fn, a, seq, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *) {
        return lai_swiglu_f32(P<float>(d, 0), P<float>(d, 1), n, inter, s);
    });
}

void qwen_add_inplace(float *x, const float *y, int n) {
    const char *fn = "qwen_add_inplace";
    if (!x || !y || n < 0) { fail(fn, LAI_ERR_INVALID, "arguments"); return; }
    std::vector<Arg> a = {{x, 4, 0, true, true}, {y, 4, 0, true, false}};
    run_op(fn, a, n, [&](cudaStream_t s, int64_t, int64_t m, void **d, int *) {
        return lai_add_f32(P<float>(d, 0), P<float>(d, 1), m, s);
    });
}

void qwen_silu(float *x, int n) {
    const char *fn = "qwen_silu";
    if (!x || n < 0) { fail(fn, LAI_ERR_INVALID, "arguments"); return; }
    std::vector<Arg> a = {{x, 4, 0, true, true}};
    run_op(fn, a, n, [&](cudaStream_t s, int64_t, int64_t m, void **d, int *) {
        return lai_silu_f32(P<float>(d, 0), m, s);
    });
}

void voc_snake_beta(float *x, const float *exp_alpha, const float *inv_exp_beta, int channels,
                    int T) {
    const char *fn = "voc_snake_beta";
    if (!x || !exp_alpha || !inv_exp_beta || channels < 0 || T < 0) {
        fail(fn, LAI_ERR_INVALID, "arguments");
        return;
    }
    if (T == 0) return;
    // rows are channels: the per-channel parameters are chunked with their rows
    std::vector<Arg> a = {{x, (size_t)T * 4, 0, true, true},
                          {exp_alpha, 4, 0, true, false},
                          {inv_exp_beta, 4, 0, true, false}};
    run_op(fn, a, channels, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *) {
        return lai_snake_beta_f32(P<float>(d, 0), P<float>(d, 1), P<float>(d, 2), 1, (int)n, T, s);
    });
}

int lai_staged_add_rmsnorm_bf16(uint16_t *x, const uint16_t *delta, const float *w,
                                uint16_t *y, int64_t rows, int dim, float eps) {
    const char *fn = "lai_staged_add_rmsnorm_bf16";
    if (!x || !delta || !w || !y || rows < 0 || dim <= 0) return fail(fn, LAI_ERR_INVALID, "arguments");
    const size_t rb = (size_t)dim * 2;
    std::vector<Arg> a = {{x, rb, 0, true, true}, {delta, rb, 0, true, false},
                          {w, 0, (size_t)dim * 4, true, false}, {y, rb, 0, false, true}};
    return run_op(fn, a, rows, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *) {
        return lai_add_rmsnorm_bf16(P<uint16_t>(d, 0), P<uint16_t>(d, 1), P<float>(d, 2),
                                    P<uint16_t>(d, 3), n, dim, eps, s);
    });
}

int lai_staged_qk_norm_rope_bf16(uint16_t *q, uint16_t *k, const float *wq, const float *wk,
                                 const float *cos_t, const float *sin_t, const int32_t *pos,
                                 int64_t table_rows, int64_t rows, int n_q_heads, int n_kv_heads,
                                 int head_dim, float eps) {
    const char *fn = "lai_staged_qk_norm_rope_bf16";
    if (!q || rows < 0 || n_q_heads <= 0 || head_dim <= 0 || (head_dim & 1) ||
        (k && n_kv_heads <= 0) || (cos_t && (!sin_t || table_rows <= 0)) ||
        (!cos_t && !wq && !wk))
        return fail(fn, LAI_ERR_INVALID, "arguments");
    const size_t hb = (size_t)head_dim;
    const size_t tb = cos_t ? (size_t)table_rows * hb * 4 : 0;
    std::vector<Arg> a = {{q, (size_t)n_q_heads * hb * 2, 0, true, true},
                          {k, (size_t)(k ? n_kv_heads : 0) * hb * 2, 0, true, true},
                          {wq, 0, hb * 4, true, false},
                          {wk, 0, hb * 4, true, false},
                          {cos_t, 0, tb, true, false},
                          {sin_t, 0, tb, true, false},
                          {pos, 4, 0, true, false}};
    return run_op(fn, a, rows, [&](cudaStream_t s, int64_t r0, int64_t n, void **d, int *err) {
        const float *c = P<float>(d, 4), *sn = P<float>(d, 5);
        int64_t trows = table_rows;
        if (!pos && c) {  // row index is the position: shift the table to this chunk's rows
            c += r0 * head_dim;
            sn += r0 * head_dim;
            trows -= r0;
        }
        return lai_qk_norm_rope_bf16(P<uint16_t>(d, 0), P<uint16_t>(d, 1), P<float>(d, 2),
                                     P<float>(d, 3), c, sn, P<int32_t>(d, 6), trows, n,
                                     n_q_heads, k ? n_kv_heads : 0, head_dim, eps, err, s);
    });
}

int lai_staged_swiglu_bf16(uint16_t *out, const uint16_t *gate_up, int64_t rows, int inter) {
    const char *fn = "lai_staged_swiglu_bf16";
    if (!out || !gate_up || rows < 0 || inter <= 0) return fail(fn, LAI_ERR_INVALID, "arguments");
    std::vector<Arg> a = {{out, (size_t)inter * 2, 0, false, true},
                          {gate_up, (size_t)inter * 4, 0, true, false}};
    return run_op(fn, a, rows, [&](cudaStream_t s, int64_t, int64_t n, void **d, int *) {
        return lai_swiglu_bf16(P<uint16_t>(d, 0), P<uint16_t>(d, 1), n, inter, s);
    });
}

void lai_embed_lookup_bf16(float *dst, const uint16_t *table, int token_id, int dim,
                           int64_t vocab) {
    const char *fn = "lai_embed_lookup_bf16";
    if (!dst || !table || dim <= 0 || token_id < 0 || (vocab > 0 && token_id >= vocab)) {
        fail(fn, vocab > 0 && token_id >= vocab ? LAI_ERR_RANGE : LAI_ERR_INVALID, "arguments");
        return;
    }
    const void *tdev = mapped_device_ptr(table);
    if (!tdev) {
        fail(fn, LAI_ERR_INVALID, "table must be device memory or registered host memory");
        return;
    }
    // Gather row 0 of the one-row view that starts at the requested row.
    const uint16_t *row = static_cast<const uint16_t *>(tdev) + (size_t)token_id * dim;
    Ctx *c = get_ctx(fn);
    if (!c) return;
    const int32_t *ids = c->zero_id;
    std::vector<Arg> a = {{dst, (size_t)dim * 4, 0, false, true}};
    run_op(fn, a, 1, [&](cudaStream_t s, int64_t, int64_t, void **d, int *) {
        return lai_embed_gather_bf16_to_f32(P<float>(d, 0), row, ids, 1, dim, 1, nullptr, s);
    });
}

int lai_register_host_table(const void *table, size_t bytes) {
    if (!table || !bytes) return fail("lai_register_host_table", LAI_ERR_INVALID, "arguments");
    cudaError_t e = cudaHostRegister(const_cast<void *>(table), bytes,
                                     cudaHostRegisterMapped | cudaHostRegisterPortable);
    return e == cudaSuccess ? LAI_OK : cuda_fail("lai_register_host_table", e);
}

int lai_unregister_host_table(const void *table) {
    cudaError_t e = cudaHostUnregister(const_cast<void *>(table));
    return e == cudaSuccess ? LAI_OK : cuda_fail("lai_unregister_host_table", e);
}

int lai_last_error(void) {
    int e = t_last_error;
    t_last_error = LAI_OK;
    return e;
}

void lai_set_stream(void *stream) { t_stream = static_cast<cudaStream_t>(stream); }
void *lai_get_stream(void) { return t_stream; }

int lai_device_error_flags(void) {
    Ctx *c = get_ctx("lai_device_error_flags");
    if (!c) return LAI_ERR_CUDA;
    int flags = 0;
    if (cudaStreamSynchronize(t_stream) != cudaSuccess ||
        cudaMemcpy(&flags, c->derr_direct, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemset(c->derr_direct, 0, sizeof(int)) != cudaSuccess)
        return cuda_fail("lai_device_error_flags", cudaGetLastError());
    return flags;
}

void lai_shutdown(void) {
    int cur = 0;
    cudaGetDevice(&cur);
    for (auto &kv : t_ctx) {
        Ctx &c = kv.second;
        cudaSetDevice(c.device);
        for (int s = 0; s < kStreams; s++)
            if (c.pipe[s]) cudaStreamSynchronize(c.pipe[s]), cudaStreamDestroy(c.pipe[s]);
        for (int s = 0; s < kSlots; s++) {
            if (c.slot[s]) cudaFree(c.slot[s]);
            for (cudaEvent_t ev : {c.in_done[s], c.k_done[s], c.out_done[s]})
                if (ev) cudaEventDestroy(ev);
        }
        if (c.whole) cudaFree(c.whole);
        if (c.derr) cudaFree(c.derr);
        if (c.start_ev) cudaEventDestroy(c.start_ev);
    }
    t_ctx.clear();
    cudaSetDevice(cur);
}

}  // extern "C"

"""Python binding of liblai_kernels.so (ctypes over the C ABI in include/*.h).

The library is the product; this module only marshals torch tensors (device
memory, streams) into the C entry points and raises on a non-zero status. There
is no fallback: if the shared library is missing or CUDA is unavailable the
calls fail loudly.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "liblai_kernels.so")

LAI_OK, LAI_ERR_INVALID, LAI_ERR_CUDA, LAI_ERR_RANGE, LAI_ERR_ALIAS, LAI_ERR_NOMEM, LAI_ERR_TOOBIG = \
    0, -1, -2, -3, -4, -5, -6
LAI_DEVERR_TOKEN_ID, LAI_DEVERR_POSITION, LAI_DEVERR_TIMEOUT, LAI_DEVERR_SMEM_ALIGN = 1, 2, 4, 8

_vp, _i32, _i64, _f32, _u64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_uint64

# name -> (restype, argtypes); every exported symbol of include/*.h
SIGNATURES: dict[str, tuple] = {
    "lai_status_string": (ctypes.c_char_p, [_i32]),
    "lai_version": (_i32, []),
    "lai_rmsnorm_bf16": (_i32, [_vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "lai_rmsnorm_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "lai_add_rmsnorm_bf16": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "lai_add_rmsnorm_f32": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "lai_qk_norm_rope_bf16": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32,
                                     _i32, _f32, _vp, _vp]),
    "lai_qk_norm_rope_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32,
                                    _i32, _f32, _vp, _vp]),
    "lai_rope_table_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "lai_swiglu_bf16": (_i32, [_vp, _vp, _i64, _i32, _vp]),
    "lai_swiglu_f32": (_i32, [_vp, _vp, _i64, _i32, _vp]),
    "lai_swiglu_separate_f32": (_i32, [_vp, _vp, _vp, _i64, _vp]),
    "lai_silu_f32": (_i32, [_vp, _i64, _vp]),
    "lai_add_bf16": (_i32, [_vp, _vp, _i64, _vp]),
    "lai_add_f32": (_i32, [_vp, _vp, _i64, _vp]),
    "lai_embed_gather_bf16": (_i32, [_vp, _vp, _vp, _i64, _i32, _i64, _vp, _vp]),
    "lai_embed_gather_bf16_to_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _i64, _vp, _vp]),
    "lai_snake_beta_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _i64, _vp]),
    "lai_gemv_bf16w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_residual_bf16w_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_swiglu_bf16w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_chain_create": (_i32, [_vp, _vp, _i32]),
    "lai_gemv_chain_run": (_i32, [_vp, _vp, _vp]),
    "lai_gemv_chain_grid": (_i32, [_vp]),
    "lai_gemv_chain_destroy": (None, [_vp]),
    "lai_gemv_f16w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_residual_f16w_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_swiglu_f16w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_i8w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_residual_i8w_f32": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_swiglu_i8w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_f32w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_residual_f32w_f32": (_i32, [_vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "lai_gemv_swiglu_f32w_f32": (_i32, [_vp, _vp, _vp, _f32, _vp, _i64, _i32, _i32, _vp]),
    "lai_quantize_rows_i8_bf16": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp]),
    "lai_logits_mask_range_f32": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _f32, _vp]),
    "lai_prefill_attention_f32": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _f32, _vp]),
    "lai_prefill_attention_rope_f32": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32,
                                              _i32, _f32, _vp, _vp, _i64, _vp]),
    "lai_voc_rvq_gather_f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp]),
    "lai_voc_linear_scale_residual_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                                 _i32, _vp, _vp]),
    "lai_history_append_i32": (_i32, [_vp, _vp, _vp, _i32, _i32, _vp, _vp]),
    "lai_convert_bf16_to_f16": (_i32, [_vp, _vp, _i64, _vp]),
    "lai_decode_attention_scratch_bytes": (ctypes.c_size_t, [_i32, _i32, _i32, _i32]),
    "lai_decode_attention_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                        _i32, _i32, _f32, _vp, _vp, _vp]),
    "lai_decode_attention_qk_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                                           _i32, _i32, _f32, _vp, _vp, _vp, _vp, _i64, _f32,
                                           _vp, _vp, _vp]),
    "lai_sample_topk_f32": (_i32, [_vp, _vp, _i32, _i32, _vp, _vp, _i32, _f32, _f32, _i32, _vp,
                                   _vp]),
    "lai_voc_bigvgan_block_f32": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp,
                                         _vp]),
    "lai_voc_pack_tconv_f32": (_i32, [_vp, _vp, _i32, _i32, _i32, _i32, _vp]),
    "lai_voc_conv1d_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32,
                                  _i32, _vp, _vp]),
    "lai_voc_conv_transpose1d_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32,
                                            _i32, _i32, _i32, _vp, _vp]),
    "lai_voc_final_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
    "lai_voc_convnext_f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _vp, _vp]),
    "lai_voc_resunits_f32": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "lai_voc_pack_conv_f32": (_i32, [_vp, _vp, _i32, _i32, _i32, _vp]),
    "lai_voc_transpose_f32": (_i32, [_vp, _vp, _i32, _i32, _i32, _vp]),
    "lai_synth_normal_bf16": (_i32, [_vp, _i64, _u64, _i64, _f32, _f32, _vp]),
    "lai_synth_normal_f32": (_i32, [_vp, _i64, _u64, _i64, _f32, _f32, _vp]),
    "lai_synth_uniform_i32": (_i32, [_vp, _i64, _u64, _i64, _i32, _i32, _vp]),
    # reference-named drop-ins (lai_qwen_dropin.h)
    "qwen_rms_norm": (None, [_vp, _vp, _vp, _i32, _i32, _f32]),
    "lai_rmsnorm_f32_host_noalloc": (_i32, [_vp, _vp, _vp, _i32, _i32, _f32, _vp]),
    "qwen_rms_norm_per_head": (None, [_vp, _vp, _i32, _i32, _i32, _f32]),
    "qwen_apply_rope_neox": (None, [_vp, _vp, _vp, _i32, _i32, _i32]),
    "qwen_compute_rope_neox": (None, [_vp, _vp, _vp, _i32, _i32, _f32]),
    "qwen_swiglu_multiply": (None, [_vp, _vp, _i32, _i32]),
    "qwen_add_inplace": (None, [_vp, _vp, _i32]),
    "qwen_silu": (None, [_vp, _i32]),
    "voc_snake_beta": (None, [_vp, _vp, _vp, _i32, _i32]),
    "lai_staged_add_rmsnorm_bf16": (_i32, [_vp, _vp, _vp, _vp, _i64, _i32, _f32]),
    "lai_staged_qk_norm_rope_bf16": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32,
                                            _i32, _i32, _f32]),
    "lai_staged_swiglu_bf16": (_i32, [_vp, _vp, _i64, _i32]),
    "lai_embed_lookup_bf16": (None, [_vp, _vp, _i32, _i32, _i64]),
    "lai_register_host_table": (_i32, [_vp, ctypes.c_size_t]),
    "lai_unregister_host_table": (_i32, [_vp]),
    "lai_last_error": (_i32, []),
    "lai_set_stream": (None, [_vp]),
    "lai_get_stream": (_vp, []),
    "lai_device_error_flags": (_i32, []),
    "lai_shutdown": (None, []),
}


class LaiError(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn} failed: {status_string(status)} ({status})")


_LIB: ctypes.CDLL | None = None


def header_symbols() -> list[str]:
    """Function names declared with LAI_API in include/*.h."""
    names = []
    inc = os.path.join(REPO, "include")
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            with open(os.path.join(inc, fn)) as f:
                names += re.findall(r"LAI_API\s+[\w\s\*]+?\b(\w+)\s*\(", f.read())
    return names


def load() -> ctypes.CDLL:
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise FileNotFoundError(
            f"{LIB_PATH} is not built; run `python local-ai-server_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def status_string(status: int) -> str:
    return load().lai_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status != LAI_OK:
        raise LaiError(fn, status)


# ---- torch helpers -------------------------------------------------------------

def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _s(stream):
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def _bf16(t):
    import torch
    assert t.dtype in (torch.bfloat16, torch.int16, torch.uint16), t.dtype
    return _p(t)


def call(name: str, *args) -> int:
    st = getattr(load(), name)(*args)
    check(name, st)
    return st


def rmsnorm(x, w, eps, y=None, stream=None):
    import torch
    y = torch.empty_like(x) if y is None else y
    fn = "lai_rmsnorm_bf16" if x.dtype == torch.bfloat16 else "lai_rmsnorm_f32"
    call(fn, _p(y), _p(x), _p(w), x.shape[0], x.shape[-1], eps, _s(stream))
    return y


def add_rmsnorm(x, delta, w, eps, y=None, stream=None):
    import torch
    y = torch.empty_like(x) if y is None else y
    fn = "lai_add_rmsnorm_bf16" if x.dtype == torch.bfloat16 else "lai_add_rmsnorm_f32"
    call(fn, _p(x), _p(delta), _p(w), _p(y), x.shape[0], x.shape[-1], eps, _s(stream))
    return y


def qk_norm_rope(q, k, wq, wk, cos_t, sin_t, pos, n_q, n_kv, head_dim, eps, err=None,
                 stream=None):
    import torch
    fn = "lai_qk_norm_rope_bf16" if q.dtype == torch.bfloat16 else "lai_qk_norm_rope_f32"
    table_rows = 0 if cos_t is None else cos_t.shape[0]
    call(fn, _p(q), _p(k), _p(wq), _p(wk), _p(cos_t), _p(sin_t), _p(pos), table_rows,
         q.shape[0], n_q, n_kv, head_dim, eps, _p(err), _s(stream))


def rope_table(pos, n, head_dim, theta, stream=None, device="cuda"):
    import torch
    c = torch.empty((n, head_dim), dtype=torch.float32, device=device)
    s = torch.empty_like(c)
    call("lai_rope_table_f32", _p(c), _p(s), _p(pos), n, head_dim, theta, _s(stream))
    return c, s


def swiglu(gate_up, inter, out=None, stream=None):
    import torch
    rows = gate_up.shape[0]
    out = torch.empty((rows, inter), dtype=gate_up.dtype, device=gate_up.device) if out is None else out
    fn = "lai_swiglu_bf16" if gate_up.dtype == torch.bfloat16 else "lai_swiglu_f32"
    call(fn, _p(out), _p(gate_up), rows, inter, _s(stream))
    return out


def swiglu_inplace(gate_up, inter, stream=None):
    """Compact [rows, 2*inter] into its own first rows*inter elements (reference call form)."""
    import torch
    fn = "lai_swiglu_bf16" if gate_up.dtype == torch.bfloat16 else "lai_swiglu_f32"
    call(fn, _p(gate_up), _p(gate_up), gate_up.shape[0], inter, _s(stream))
    return gate_up.view(-1)[: gate_up.shape[0] * inter].view(gate_up.shape[0], inter)


def add(x, y, stream=None):
    import torch
    fn = "lai_add_bf16" if x.dtype == torch.bfloat16 else "lai_add_f32"
    call(fn, _p(x), _p(y), x.numel(), _s(stream))
    return x


def embed_gather(table, ids, to_f32: bool, err=None, stream=None):
    import torch
    n, dim = ids.shape[0], table.shape[1]
    out = torch.empty((n, dim), dtype=torch.float32 if to_f32 else table.dtype, device=ids.device)
    fn = "lai_embed_gather_bf16_to_f32" if to_f32 else "lai_embed_gather_bf16"
    call(fn, _p(out), _p(table), _p(ids), n, dim, table.shape[0], _p(err), _s(stream))
    return out


def snake_beta(x, ea, ieb, stream=None):
    b, c, t = (1, *x.shape) if x.dim() == 2 else x.shape
    call("lai_snake_beta_f32", _p(x), _p(ea), _p(ieb), b, c, t, _s(stream))
    return x


def _wfmt(W, scales):
    """The entry-point suffix for a weight tensor's format: torch.bfloat16 -> bf16w,
    float16 -> f16w, int8 (needs per-row scales) -> i8w, float32 -> f32w."""
    import torch
    fmt = {torch.bfloat16: "bf16w", torch.float16: "f16w", torch.int8: "i8w",
           torch.float32: "f32w"}.get(W.dtype)
    if fmt is None:
        raise TypeError(f"unsupported weight dtype {W.dtype}")
    if (fmt == "i8w") != (scales is not None):
        raise ValueError("INT8 weights need per-row scales (and only they take them)")
    return fmt


def gemv(x, W, norm_w=None, eps=1e-6, y=None, stream=None, scales=None):
    """y[M,N] = W[N,K] @ (RMSNorm(x) if norm_w is given else x), x [M,K] FP32; W BF16, FP16,
    F32, or INT8 with scales [N] (y = (q . x) * scale)."""
    import torch
    M, K = x.shape
    N = W.shape[0]
    y = torch.empty((M, N), dtype=torch.float32, device=x.device) if y is None else y
    fmt = _wfmt(W, scales)
    sc = (_p(scales),) if fmt == "i8w" else ()
    call(f"lai_gemv_{fmt}_f32", _p(y), _p(x), _p(norm_w), eps, _p(W), *sc, M, K, N, _s(stream))
    return y


def gemv_residual(x_res, a, W, stream=None, scales=None):
    """x_res[M,N] += W[N,K] @ a[M,K]."""
    fmt = _wfmt(W, scales)
    sc = (_p(scales),) if fmt == "i8w" else ()
    call(f"lai_gemv_residual_{fmt}_f32", _p(x_res), _p(a), _p(W), *sc, a.shape[0], a.shape[1],
         W.shape[0], _s(stream))
    return x_res


def gemv_swiglu(x, W_gu, norm_w=None, eps=1e-6, out=None, stream=None, scales=None):
    """out[M,I] = silu(W_gu[2j].xn) * W_gu[2j+1].xn, W_gu [2I, K] rows interleaved."""
    import torch
    M, K = x.shape
    inter = W_gu.shape[0] // 2
    out = torch.empty((M, inter), dtype=torch.float32, device=x.device) if out is None else out
    fmt = _wfmt(W_gu, scales)
    sc = (_p(scales),) if fmt == "i8w" else ()
    call(f"lai_gemv_swiglu_{fmt}_f32", _p(out), _p(x), _p(norm_w), eps, _p(W_gu), *sc, M, K,
         inter, _s(stream))
    return out


CHAIN_STORE, CHAIN_RESIDUAL, CHAIN_SWIGLU = 0, 1, 2


class GemvChainOp(ctypes.Structure):
    """lai_gemv_chain_op_t: one fused M = 1 GEMV of a chain (device pointers)."""
    _fields_ = [("w", _vp), ("in_", _vp), ("norm_w", _vp), ("out", _vp), ("n", ctypes.c_int32),
                ("k", ctypes.c_int32), ("epilogue", ctypes.c_int32), ("eps", _f32)]


class GemvChain:
    """A decode step's GEMVs as one persistent kernel (lai_gemv_chain_*). `ops`: a list of
    (kind, W [n, k] BF16, in [k] FP32, norm_w [k] or None, out, eps) with kind one of
    CHAIN_STORE / CHAIN_RESIDUAL / CHAIN_SWIGLU; the tensors must stay alive (the chain
    keeps references) and are read and written in place by every run()."""

    def __init__(self, ops):
        import torch
        self._keep = []
        arr = (GemvChainOp * max(1, len(ops)))()
        for j, (kind, W, x, norm_w, out, eps) in enumerate(ops):
            assert W.dtype == torch.bfloat16 and x.dtype == torch.float32
            arr[j] = GemvChainOp(W.data_ptr(), x.data_ptr(),
                                 norm_w.data_ptr() if norm_w is not None else None, out.data_ptr(),
                                 W.shape[0], W.shape[1], kind, eps)
            self._keep += [W, x, norm_w, out]
        h = _vp()
        call("lai_gemv_chain_create", ctypes.byref(h), arr, len(ops))
        self._h = h
        dev = ops[0][1].device if ops else "cuda"
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)

    @property
    def grid(self) -> int:
        return load().lai_gemv_chain_grid(self._h)

    def run(self, stream=None):
        call("lai_gemv_chain_run", self._h, _p(self.err), _s(stream))

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            load().lai_gemv_chain_destroy(h)
            self._h = None


def quantize_rows_i8(W, stream=None):
    """BF16 W [N, K] -> (INT8 q [N, K], F32 scales [N]): scale = max|row| / 127,
    q = round(w / scale)."""
    import torch
    N, K = W.shape
    q = torch.empty((N, K), dtype=torch.int8, device=W.device)
    scales = torch.empty((N,), dtype=torch.float32, device=W.device)
    call("lai_quantize_rows_i8_bf16", _p(q), _p(scales), _p(W), N, K, _s(stream))
    return q, scales


def convert_bf16_to_f16(W, stream=None):
    """BF16 tensor -> FP16 tensor of the same shape (round to nearest even)."""
    import torch
    out = torch.empty(W.shape, dtype=torch.float16, device=W.device)
    call("lai_convert_bf16_to_f16", _p(out), _p(W), W.numel(), _s(stream))
    return out


def logits_mask_range(logits, lo, hi, keep=-1, value=-1.0e9, stream=None):
    """logits [rows, vocab]: [lo, hi) set to value except column keep (in place)."""
    rows, vocab = (1, logits.shape[0]) if logits.dim() == 1 else logits.shape
    call("lai_logits_mask_range_f32", _p(logits), vocab, rows, lo, hi, keep, value, _s(stream))
    return logits


def history_append(history, history_len, tokens, err=None, stream=None):
    """history [rows, stride] int32, history_len [rows] int32, tokens [rows] int32 (device)."""
    rows, stride = (1, history.shape[0]) if history.dim() == 1 else history.shape
    call("lai_history_append_i32", _p(history), _p(history_len), _p(tokens), rows, stride,
         _p(err), _s(stream))


def prefill_attention(q, k, v, n_heads, n_kv_heads, head_dim, scale=None, out=None,
                      stream=None):
    """Causal self-attention: q [T, H*hd], k / v [T, Hkv*hd] -> out [T, H*hd]."""
    import torch
    T = q.shape[0]
    out = torch.empty_like(q) if out is None else out
    call("lai_prefill_attention_f32", _p(out), _p(q), _p(k), _p(v), T, n_heads, n_kv_heads,
         head_dim, head_dim ** -0.5 if scale is None else scale, _s(stream))
    return out


def prefill_attention_rope(qkv, n_heads, n_kv_heads, head_dim, cos_t, sin_t, scale=None,
                           out=None, stream=None):
    """Causal self-attention with NeoX RoPE on q and k, read from a fused projection output
    qkv [T, (H + 2 Hkv) hd] (q | k | v column blocks) -> out [T, H*hd]."""
    import torch
    T = qkv.shape[0]
    qd, kvd = n_heads * head_dim, n_kv_heads * head_dim
    out = torch.empty((T, qd), dtype=torch.float32, device=qkv.device) if out is None else out
    base, ld = qkv.data_ptr(), qkv.stride(0)
    call("lai_prefill_attention_rope_f32", _p(out), base, base + 4 * qd, base + 4 * (qd + kvd), ld,
         ld, T, n_heads, n_kv_heads, head_dim, head_dim ** -0.5 if scale is None else scale,
         _p(cos_t), _p(sin_t), 0 if cos_t is None else cos_t.shape[0], _s(stream))
    return out


def voc_rvq_gather(codebooks, codes, out=None, err=None, stream=None):
    """codebooks [n_cb, size, dim] F32, codes [T, n_cb] int64 -> [T, n_cb*dim]."""
    import torch
    n_cb, size, dim = codebooks.shape
    T = codes.shape[0]
    out = torch.empty((T, n_cb * dim), dtype=torch.float32, device=codes.device) if out is None else out
    call("lai_voc_rvq_gather_f32", _p(out), _p(codebooks), _p(codes), T, n_cb, size, dim, _p(err),
         _s(stream))
    return out


def voc_linear_scale_residual(x_res, inp, w_packed, bias, gamma, scratch=None, passes=3, err=None,
                              stream=None):
    """x_res [rows, c_out] += gamma * (inp [rows, c_in] . W^T + bias); w_packed from
    voc_pack_conv(W[c_out, c_in, 1])."""
    import torch
    rows, c_in = inp.shape
    c_out = x_res.shape[1]
    if scratch is None:
        scratch = torch.empty(2 * rows * c_in, dtype=torch.float32, device=inp.device)
    call("lai_voc_linear_scale_residual_f32", _p(x_res), _p(inp), _p(scratch), _p(w_packed),
         _p(bias), _p(gamma), rows, c_in, c_out, passes, _p(err), _s(stream))
    return x_res


def decode_attention_scratch(n_seqs, n_heads, n_kv_heads, max_seq, device="cuda"):
    """Zeroed scratch for decode_attention (reusable across calls)."""
    import torch
    nb = load().lai_decode_attention_scratch_bytes(n_seqs, n_heads, n_kv_heads, max_seq)
    return torch.zeros((nb + 15) // 16 * 4, dtype=torch.float32, device=device)


def decode_attention(q, k_new, v_new, k_cache, v_cache, pos, n_heads, n_kv_heads, scratch=None,
                     scale=None, out=None, err=None, stream=None, qk=None):
    """One token per sequence: append k_new/v_new at pos[s] and attend over keys 0..pos[s].
    q [S, H*128]; k_new/v_new [S, Hkv*128]; caches [S, max_seq, Hkv*128].
    qk = (wq, wk, cos_t, sin_t, eps): fold the per-head q/k RMSNorm + NeoX RoPE at pos into the
    same launch (q and k_new are then read raw; the cache receives the transformed key)."""
    import torch
    S, max_seq = k_cache.shape[0], k_cache.shape[1]
    hd = q.shape[1] // n_heads
    if scratch is None:
        scratch = decode_attention_scratch(S, n_heads, n_kv_heads, max_seq, q.device)
    out = torch.empty_like(q) if out is None else out
    sc = hd ** -0.5 if scale is None else scale
    if qk is None:
        call("lai_decode_attention_f32", _p(out), _p(q), _p(k_new), _p(v_new), _p(k_cache),
             _p(v_cache), _p(pos), S, n_heads, n_kv_heads, hd, max_seq, sc, _p(scratch),
             _p(err), _s(stream))
    else:
        wq, wk, cos_t, sin_t, eps = qk
        call("lai_decode_attention_qk_f32", _p(out), _p(q), _p(k_new), _p(v_new), _p(k_cache),
             _p(v_cache), _p(pos), S, n_heads, n_kv_heads, hd, max_seq, sc, _p(wq), _p(wk),
             _p(cos_t), _p(sin_t), 0 if cos_t is None else cos_t.shape[0], eps, _p(scratch),
             _p(err), _s(stream))
    return out


def sample_topk(logits, u, temperature=1.0, top_k=50, history=None, history_len=None,
                penalty=1.0, out=None, stream=None):
    """Per row: repetition penalty (in place on logits) then top-k sampling with draw u[row].
    logits [rows, vocab] F32; history [rows, stride] int32 + history_len [rows]; u [rows]."""
    import torch
    rows, vocab = logits.shape
    out = torch.empty(rows, dtype=torch.int32, device=logits.device) if out is None else out
    stride = history.shape[1] if history is not None else 0
    call("lai_sample_topk_f32", _p(out), _p(logits), vocab, rows, _p(history), _p(history_len),
         stride, penalty, temperature, top_k, _p(u), _s(stream))
    return out


class VocResUnit(ctypes.Structure):
    """lai_voc_resunit_t: device pointers of one ResUnit's parameters."""
    _fields_ = [("snake1_ea", _vp), ("snake1_ieb", _vp), ("conv1_w", _vp), ("conv1_b", _vp),
                ("snake2_ea", _vp), ("snake2_ieb", _vp), ("conv2_w", _vp), ("conv2_b", _vp),
                ("dilation", _i32)]


class VocBigVGANBlock(ctypes.Structure):
    """lai_voc_bigvgan_block_t."""
    _fields_ = [("snake_ea", _vp), ("snake_ieb", _vp), ("tconv_w", _vp), ("tconv_b", _vp),
                ("rate", _i32), ("n_units", _i32), ("units", _vp)]


def voc_pack_tconv(w, stride, stream=None):
    """Reference transposed-conv weight [c_in, c_out, kernel] (kernel = stride or 2 stride) ->
    packed [2, stride, kernel / stride, c_out, c_in]."""
    import torch
    c_in, c_out, kernel = w.shape
    dst = torch.empty((2, stride, kernel // stride, c_out, c_in), dtype=torch.float32,
                      device=w.device)
    call("lai_voc_pack_tconv_f32", _p(dst), _p(w), c_in, c_out, kernel, stride, _s(stream))
    return dst


def voc_block_params(blk):
    """blk: dict with ea, ieb [c_in], w [c_in, c_out, 2r], b [c_out], rate, units (list of
    ResUnit dicts as voc_units takes). Returns (lai_voc_bigvgan_block_t, tensors kept alive)."""
    wp = voc_pack_tconv(blk["w"], blk["rate"])
    arr, keep = voc_units(blk["units"]) if blk["units"] else (None, [])
    st = VocBigVGANBlock(blk["ea"].data_ptr(), blk["ieb"].data_ptr(), wp.data_ptr(),
                         blk["b"].data_ptr(), int(blk["rate"]), len(blk["units"]),
                         ctypes.cast(arr, _vp).value if arr is not None else None)
    return st, [wp, arr, keep, blk]


def voc_bigvgan_block(x, params, c_out, scratch=None, passes=3, err=None, stream=None):
    """x [batch, T, c_in] -> new tensor [batch, (T - 1) rate, c_out]."""
    import torch
    b, t, c_in = (1, *x.shape) if x.dim() == 2 else x.shape
    st = params[0] if isinstance(params, tuple) else params
    t_out = (t - 1) * st.rate
    out = torch.empty((b, t_out, c_out), dtype=torch.float32, device=x.device)
    if scratch is None:
        scratch = torch.empty(2 * b * t * c_in + 4 * b * t_out * c_out, dtype=torch.float32,
                              device=x.device)
    call("lai_voc_bigvgan_block_f32", _p(out), _p(x), _p(scratch), ctypes.byref(st), b, c_in,
         c_out, t, passes, _p(err), _s(stream))
    return out


def voc_conv1d(x, w_packed, bias, c_out, kernel, dilation=1, scratch=None, passes=3, err=None,
               stream=None):
    """Causal conv on x [batch, T, c_in] -> new [batch, T, c_out]; w_packed from voc_pack_conv."""
    import torch
    b, t, c_in = x.shape
    out = torch.empty((b, t, c_out), dtype=torch.float32, device=x.device)
    if scratch is None:
        scratch = torch.empty(2 * b * t * c_in, dtype=torch.float32, device=x.device)
    call("lai_voc_conv1d_f32", _p(out), _p(x), _p(scratch), _p(w_packed), _p(bias), b, c_in, c_out,
         t, kernel, dilation, passes, _p(err), _s(stream))
    return out


def voc_conv_transpose1d(x, w_packed, bias, c_out, kernel, stride, scratch=None, passes=3,
                         err=None, stream=None):
    """Transposed conv on x [batch, T, c_in] -> new [batch, (T + 1) stride - kernel, c_out]."""
    import torch
    b, t, c_in = x.shape
    out = torch.empty((b, (t + 1) * stride - kernel, c_out), dtype=torch.float32, device=x.device)
    if scratch is None:
        scratch = torch.empty(2 * b * t * c_in, dtype=torch.float32, device=x.device)
    call("lai_voc_conv_transpose1d_f32", _p(out), _p(x), _p(scratch), _p(w_packed), _p(bias), b,
         c_in, c_out, t, kernel, stride, passes, _p(err), _s(stream))
    return out


def voc_final(x, ea, ieb, w, bias, out=None, stream=None):
    """SnakeBeta -> conv C -> 1 (k = 7) -> clamp on x [batch, T, C]; returns audio [batch, T]."""
    import torch
    b, t, c = x.shape
    out = torch.empty((b, t), dtype=torch.float32, device=x.device) if out is None else out
    call("lai_voc_final_f32", _p(out), _p(x), _p(ea), _p(ieb), _p(w), _p(bias), b, c, t, _s(stream))
    return out


class VocConvNeXt(ctypes.Structure):
    """lai_voc_convnext_t: device pointers of one ConvNeXt block's parameters."""
    _fields_ = [("dw_w", _vp), ("dw_b", _vp), ("norm_w", _vp), ("norm_b", _vp),
                ("pw1_w", _vp), ("pw1_b", _vp), ("pw2_w", _vp), ("pw2_b", _vp), ("gamma", _vp)]


def voc_convnext_params(p):
    """p: dict of CUDA tensors in the reference's layouts (dw_w [C,1,7], pw1_w [4C,C,1],
    pw2_w [C,4C,1], ...). Returns (lai_voc_convnext_t, tensors kept alive)."""
    w1, w2 = voc_pack_conv(p["pw1_w"]), voc_pack_conv(p["pw2_w"])
    st = VocConvNeXt(p["dw_w"].data_ptr(), p["dw_b"].data_ptr(), p["norm_w"].data_ptr(),
                     p["norm_b"].data_ptr(), w1.data_ptr(), p["pw1_b"].data_ptr(), w2.data_ptr(),
                     p["pw2_b"].data_ptr(), p["gamma"].data_ptr())
    return st, [w1, w2, p]


def voc_convnext(x, params, scratch=None, passes=3, err=None, stream=None):
    """In place on x [batch, T, C]; params from voc_convnext_params()."""
    import torch
    b, t, c = (1, *x.shape) if x.dim() == 2 else x.shape
    if scratch is None:
        scratch = torch.empty(10 * b * t * c, dtype=torch.float32, device=x.device)
    st = params[0] if isinstance(params, tuple) else params
    call("lai_voc_convnext_f32", _p(x), _p(scratch), ctypes.byref(st), b, c, t, passes, _p(err),
         _s(stream))
    return x


def voc_pack_conv(w, stream=None):
    """Reference conv weight [c_out, c_in, k] -> packed [2, k, c_out, c_in] (TF32 hi, lo)."""
    import torch
    c_out, c_in, k = w.shape
    dst = torch.empty((2, k, c_out, c_in), dtype=torch.float32, device=w.device)
    call("lai_voc_pack_conv_f32", _p(dst), _p(w), c_out, c_in, k, _s(stream))
    return dst


def voc_transpose(src, stream=None):
    """[batch, R, C] -> [batch, C, R] (a 2-D tensor is batch 1)."""
    import torch
    b, r, c = (1, *src.shape) if src.dim() == 2 else src.shape
    shape = (c, r) if src.dim() == 2 else (b, c, r)
    dst = torch.empty(shape, dtype=torch.float32, device=src.device)
    call("lai_voc_transpose_f32", _p(dst), _p(src), b, r, c, _s(stream))
    return dst


def voc_units(params, packed=None):
    """params: list of dicts (ea1, ieb1, w1 [C,C,7], b1, ea2, ieb2, w2 [C,C,1], b2, dilation)
    of CUDA tensors. Returns (ctypes array of lai_voc_resunit_t, tensors kept alive)."""
    keep = []
    arr = (VocResUnit * len(params))()
    for i, p in enumerate(params):
        w1 = packed[i][0] if packed else voc_pack_conv(p["w1"])
        w2 = packed[i][1] if packed else voc_pack_conv(p["w2"])
        keep += [w1, w2]
        arr[i] = VocResUnit(p["ea1"].data_ptr(), p["ieb1"].data_ptr(), w1.data_ptr(),
                            p["b1"].data_ptr(), p["ea2"].data_ptr(), p["ieb2"].data_ptr(),
                            w2.data_ptr(), p["b2"].data_ptr(), int(p["dilation"]))
    return arr, keep


def voc_resunits(x, units, scratch=None, passes=3, err=None, stream=None):
    """In place on x [batch, T, C] (channels-last); units from voc_units()."""
    import torch
    b, t, c = (1, *x.shape) if x.dim() == 2 else x.shape
    if scratch is None:
        scratch = torch.empty(4 * b * t * c, dtype=torch.float32, device=x.device)
    arr = units[0] if isinstance(units, tuple) else units
    call("lai_voc_resunits_f32", _p(x), _p(scratch), ctypes.cast(arr, _vp), len(arr), b, c, t,
         passes, _p(err), _s(stream))
    return x


def synth_normal(t, seed, offset=0, mean=0.0, std=1.0, stream=None):
    import torch
    fn = "lai_synth_normal_bf16" if t.dtype == torch.bfloat16 else "lai_synth_normal_f32"
    call(fn, _p(t), t.numel(), seed, offset, mean, std, _s(stream))
    return t


def synth_uniform_i32(t, seed, lo, hi, offset=0, stream=None):
    call("lai_synth_uniform_i32", _p(t), t.numel(), seed, offset, lo, hi, _s(stream))
    return t

"""ctypes access to the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this
module, as the parity checker or as the timed CPU reference. The product library
(local-ai-server_b200/liblai_kernels.so) never loads anything under oracle/.

Libraries (built by oracle/Makefile):
  _build/liblai_oracle.so    restatement of the reference ops, checker flags
  _build/liblai_cpuref.so    the same restatement, reference optimisation tier + OpenMP
  _ref/libvoc_ref_scalar.so  the reference's own voc_snake_beta (src/tts_vocoder_ops.c),
                             scalar sinf build: the SnakeBeta parity oracle
  _ref/libvoc_ref_avx2.so    the same function as shipped (AVX2 fast sin)
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_F = ctypes.POINTER(ctypes.c_float)
_U16 = ctypes.POINTER(ctypes.c_uint16)
_I32 = ctypes.POINTER(ctypes.c_int32)
_I8 = ctypes.POINTER(ctypes.c_int8)
_c_int, _c_float, _c_i64 = ctypes.c_int, ctypes.c_float, ctypes.c_int64


def build() -> None:
    """Compile the oracle and (when the reference source is present) oracle/_ref."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _lib_path(name: str) -> str:
    sub = "_ref" if name.startswith(("libvoc_ref", "libtts_sampling_ref")) else "_build"
    return os.path.join(HERE, sub, name)


_LIBS: dict[str, ctypes.CDLL] = {}


def load(name: str = "liblai_oracle.so") -> ctypes.CDLL:
    if name in _LIBS:
        return _LIBS[name]
    path = _lib_path(name)
    if not os.path.exists(path):
        build()
    lib = ctypes.CDLL(path)
    if name.startswith("liblai_"):
        _declare(lib)
    elif name.startswith("libtts_sampling"):
        lib.tts_apply_repetition_penalty.argtypes = [_F, _c_int, _I32, _c_int, _c_float]
        lib.tts_apply_repetition_penalty.restype = None
        lib.tts_sample_topk.argtypes = [_F, _c_int, _c_float, _c_int]
        lib.tts_sample_topk.restype = _c_int
    else:
        lib.voc_snake_beta.argtypes = [_F, _F, _F, _c_int, _c_int]
        lib.voc_snake_beta.restype = None
        lib.voc_layer_norm_channels.argtypes = [_F, _F, _F, _c_int, _c_int, _c_float]
        lib.voc_layer_norm_channels.restype = None
        lib.voc_gelu.argtypes = [_F, _c_int]
        lib.voc_gelu.restype = None
        lib.voc_conv1d_causal.argtypes = [_F, _F, _F, _F, _c_int, _c_int, _c_int, _c_int,
                                          _c_int, _c_int, _F]
        lib.voc_conv1d_causal.restype = None
        lib.voc_conv_transpose1d.argtypes = [_F, _F, _F, _F, _c_int, _c_int, _c_int, _c_int,
                                             _c_int, _F]
        lib.voc_conv_transpose1d.restype = None
    _LIBS[name] = lib
    return lib


def have_ref() -> bool:
    return os.path.exists(_lib_path("libvoc_ref_scalar.so"))


def _declare(lib: ctypes.CDLL) -> None:
    sig = {
        "oracle_rms_norm": [_F, _F, _F, _c_int, _c_int, _c_float],
        "oracle_rms_norm_per_head": [_F, _F, _c_int, _c_int, _c_int, _c_float],
        "oracle_apply_rope_neox": [_F, _F, _F, _c_int, _c_int, _c_int],
        "oracle_apply_rope_neox_pos": [_F, _F, _F, _I32, _c_int, _c_int, _c_int],
        "oracle_compute_rope_neox": [_F, _F, _I32, _c_int, _c_int, _c_float],
        "oracle_rope_inv_freq": [_F, _c_int, _c_float],
        "oracle_swiglu_multiply": [_F, _F, _c_int, _c_int],
        "oracle_swiglu_separate": [_F, _F, _F, _c_int],
        "oracle_add_inplace": [_F, _F, _c_int],
        "oracle_silu": [_F, _c_int],
        "oracle_snake_beta": [_F, _F, _F, _c_int, _c_int],
        "oracle_embed_gather_bf16_to_f32": [_F, _U16, _I32, _c_int, _c_int],
        "oracle_embed_gather_bf16": [_U16, _U16, _I32, _c_int, _c_int],
        "oracle_rms_norm_bf16": [_U16, _U16, _F, _c_int, _c_int, _c_float],
        "oracle_add_rms_norm_bf16": [_U16, _U16, _F, _U16, _c_int, _c_int, _c_float],
        "oracle_add_rms_norm_f32": [_F, _F, _F, _F, _c_int, _c_int, _c_float],
        "oracle_qk_norm_rope_bf16": [_U16, _U16, _F, _F, _F, _F, _I32, _c_int, _c_int,
                                     _c_int, _c_int, _c_float],
        "oracle_qk_norm_rope_f32": [_F, _F, _F, _F, _F, _F, _I32, _c_int, _c_int, _c_int,
                                    _c_int, _c_float],
        "oracle_swiglu_bf16": [_U16, _U16, _c_int, _c_int],
        "oracle_add_bf16": [_U16, _U16, _c_i64],
        "oracle_layer_chain_f32": [_F, _F, _F, _F, _F, _F, _F, _F, _F, _F, _F, _F, _F,
                                   _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_float],
        "oracle_linear_bf16": [_F, _F, _U16, _c_int, _c_int, _c_int],
        "oracle_linear_f16": [_F, _F, _U16, _c_int, _c_int, _c_int],
        "oracle_causal_attention": [_F, _F, _F, _F, _c_int, _c_int, _c_int, _c_int, _c_float],
        "oracle_linear_i8": [_F, _F, _I8, _F, _c_int, _c_int, _c_int],
        "oracle_linear_f32": [_F, _F, _F, _c_int, _c_int, _c_int],
        "oracle_quantize_rows_i8_bf16": [_I8, _F, _U16, _c_int, _c_int],
        "oracle_f32_to_f16_array": [_U16, _F, _c_i64],
        "oracle_decode_attention": [_F, _F, _F, _F, _I32, _c_int, _c_int, _c_int, _c_int,
                                    _c_int, _c_float],
        "oracle_repetition_penalty": [_F, _c_int, _I32, _c_int, _c_float],
        "oracle_sample_topk": [_F, _c_int, _c_float, _c_int, _c_float, _F, _F],
        "oracle_voc_conv_transpose1d": [_F, _F, _F, _F, _c_int, _c_int, _c_int, _c_int, _c_int],
        "oracle_voc_conv1d_depthwise": [_F, _F, _F, _F, _c_int, _c_int, _c_int],
        "oracle_voc_layer_norm_channels": [_F, _F, _F, _c_int, _c_int, _c_float],
        "oracle_voc_gelu": [_F, _c_i64],
        "oracle_voc_convnext": [_F, _F, _F, _F, _F, _F, _F, _F, _F, _F, _c_int, _c_int, _F],
        "oracle_voc_conv1d_causal": [_F, _F, _F, _F, _c_int, _c_int, _c_int, _c_int, _c_int],
        "oracle_voc_resunit": [_F, _F, _F, _F, _F, _F, _F, _F, _F, _c_int, _c_int, _c_int, _F],
        "oracle_num_threads": [],
        "oracle_set_threads": [_c_int],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = _c_int if name in ("oracle_num_threads", "oracle_sample_topk") else None
    lib.oracle_f32_to_bf16.argtypes = [_c_float]
    lib.oracle_f32_to_bf16.restype = ctypes.c_uint16


def ptr(a: np.ndarray | None, kind=_F):
    """Pointer to a C-contiguous numpy array (None -> NULL)."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(kind)


# ---- numpy helpers for BF16 as uint16 bit patterns ----

def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even F32 -> BF16 bit patterns (same rule as the oracle's C)."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


# ---- thin wrappers (arrays in, arrays out; inputs are never modified) ----

def rms_norm(x, w, eps, lib=None):
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    seq, dim = x.shape
    lib.oracle_rms_norm(ptr(out), ptr(x), ptr(np.ascontiguousarray(w, np.float32)), seq, dim,
                        eps)
    return out


def rms_norm_per_head(x, w, n_heads, head_dim, eps, lib=None):
    lib = lib or load()
    y = np.array(x, np.float32, copy=True, order="C")
    lib.oracle_rms_norm_per_head(ptr(y), ptr(np.ascontiguousarray(w, np.float32)), y.shape[0],
                                 n_heads, head_dim, eps)
    return y


def apply_rope_neox(x, cos_t, sin_t, n_heads, head_dim, lib=None):
    lib = lib or load()
    y = np.array(x, np.float32, copy=True, order="C")
    lib.oracle_apply_rope_neox(ptr(y), ptr(np.ascontiguousarray(cos_t, np.float32)),
                               ptr(np.ascontiguousarray(sin_t, np.float32)), y.shape[0],
                               n_heads, head_dim)
    return y


def compute_rope_neox(pos, head_dim, theta, lib=None):
    lib = lib or load()
    pos = np.ascontiguousarray(pos, np.int32)
    n = pos.shape[0]
    c = np.empty((n, head_dim), np.float32)
    s = np.empty((n, head_dim), np.float32)
    lib.oracle_compute_rope_neox(ptr(c), ptr(s), ptr(pos, _I32), n, head_dim, theta)
    return c, s


def rope_inv_freq(head_dim, theta, lib=None):
    lib = lib or load()
    f = np.empty(head_dim // 2, np.float32)
    lib.oracle_rope_inv_freq(ptr(f), head_dim, theta)
    return f


def swiglu_multiply(gate_up, inter, lib=None):
    lib = lib or load()
    g = np.ascontiguousarray(gate_up, np.float32)
    seq = g.shape[0]
    out = np.empty((seq, inter), np.float32)
    lib.oracle_swiglu_multiply(ptr(out), ptr(g), seq, inter)
    return out


def swiglu_separate(gate, up, lib=None):
    lib = lib or load()
    g = np.ascontiguousarray(gate, np.float32)
    u = np.ascontiguousarray(up, np.float32)
    out = np.empty_like(g)
    lib.oracle_swiglu_separate(ptr(out), ptr(g), ptr(u), g.size)
    return out


def silu(x, lib=None):
    lib = lib or load()
    y = np.array(x, np.float32, copy=True, order="C")
    lib.oracle_silu(ptr(y), y.size)
    return y


def add_inplace(x, y, lib=None):
    lib = lib or load()
    r = np.array(x, np.float32, copy=True, order="C")
    lib.oracle_add_inplace(ptr(r), ptr(np.ascontiguousarray(y, np.float32)), r.size)
    return r


def snake_beta(x, ea, ieb, lib=None):
    lib = lib or load()
    y = np.array(x, np.float32, copy=True, order="C")
    C, T = y.shape[-2], y.shape[-1]
    rows = y.reshape(-1, C, T)
    for b in range(rows.shape[0]):
        lib.oracle_snake_beta(ptr(rows[b]), ptr(np.ascontiguousarray(ea, np.float32)),
                              ptr(np.ascontiguousarray(ieb, np.float32)), C, T)
    return y


def ref_snake_beta(x, ea, ieb, build: str = "scalar"):
    """The reference's own voc_snake_beta (compiled from src/tts_vocoder_ops.c)."""
    lib = load(f"libvoc_ref_{build}.so")
    y = np.array(x, np.float32, copy=True, order="C")
    C, T = y.shape[-2], y.shape[-1]
    rows = y.reshape(-1, C, T)
    ea = np.ascontiguousarray(ea, np.float32)
    ieb = np.ascontiguousarray(ieb, np.float32)
    for b in range(rows.shape[0]):
        lib.voc_snake_beta(ptr(rows[b]), ptr(ea), ptr(ieb), C, T)
    return y


def gather_bf16_to_f32(table, ids, lib=None):
    lib = lib or load()
    table = np.ascontiguousarray(table, np.uint16)
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty((ids.shape[0], table.shape[1]), np.float32)
    lib.oracle_embed_gather_bf16_to_f32(ptr(out), ptr(table, _U16), ptr(ids, _I32), ids.shape[0],
                                        table.shape[1])
    return out


def gather_bf16(table, ids, lib=None):
    lib = lib or load()
    table = np.ascontiguousarray(table, np.uint16)
    ids = np.ascontiguousarray(ids, np.int32)
    out = np.empty((ids.shape[0], table.shape[1]), np.uint16)
    lib.oracle_embed_gather_bf16(ptr(out, _U16), ptr(table, _U16), ptr(ids, _I32), ids.shape[0],
                                 table.shape[1])
    return out


def add_rms_norm_bf16(x, delta, w, eps, lib=None):
    lib = lib or load()
    xo = np.array(x, np.uint16, copy=True, order="C")
    y = np.empty_like(xo)
    seq, dim = xo.shape
    lib.oracle_add_rms_norm_bf16(ptr(xo, _U16), ptr(np.ascontiguousarray(delta, np.uint16), _U16),
                                 ptr(np.ascontiguousarray(w, np.float32)), ptr(y, _U16), seq, dim,
                                 eps)
    return xo, y


def add_rms_norm_f32(x, delta, w, eps, lib=None):
    lib = lib or load()
    xo = np.array(x, np.float32, copy=True, order="C")
    y = np.empty_like(xo)
    seq, dim = xo.shape
    lib.oracle_add_rms_norm_f32(ptr(xo), ptr(np.ascontiguousarray(delta, np.float32)),
                                ptr(np.ascontiguousarray(w, np.float32)), ptr(y), seq, dim, eps)
    return xo, y


def rms_norm_bf16(x, w, eps, lib=None):
    lib = lib or load()
    x = np.ascontiguousarray(x, np.uint16)
    y = np.empty_like(x)
    seq, dim = x.shape
    lib.oracle_rms_norm_bf16(ptr(y, _U16), ptr(x, _U16), ptr(np.ascontiguousarray(w, np.float32)),
                             seq, dim, eps)
    return y


def qk_norm_rope(q, k, wq, wk, cos_t, sin_t, pos, n_q, n_kv, hd, eps, bf16: bool, lib=None):
    """Per-head RMSNorm of q and k, then NeoX RoPE at table row pos[r] (None -> r).
    wq/wk None skip the norm; cos_t None skips RoPE."""
    lib = lib or load()
    kind = _U16 if bf16 else _F
    dt = np.uint16 if bf16 else np.float32
    qo = np.array(q, dt, copy=True, order="C")
    ko = None if k is None else np.array(k, dt, copy=True, order="C")
    c = None if cos_t is None else np.ascontiguousarray(cos_t, np.float32)
    s = None if sin_t is None else np.ascontiguousarray(sin_t, np.float32)
    p = None if pos is None else np.ascontiguousarray(pos, np.int32)
    wqa = None if wq is None else np.ascontiguousarray(wq, np.float32)
    wka = None if wk is None else np.ascontiguousarray(wk, np.float32)
    fn = lib.oracle_qk_norm_rope_bf16 if bf16 else lib.oracle_qk_norm_rope_f32
    fn(ptr(qo, kind), ptr(ko, kind), ptr(wqa), ptr(wka), ptr(c), ptr(s), ptr(p, _I32),
       qo.shape[0], n_q, n_kv, hd, eps)
    return qo, ko


def swiglu_bf16(gate_up, inter, lib=None):
    lib = lib or load()
    g = np.ascontiguousarray(gate_up, np.uint16)
    seq = g.shape[0]
    out = np.empty((seq, inter), np.uint16)
    lib.oracle_swiglu_bf16(ptr(out, _U16), ptr(g, _U16), seq, inter)
    return out


def linear_bf16(x, W, lib=None):
    """out[M,N] = x[M,K] @ W[N,K]^T with W as BF16 bit patterns (linear_bf16's contract)."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    W = np.ascontiguousarray(W, np.uint16)
    M, K = x.shape
    N = W.shape[0]
    out = np.empty((M, N), np.float32)
    lib.oracle_linear_bf16(ptr(out), ptr(x), ptr(W, _U16), M, K, N)
    return out


def causal_attention(q, k, v, n_heads, n_kv_heads, head_dim, scale=None, lib=None):
    """Row t of q [T, H*hd] attends keys 0..t of k / v [T, Hkv*hd]."""
    lib = lib or load()
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.empty_like(q)
    lib.oracle_causal_attention(ptr(out), ptr(q), ptr(k), ptr(v), q.shape[0], n_heads,
                                n_kv_heads, head_dim, head_dim ** -0.5 if scale is None else scale)
    return out


def linear_f16(x, W, lib=None):
    """out[M,N] = x[M,K] @ W[N,K]^T with W as IEEE binary16 bit patterns."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    W = np.ascontiguousarray(W, np.uint16)
    M, K = x.shape
    out = np.empty((M, W.shape[0]), np.float32)
    lib.oracle_linear_f16(ptr(out), ptr(x), ptr(W, _U16), M, K, W.shape[0])
    return out


def linear_i8(x, q, scales, lib=None):
    """out[M,N] = (x[M,K] @ q[N,K]^T) * scales[N] with INT8 q."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    q = np.ascontiguousarray(q, np.int8)
    scales = np.ascontiguousarray(scales, np.float32)
    M, K = x.shape
    out = np.empty((M, q.shape[0]), np.float32)
    lib.oracle_linear_i8(ptr(out), ptr(x), ptr(q, _I8), ptr(scales), M, K, q.shape[0])
    return out


def linear_f32(x, W, lib=None):
    """out[M,N] = x[M,K] @ W[N,K]^T with F32 W."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    W = np.ascontiguousarray(W, np.float32)
    M, K = x.shape
    out = np.empty((M, W.shape[0]), np.float32)
    lib.oracle_linear_f32(ptr(out), ptr(x), ptr(W), M, K, W.shape[0])
    return out


def quantize_rows_i8_bf16(W, lib=None):
    """BF16 bit patterns W [N, K] -> (INT8 q [N, K], F32 scales [N])."""
    lib = lib or load()
    W = np.ascontiguousarray(W, np.uint16)
    N, K = W.shape
    q = np.empty((N, K), np.int8)
    scales = np.empty(N, np.float32)
    lib.oracle_quantize_rows_i8_bf16(ptr(q, _I8), ptr(scales), ptr(W, _U16), N, K)
    return q, scales


def f32_to_f16_bits(x, lib=None):
    """F32 values -> IEEE binary16 bit patterns, round to nearest even."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib.oracle_f32_to_f16_array(ptr(out, _U16), ptr(x), x.size)
    return out


def add_bf16(x, y, lib=None):
    lib = lib or load()
    r = np.array(x, np.uint16, copy=True, order="C")
    lib.oracle_add_bf16(ptr(r, _U16), ptr(np.ascontiguousarray(y, np.uint16), _U16), r.size)
    return r


# ---- vocoder ResUnit, channels-first [C, T] (per batch item) ----

def voc_conv1d_causal(x, w, bias, dilation=1, lib=None):
    """out[o,t] = bias[o] + sum_{c,k} w[o,c,k] * x[c, t - (K-1-k)*dilation] (zero before 0)."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    c_out, c_in, kernel = w.shape
    T = x.shape[-1]
    out = np.empty((c_out, T), np.float32)
    lib.oracle_voc_conv1d_causal(ptr(out), ptr(x), ptr(w),
                                 ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                                 c_in, c_out, T, kernel, dilation)
    return out


def ref_voc_conv1d_causal(x, w, bias, dilation=1, build: str = "scalar"):
    """The reference's own voc_conv1d_causal (compiled from src/tts_vocoder_ops.c, no BLAS:
    left padding, im2col, float dot products)."""
    lib = load(f"libvoc_ref_{build}.so")
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    c_out, c_in, kernel = w.shape
    T = x.shape[-1]
    pad = dilation * (kernel - 1)
    scratch = np.empty(c_in * (T + pad) + c_in * kernel * T, np.float32)
    out = np.empty((c_out, T), np.float32)
    lib.voc_conv1d_causal(ptr(out), ptr(x), ptr(w),
                          ptr(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                          c_in, c_out, T, kernel, dilation, 1, ptr(scratch))
    return out


def voc_resunit(x, p, dilation, lib=None):
    """run_resunit on x [C, T] (or [B, C, T]); p: dict of ea1, ieb1, w1 [C,C,7], b1, ea2,
    ieb2, w2 [C,C,1], b2 in the reference's layouts."""
    lib = lib or load()
    y = np.array(x, np.float32, copy=True, order="C")
    C, T = y.shape[-2], y.shape[-1]
    rows = y.reshape(-1, C, T)
    scratch = np.empty(2 * C * T, np.float32)
    q = {k: np.ascontiguousarray(v, np.float32) for k, v in p.items()}
    for b in range(rows.shape[0]):
        lib.oracle_voc_resunit(ptr(rows[b]), ptr(q["ea1"]), ptr(q["ieb1"]), ptr(q["w1"]),
                               ptr(q["b1"]), ptr(q["ea2"]), ptr(q["ieb2"]), ptr(q["w2"]),
                               ptr(q["b2"]), C, T, dilation, ptr(scratch))
    return y


def ref_voc_resunit(x, p, dilation, build: str = "scalar"):
    """run_resunit's sequence (src/tts_vocoder.c:540-583) built from the reference's own
    compiled voc_snake_beta and voc_conv1d_causal (the k = 1 conv through the same
    function, which equals its naive pointwise loop term for term)."""
    y = np.array(x, np.float32, copy=True, order="C")
    C, T = y.shape[-2], y.shape[-1]
    rows = y.reshape(-1, C, T)
    for b in range(rows.shape[0]):
        r = rows[b].copy()
        s = ref_snake_beta(rows[b], p["ea1"], p["ieb1"], build)
        h = ref_voc_conv1d_causal(s, p["w1"], p["b1"], dilation, build)
        h = ref_snake_beta(h, p["ea2"], p["ieb2"], build)
        rows[b] = ref_voc_conv1d_causal(h, p["w2"], p["b2"], 1, build) + r
    return y


def decode_attention(q, k_cache, v_cache, pos, n_heads, n_kv_heads, head_dim, scale=None,
                     lib=None):
    """q [S, H*hd]; caches [S, max_seq, Hkv*hd]; attends keys 0..pos[s]. Returns [S, H*hd]."""
    lib = lib or load()
    q = np.ascontiguousarray(q, np.float32)
    k_cache = np.ascontiguousarray(k_cache, np.float32)
    v_cache = np.ascontiguousarray(v_cache, np.float32)
    pos = np.ascontiguousarray(pos, np.int32)
    S, max_seq = k_cache.shape[0], k_cache.shape[1]
    out = np.empty((S, n_heads * head_dim), np.float32)
    scale = head_dim ** -0.5 if scale is None else scale
    lib.oracle_decode_attention(ptr(out), ptr(q), ptr(k_cache), ptr(v_cache), ptr(pos, _I32), S,
                                n_heads, n_kv_heads, head_dim, max_seq, scale)
    return out


# ---- token sampling (src/tts_sampling.c) ----

def repetition_penalty(logits, history, penalty, lib=None):
    lib = lib or load()
    y = np.array(logits, np.float32, copy=True, order="C")
    h = np.ascontiguousarray(history, np.int32)
    lib.oracle_repetition_penalty(ptr(y), y.size, ptr(h, _I32), h.size, penalty)
    return y


def sample_topk(logits, temperature, top_k, u, lib=None):
    """(token, margin, sum): tts_sample_topk's choice for the uniform draw u, the distance of
    r = u * sum from the nearest cumulative boundary, and the softmax denominator."""
    lib = lib or load()
    y = np.ascontiguousarray(logits, np.float32)
    m, sm = ctypes.c_float(), ctypes.c_float()
    tok = lib.oracle_sample_topk(ptr(y), y.size, temperature, top_k, np.float32(u),
                                 ctypes.byref(m), ctypes.byref(sm))
    return tok, m.value, sm.value


def have_ref_sampling() -> bool:
    return os.path.exists(_lib_path("libtts_sampling_ref.so"))


def ref_rand_draw(seed: int) -> float:
    """The u that tts_sample_topk computes from libc's first rand() after srand(seed):
    (float)rand() / (float)RAND_MAX in float arithmetic (src/tts_sampling.c:92)."""
    libc = ctypes.CDLL(None)
    libc.srand(ctypes.c_uint(seed))
    x = libc.rand()
    return float(np.float32(x) / np.float32(2147483647))


def ref_sample_topk(logits, temperature, top_k, seed: int):
    """The reference's own tts_sample_topk (compiled from src/tts_sampling.c), its rand()
    seeded with srand(seed) just before the call."""
    lib = load("libtts_sampling_ref.so")
    y = np.array(logits, np.float32, copy=True, order="C")
    libc = ctypes.CDLL(None)
    libc.srand(ctypes.c_uint(seed))
    return lib.tts_sample_topk(ptr(y), y.size, temperature, top_k)


def ref_repetition_penalty(logits, history, penalty):
    lib = load("libtts_sampling_ref.so")
    y = np.array(logits, np.float32, copy=True, order="C")
    h = np.ascontiguousarray(history, np.int32)
    lib.tts_apply_repetition_penalty(ptr(y), y.size, ptr(h, _I32), h.size, penalty)
    return y


# ---- ConvNeXt block (channels-first [C, T] per batch item) ----
CONVNEXT_KEYS = ("dw_w", "dw_b", "norm_w", "norm_b", "pw1_w", "pw1_b", "pw2_w", "pw2_b", "gamma")


def voc_convnext(x, p, lib=None):
    """run_convnext on x [C, T] or [B, C, T]; p: dw_w [C,1,7], dw_b, norm_w, norm_b,
    pw1_w [4C,C,1], pw1_b, pw2_w [C,4C,1], pw2_b, gamma."""
    lib = lib or load()
    y = np.array(x, np.float32, copy=True, order="C")
    C, T = y.shape[-2], y.shape[-1]
    rows = y.reshape(-1, C, T)
    q = [np.ascontiguousarray(p[k], np.float32) for k in CONVNEXT_KEYS]
    scratch = np.empty(5 * C * T, np.float32)
    for b in range(rows.shape[0]):
        lib.oracle_voc_convnext(ptr(rows[b]), *[ptr(a) for a in q], C, T, ptr(scratch))
    return y


def ref_voc_convnext(x, p, build: str = "scalar"):
    """run_convnext's sequence (src/tts_vocoder.c:463-533) composed from the reference's own
    compiled voc_conv1d_causal (depthwise branch, and k = 1 for the pointwise convs),
    voc_layer_norm_channels and voc_gelu."""
    lib = load(f"libvoc_ref_{build}.so")
    y = np.array(x, np.float32, copy=True, order="C")
    C, T = y.shape[-2], y.shape[-1]
    rows = y.reshape(-1, C, T)
    f = lambda a: np.ascontiguousarray(a, np.float32)  # noqa: E731
    for b in range(rows.shape[0]):
        r = rows[b].copy()
        xin = rows[b].copy()
        dw = np.empty((C, T), np.float32)
        scratch = np.empty(C * (T + 6) + 16, np.float32)
        lib.voc_conv1d_causal(ptr(dw), ptr(xin), ptr(f(p["dw_w"])), ptr(f(p["dw_b"])), C, C, T, 7,
                              1, C, ptr(scratch))
        lib.voc_layer_norm_channels(ptr(dw), ptr(f(p["norm_w"])), ptr(f(p["norm_b"])), C, T, 1e-6)
        h = ref_voc_conv1d_causal(dw, p["pw1_w"], p["pw1_b"], 1, build)
        lib.voc_gelu(ptr(h), h.size)
        out = ref_voc_conv1d_causal(h, p["pw2_w"], p["pw2_b"], 1, build)
        rows[b] = out * f(p["gamma"])[:, None] + r
    return y


# ---- BigVGAN block: SnakeBeta -> ConvTranspose1d (k = 2r, stride r) -> 3 ResUnits ----

def voc_conv_transpose1d(x, w, bias, stride, lib=None):
    """x [c_in, T], w [c_in, c_out, kernel] -> [c_out, (T + 1) * stride - kernel]."""
    lib = lib or load()
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    c_in, c_out, kernel = w.shape
    T = x.shape[-1]
    out = np.empty((c_out, (T + 1) * stride - kernel), np.float32)
    lib.oracle_voc_conv_transpose1d(ptr(out), ptr(x), ptr(w), ptr(np.ascontiguousarray(bias, np.float32)),
                                    c_in, c_out, T, kernel, stride)
    return out


def ref_voc_conv_transpose1d(x, w, bias, stride, build: str = "scalar"):
    """The reference's own voc_conv_transpose1d (compiled, no BLAS: scatter-add loop)."""
    lib = load(f"libvoc_ref_{build}.so")
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    c_in, c_out, kernel = w.shape
    T = x.shape[-1]
    out = np.empty((c_out, (T + 1) * stride - kernel), np.float32)
    lib.voc_conv_transpose1d(ptr(out), ptr(x), ptr(w), ptr(np.ascontiguousarray(bias, np.float32)),
                             c_in, c_out, T, kernel, stride, None)
    return out


def voc_bigvgan_block(x, blk, lib=None):
    """One block of tts_vocoder_run (src/tts_vocoder.c:709-728) on x [c_in, T] or [B, c_in, T]:
    snake (blk["ea"], blk["ieb"]), transposed conv (blk["w"] [c_in, c_out, 2r], blk["b"],
    stride blk["rate"]), then the ResUnits blk["units"] (dicts as voc_resunit's, with
    "dilation")."""
    y = np.asarray(x, np.float32)
    batch = y.reshape(-1, y.shape[-2], y.shape[-1])
    outs = []
    for b in range(batch.shape[0]):
        s = snake_beta(batch[b], blk["ea"], blk["ieb"], lib)
        h = voc_conv_transpose1d(s, blk["w"], blk["b"], blk["rate"], lib)
        for u in blk["units"]:
            h = voc_resunit(h, {k: v for k, v in u.items() if k != "dilation"}, u["dilation"], lib)
        outs.append(h)
    return np.stack(outs)


# ---- the vocoder's front: RVQ decode -> pre_conv -> pre-transformer ----

def voc_front(p, codes, lib=None, linear=None):
    """tts_vocoder_run stages 1-3 (src/tts_vocoder.c:589-640) restated from the oracle's
    functions: rvq_decode (:428-455, the 16 projected codebook rows summed in codebook order),
    voc_conv1d_causal pre_conv (:612-616, channels-first as the reference runs it), then
    voc_pre_transformer (src/tts_vocoder_xfmr.c:126-225) in [T, C]. p: numpy arrays in the
    reference's layouts (codebooks [16, 2048, 256], proj [16, 512, 256], pre_w [1024, 512, 3],
    pre_b, in_w [512, 1024], in_b, layers: in_norm, wq / wk / wv [1024, 512], wo [512, 1024],
    attn_ls, post_norm, gate / up [1024, 512], down [512, 1024], mlp_ls; final_norm,
    out_w [1024, 512], out_b); codes [T, 16]. linear(x, W) defaults to linear_f32 (the
    reference's linear_f32: out = x . W^T). Returns [T, 1024]."""
    lib = lib or load()
    lin = linear or (lambda x, W: linear_f32(x, W, lib=lib))
    codes = np.asarray(codes)
    T = codes.shape[0]
    rvq = np.zeros((T, p["proj"].shape[1]), np.float32)
    for cb in range(p["codebooks"].shape[0]):
        rvq += lin(p["codebooks"][cb][codes[:, cb]], p["proj"][cb])
    pre = voc_conv1d_causal(np.ascontiguousarray(rvq.T), p["pre_w"], p["pre_b"], lib=lib)
    x = lin(np.ascontiguousarray(pre.T), p["in_w"]) + p["in_b"]
    hd = 64
    heads = p["layers"][0]["wq"].shape[0] // hd
    cos_t, sin_t = compute_rope_neox(np.arange(T, dtype=np.int32), hd, 10000.0, lib=lib)
    for L in p["layers"]:
        xn = rms_norm(x, L["in_norm"], 1e-5, lib=lib)
        q = apply_rope_neox(lin(xn, L["wq"]), cos_t, sin_t, heads, hd, lib=lib)
        k = apply_rope_neox(lin(xn, L["wk"]), cos_t, sin_t, heads, hd, lib=lib)
        a = causal_attention(q, k, lin(xn, L["wv"]), heads, heads, hd, lib=lib)
        x = add_inplace(x, lin(a, L["wo"]) * L["attn_ls"], lib=lib)
        xn = rms_norm(x, L["post_norm"], 1e-5, lib=lib)
        ffn = swiglu_separate(lin(xn, L["gate"]), lin(xn, L["up"]), lib=lib)
        x = add_inplace(x, lin(ffn, L["down"]) * L["mlp_ls"], lib=lib)
    x = rms_norm(x, p["final_norm"], 1e-5, lib=lib)
    return lin(x, p["out_w"]) + p["out_b"]

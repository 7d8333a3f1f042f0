"""The C ABI library: loads, exports what include/*.h declares, rejects bad arguments.

CPU only. The argument checks below return before any CUDA call, so they run
without a GPU; no kernel is launched here.
"""
import ctypes
import subprocess

import pytest

import lai
from conftest import arena_ptr

V = ctypes.c_void_p


def test_library_loads_and_reports_version():
    lib = lai.load()
    assert lib.lai_version() >= 100
    assert lai.status_string(lai.LAI_ERR_ALIAS) == "unsupported overlap of output and input"


def test_exports_every_header_symbol():
    declared = set(lai.header_symbols())
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", lai.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert declared <= exported, sorted(declared - exported)
    # the binding covers exactly the header
    assert declared == set(lai.SIGNATURES), sorted(declared ^ set(lai.SIGNATURES))


def test_no_internal_symbols_leak():
    out = subprocess.run(["nm", "-D", "--defined-only", lai.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert not [s for s in exported if s.startswith("_ZN3lai")]


def test_oracle_is_not_linked_into_the_product():
    out = subprocess.run(["nm", "-D", lai.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    assert "oracle_" not in out
    deps = subprocess.run(["ldd", lai.LIB_PATH], capture_output=True, text=True).stdout
    assert "lai_oracle" not in deps and "cpuref" not in deps


class _Arena:
    """A(off): a pointer `off` bytes into a real, zeroed 64 MiB allocation (conftest)."""

    def __call__(self, off):
        return arena_ptr(off)


A = _Arena()


class _P:
    """P: a non-NULL pointer into the arena; the checks below fail before any use."""

    @property
    def _as_parameter_(self):
        return arena_ptr(16)


P = _P()


def chain_create(lib, **kw):
    """lai_gemv_chain_create on one op (arena pointers) with fields overridden by kw."""
    op = dict(w=A(1 << 20).value, in_=A(4096).value, norm_w=None, out=A(1 << 16).value, n=8,
              k=256, epilogue=lai.CHAIN_STORE, eps=1e-6)
    op.update(kw)
    arr = (lai.GemvChainOp * 1)(lai.GemvChainOp(**op))
    h = ctypes.c_void_p()
    st = lib.lai_gemv_chain_create(ctypes.byref(h), arr, 1)
    if h.value:
        lib.lai_gemv_chain_destroy(h)
    return st


@pytest.mark.parametrize("call, want", [
    (lambda l: l.lai_rmsnorm_bf16(P, P, P, -1, 1024, 1e-6, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_rmsnorm_f32(P, None, P, 4, 1024, 1e-6, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_rmsnorm_f32(P, P, P, 4, 0, 1e-6, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_add_rmsnorm_bf16(A(4096), P, P, A(4096), 4, 256, 1e-6, None), lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_qk_norm_rope_bf16(P, None, None, None, None, None, None, 0, 4, 16, 8, 128,
                                       1e-6, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_qk_norm_rope_f32(P, None, P, None, None, None, None, 0, 4, 16, 8, 127,
                                      1e-6, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_qk_norm_rope_f32(P, None, None, None, P, None, None, 8, 4, 16, 8, 128,
                                      1e-6, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_swiglu_bf16(A(4096 + 2), A(4096), 4, 64, None), lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_swiglu_f32(P, P, 4, 0, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_add_f32(A(4096), A(4096 + 4), 64, None), lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_embed_gather_bf16(P, P, P, 4, 1024, 0, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_snake_beta_f32(P, P, None, 1, 4, 16, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_rope_table_f32(P, P, None, 4, 1024, 1e6, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_synth_uniform_i32(P, 4, 1, 0, 5, 5, None), lai.LAI_ERR_INVALID),
    # decode attention: head_dim other than 128, heads not a multiple of kv heads, group of 3
    (lambda l: l.lai_decode_attention_f32(P, P, P, P, P, P, P, 1, 16, 8, 64, 100, 0.1, P, None,
                                          None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_decode_attention_f32(P, P, P, P, P, P, P, 1, 12, 4, 128, 100, 0.1, P, None,
                                          None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_decode_attention_f32(A(4096), P, P, P, A(4096), P, P, 1, 16, 8, 128, 100,
                                          0.1, P, None, None), lai.LAI_ERR_ALIAS),
    # sampling: empty vocab; history without lengths; shared memory beyond 200 KiB
    (lambda l: l.lai_sample_topk_f32(P, P, 0, 1, None, None, 0, 1.0, 1.0, 5, P, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_sample_topk_f32(P, P, 100, 1, P, None, 4, 1.0, 1.0, 5, P, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_sample_topk_f32(P, P, 1 << 22, 1, None, None, 0, 1.0, 1.0, 1 << 20, P, None),
     lai.LAI_ERR_TOOBIG),
    # vocoder: passes other than 1 / 3; channels not a multiple of 32; unsupported ConvNeXt
    # width; a BigVGAN block needs T >= 2; packers need their weights
    (lambda l: l.lai_voc_resunits_f32(P, P, P, 1, 1, 96, 128, 2, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_resunits_f32(P, P, P, 1, 1, 80, 128, 3, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_convnext_f32(P, P, P, 1, 300, 64, 3, None, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_bigvgan_block_f32(P, P, P, None, 1, 64, 32, 10, 3, None, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_pack_conv_f32(P, None, 8, 8, 7, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_pack_tconv_f32(P, P, 8, 8, 3, 2, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_conv1d_f32(P, P, P, P, P, 1, 48, 64, 10, 7, 1, 3, None, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_conv_transpose1d_f32(P, P, P, P, P, 1, 64, 64, 10, 3, 2, 3, None, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_final_f32(P, P, P, P, P, None, 1, 96, 100, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_voc_transpose_f32(A(4096), A(4096 + 8), 1, 4, 4, None), lai.LAI_ERR_ALIAS),
    # decode GEMVs: output overlapping input; K beyond the staged maximum
    (lambda l: l.lai_gemv_bf16w_f32(A(256), A(256), None, 1e-6, P, 1, 64, 8, None),
     lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_gemv_bf16w_f32(A(256), A(1 << 24), None, 1e-6, P, 1, 60000, 8, None),
     lai.LAI_ERR_TOOBIG),
    # other weight formats: INT8 needs its scales; odd SwiGLU width; quantizer / converter
    (lambda l: l.lai_gemv_i8w_f32(P, A(1 << 20), None, 1e-6, P, None, 1, 64, 8, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_gemv_swiglu_f16w_f32(P, A(1 << 20), None, 1e-6, P, 1, 64, 0, None),
     lai.LAI_ERR_INVALID),
    (lambda l: l.lai_gemv_residual_f32w_f32(A(256), A(256), P, 1, 64, 8, None), lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_quantize_rows_i8_bf16(P, P, P, 4, 0, None), lai.LAI_ERR_INVALID),
    (lambda l: l.lai_quantize_rows_i8_bf16(A(4096), A(1 << 20), A(4096 + 16), 4, 64, None),
     lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_convert_bf16_to_f16(A(4096), A(4096 + 2), 64, None), lai.LAI_ERR_ALIAS),
    # GEMV chain: NULL table; k not a multiple of 256; a row beyond one stage; odd SwiGLU
    # rows; an output over its input (all rejected before any device call)
    (lambda l: l.lai_gemv_chain_create(ctypes.byref(ctypes.c_void_p()), None, 1), lai.LAI_ERR_INVALID),
    (lambda l: chain_create(l, k=100), lai.LAI_ERR_INVALID),
    (lambda l: chain_create(l, k=8192), lai.LAI_ERR_TOOBIG),
    (lambda l: chain_create(l, epilogue=lai.CHAIN_SWIGLU, n=7), lai.LAI_ERR_INVALID),
    (lambda l: chain_create(l, out=A(4096 + 16).value), lai.LAI_ERR_ALIAS),
    (lambda l: l.lai_gemv_chain_run(None, P, None), lai.LAI_ERR_INVALID),
])
def test_argument_checks(call, want):
    assert call(lai.load()) == want


@pytest.mark.parametrize("call", [
    lambda l: l.lai_rmsnorm_bf16(P, P, P, 0, 1024, 1e-6, None),
    lambda l: l.lai_swiglu_f32(P, P, 0, 64, None),
    lambda l: l.lai_add_bf16(P, P, 0, None),
    lambda l: l.lai_snake_beta_f32(P, P, P, 0, 4, 16, None),
])
def test_empty_inputs_are_no_ops(call):
    assert call(lai.load()) == lai.LAI_OK

"""Vocoder ConvNeXt block against the oracle's run_convnext.

run_convnext (src/tts_vocoder.c:463-533): depthwise causal conv k=7, LayerNorm over
channels, pointwise C -> 4C + GELU, pointwise 4C -> C, layer scale, residual. Device:
channels-last [B, T, C]; oracle: the reference's [C, T] per item.
Tolerance, max |d| / max(1, |ref|): 1e-5 with passes = 3, 1e-2 with passes = 1.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_BF16, TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_block(C, rng):
    f = lambda a: np.asarray(a, np.float32)  # noqa: E731
    return {"dw_w": f(rng.standard_normal((C, 1, 7)) / np.sqrt(7)), "dw_b": f(rng.normal(0, 0.1, C)),
            "norm_w": f(1 + rng.normal(0, 0.1, C)), "norm_b": f(rng.normal(0, 0.1, C)),
            "pw1_w": f(rng.standard_normal((4 * C, C, 1)) / np.sqrt(C)),
            "pw1_b": f(rng.normal(0, 0.1, 4 * C)),
            "pw2_w": f(rng.standard_normal((C, 4 * C, 1)) / np.sqrt(4 * C)),
            "pw2_b": f(rng.normal(0, 0.1, C)), "gamma": f(rng.normal(0, 0.3, C))}


def run_device(x_ct, p, passes):
    dp = {k: torch.from_numpy(v).to(DEV) for k, v in p.items()}
    params = lai.voc_convnext_params(dp)
    x = torch.from_numpy(x_ct).to(DEV).transpose(1, 2).contiguous()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    lai.voc_convnext(x, params, passes=passes, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return x.transpose(1, 2).contiguous().cpu().numpy()


# (batch, C, T): the reference's C = 1024; smaller widths; T below the 7-tap window and below
# one 128-row tile; ragged tiles; batch > 1 (no tap may read the previous item's rows)
@pytest.mark.parametrize("B,C,T", [(1, 1024, 150), (2, 256, 300), (1, 128, 5), (3, 512, 129),
                                   (1, 2048, 40)])
def test_convnext_f32(B, C, T):
    rng = np.random.default_rng(C + T)
    p = make_block(C, rng)
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    assert max_rel_err(run_device(x, p, 3), oracle.voc_convnext(x, p)) <= TOL_F32


def test_convnext_tf32():
    rng = np.random.default_rng(3)
    p = make_block(1024, rng)
    x = rng.standard_normal((2, 1024, 200)).astype(np.float32)
    assert max_rel_err(run_device(x, p, 1), oracle.voc_convnext(x, p)) <= TOL_BF16


@pytest.mark.skipif(not oracle.have_ref(), reason="reference vocoder ops not built")
def test_convnext_matches_reference_functions():
    # the block composed from the reference's own compiled voc_conv1d_causal (depthwise and
    # pointwise), voc_layer_norm_channels and voc_gelu (scalar build)
    rng = np.random.default_rng(8)
    p = make_block(256, rng)
    x = rng.standard_normal((1, 256, 180)).astype(np.float32)
    assert max_rel_err(run_device(x, p, 3), oracle.ref_voc_convnext(x, p)) <= TOL_F32


def test_convnext_argument_checks():
    L = lai.load()
    import ctypes
    x = torch.zeros(1, 64, 256, device=DEV)
    s = torch.zeros(10 * 64 * 256, device=DEV)
    p = lai.voc_convnext_params({k: torch.from_numpy(v).to(DEV)
                                 for k, v in make_block(256, np.random.default_rng(0)).items()})
    f = L.lai_voc_convnext_f32
    ref = ctypes.byref(p[0])
    assert f(lai._p(x), lai._p(s), ref, 1, 300, 64, 3, None, None) == lai.LAI_ERR_INVALID
    assert f(lai._p(x), lai._p(s), ref, 1, 256, 64, 2, None, None) == lai.LAI_ERR_INVALID
    assert f(lai._p(x), lai._p(x), ref, 1, 256, 64, 3, None, None) == lai.LAI_ERR_ALIAS
    assert f(lai._p(x), lai._p(s), ref, 0, 256, 64, 3, None, None) == lai.LAI_OK

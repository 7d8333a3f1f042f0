"""Vocoder BigVGAN block (SnakeBeta -> ConvTranspose1d k = 2r, stride r -> ResUnits) against
the oracle and the reference's own compiled functions.

tts_vocoder_run's block loop (src/tts_vocoder.c:709-728) with voc_conv_transpose1d
(src/tts_vocoder_ops.c:153-221). The transposed conv alone (no ResUnits) is held to
max |d| / max(1, |ref|) <= 1e-5; a whole block (3 chained ResUnits, whose perturbation gain
is above 1) to twice the reference F32 code's own drift from the double-precision oracle.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_F32, max_rel_err
from test_gpu_resunit import make_unit

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_block(c_in, c_out, rate, n_units, rng):
    f = lambda a: np.asarray(a, np.float32)  # noqa: E731
    return {"ea": f(np.exp(rng.normal(0, 0.1, c_in))), "ieb": f(1 / np.exp(rng.normal(0, 0.1, c_in))),
            "w": f(rng.standard_normal((c_in, c_out, 2 * rate)) / np.sqrt(2 * c_in)),
            "b": f(rng.normal(0, 0.1, c_out)), "rate": rate,
            "units": [make_unit(c_out, d, rng) for d in (1, 3, 9)[:n_units]]}


def run_device(x_ct, blk, c_out, passes=3):
    dev = {k: (torch.from_numpy(v).to(DEV) if isinstance(v, np.ndarray) else v)
           for k, v in blk.items() if k != "units"}
    dev["units"] = [{k: (torch.from_numpy(v).to(DEV) if isinstance(v, np.ndarray) else v)
                     for k, v in u.items()} for u in blk["units"]]
    params = lai.voc_block_params(dev)
    x = torch.from_numpy(x_ct).to(DEV).transpose(1, 2).contiguous()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = lai.voc_bigvgan_block(x, params, c_out, passes=passes, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.transpose(1, 2).contiguous().cpu().numpy()


# (batch, c_in, c_out, T, rate): the reference's rates 8, 5, 4, 3; channel halving as in the
# decoder; T below and across a 128-row tile
@pytest.mark.parametrize("B,c_in,c_out,T,rate", [(1, 64, 32, 50, 8), (2, 96, 64, 140, 5),
                                                  (1, 192, 96, 33, 4), (2, 256, 128, 129, 3),
                                                  (1, 1536, 768, 20, 8)])
def test_transposed_conv_f32(B, c_in, c_out, T, rate):
    rng = np.random.default_rng(c_in + T + rate)
    blk = make_block(c_in, c_out, rate, 0, rng)
    x = rng.standard_normal((B, c_in, T)).astype(np.float32)
    got = run_device(x, blk, c_out)
    assert got.shape == (B, c_out, (T - 1) * rate)
    assert max_rel_err(got, oracle.voc_bigvgan_block(x, blk)) <= TOL_F32


@pytest.mark.skipif(not oracle.have_ref(), reason="reference vocoder ops not built")
def test_transposed_conv_matches_reference_functions():
    rng = np.random.default_rng(21)
    blk = make_block(64, 32, 5, 0, rng)
    x = rng.standard_normal((1, 64, 60)).astype(np.float32)
    s = oracle.ref_snake_beta(x[0], blk["ea"], blk["ieb"])
    ref = oracle.ref_voc_conv_transpose1d(s, blk["w"], blk["b"], 5)
    assert max_rel_err(run_device(x, blk, 32)[0], ref) <= TOL_F32


@pytest.mark.skipif(not oracle.have_ref(), reason="reference vocoder ops not built")
@pytest.mark.parametrize("c_in,c_out,rate", [(192, 96, 3), (96, 64, 8)])
def test_block_as_accurate_as_reference_f32(c_in, c_out, rate):
    rng = np.random.default_rng(c_in * rate)
    blk = make_block(c_in, c_out, rate, 3, rng)
    x = rng.standard_normal((1, c_in, 40)).astype(np.float32)
    ora = oracle.voc_bigvgan_block(x, blk)
    h = oracle.ref_voc_conv_transpose1d(oracle.ref_snake_beta(x[0], blk["ea"], blk["ieb"]),
                                        blk["w"], blk["b"], rate)
    for u in blk["units"]:
        h = oracle.ref_voc_resunit(h, {k: v for k, v in u.items() if k != "dilation"},
                                   u["dilation"])
    drift = max_rel_err(h[None], ora)
    assert max_rel_err(run_device(x, blk, c_out), ora) <= max(TOL_F32, 2 * drift)


def test_block_argument_checks():
    L = lai.load()
    import ctypes
    rng = np.random.default_rng(0)
    blk = make_block(64, 32, 4, 0, rng)
    dev = {k: (torch.from_numpy(v).to(DEV) if isinstance(v, np.ndarray) else v)
           for k, v in blk.items()}
    params = lai.voc_block_params(dev)
    x = torch.zeros(1, 10, 64, device=DEV)
    out = torch.zeros(1, 36, 32, device=DEV)
    s = torch.zeros(2 * 10 * 64 + 4 * 36 * 32, device=DEV)
    f = L.lai_voc_bigvgan_block_f32
    ref = ctypes.byref(params[0])
    assert f(lai._p(out), lai._p(x), lai._p(s), ref, 1, 64, 32, 1, 3, None, None) == lai.LAI_ERR_INVALID
    assert f(lai._p(out), lai._p(x), lai._p(s), ref, 1, 60, 32, 10, 3, None, None) == lai.LAI_ERR_INVALID
    assert f(lai._p(out), lai._p(out), lai._p(s), ref, 1, 64, 32, 10, 3, None, None) == lai.LAI_ERR_ALIAS
    assert f(lai._p(out), lai._p(x), lai._p(s), ref, 0, 64, 32, 10, 3, None, None) == lai.LAI_OK

"""Vocoder BigVGAN ResUnits on tensor cores against the oracle's run_resunit.

run_resunit (src/tts_vocoder.c:540-583), three per block with dilations 1, 3, 9
(src/tts_vocoder.c:269, 725-728). The device path runs channels-last [B, T, C]; the
oracle runs the reference's channels-first [C, T] per batch item.
Tolerance, max |d| / max(1, |ref|), per unit on identical inputs: 1e-5 with passes = 3
(the F32 bar), 1e-2 with passes = 1 (TF32 inputs carry 10 mantissa bits; the BF16 bar).
A whole block is held to twice the reference F32 code's own drift from the oracle.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_BF16, TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"


def make_unit(C, dilation, rng):
    f = lambda a: np.asarray(a, np.float32)
    return {
        "ea1": f(np.exp(rng.normal(0, 0.1, C))), "ieb1": f(1 / np.exp(rng.normal(0, 0.1, C))),
        "w1": f(rng.standard_normal((C, C, 7)) / np.sqrt(7 * C)), "b1": f(rng.normal(0, 0.1, C)),
        "ea2": f(np.exp(rng.normal(0, 0.1, C))), "ieb2": f(1 / np.exp(rng.normal(0, 0.1, C))),
        "w2": f(rng.standard_normal((C, C, 1)) / np.sqrt(C)), "b2": f(rng.normal(0, 0.1, C)),
        "dilation": dilation,
    }


def to_dev(p):
    return {k: (torch.from_numpy(v).to(DEV) if isinstance(v, np.ndarray) else v)
            for k, v in p.items()}


def run_device(x_ct, units_np, passes):
    """x_ct [B, C, T] numpy -> device channels-last ResUnits -> [B, C, T] numpy."""
    units = [to_dev(p) for p in units_np]
    x = torch.from_numpy(x_ct).to(DEV).transpose(1, 2).contiguous()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    lai.voc_resunits(x, lai.voc_units(units), passes=passes, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return x.transpose(1, 2).contiguous().cpu().numpy()


def run_oracle(x_ct, units_np):
    y = x_ct
    for p in units_np:
        y = oracle.voc_resunit(y, {k: v for k, v in p.items() if k != "dilation"},
                               p["dilation"])
    return y


# (batch, C, T, dilations): vocoder widths 768/384/192/96 and small ones; T below one
# 128-row tile, ragged last tiles, dilation 9 reaching wholly into the causal padding,
# batch > 1 (no tap may read the previous item's rows)
CASES = [(1, 32, 300, [1]), (2, 96, 1000, [1, 3, 9]), (1, 192, 517, [3]), (3, 64, 50, [9]),
         (1, 256, 130, [9]), (1, 384, 257, [1, 3]), (1, 768, 200, [1, 3, 9]), (2, 160, 129, [3])]


@pytest.mark.parametrize("B,C,T,dils", CASES)
def test_resunits_f32(B, C, T, dils):
    # every fused unit on identical inputs: unit k applied by the oracle to the device's
    # own output after k - 1 units (the chain call with k units also exercises conv2's
    # epilogue writing the next unit's snake1 input)
    rng = np.random.default_rng(C * 7 + T)
    units = [make_unit(C, d, rng) for d in dils]
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    prev = x
    for k in range(1, len(units) + 1):
        got = run_device(x, units[:k], 3)
        assert max_rel_err(got, run_oracle(prev, [units[k - 1]])) <= TOL_F32
        prev = got


@pytest.mark.parametrize("B,C,T,dils", [(2, 96, 1000, [1, 3, 9]), (1, 768, 200, [1])])
def test_resunits_tf32(B, C, T, dils):
    rng = np.random.default_rng(5)
    units = [make_unit(C, d, rng) for d in dils]
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    prev = x
    for k in range(1, len(units) + 1):
        got = run_device(x, units[:k], 1)
        assert max_rel_err(got, run_oracle(prev, [units[k - 1]])) <= TOL_BF16
        prev = got


@pytest.mark.skipif(not oracle.have_ref(), reason="reference vocoder ops not built")
@pytest.mark.parametrize("C", [96, 768])
def test_block_chain_as_accurate_as_reference_f32(C):
    # a whole block (dilations 1, 3, 9) end to end: each unit feeds perturbations of its
    # input forward with gain > 1, so the reference's own F32 code drifts from the
    # double-precision oracle too; the device stays within twice that drift
    rng = np.random.default_rng(C)
    units = [make_unit(C, d, rng) for d in (1, 3, 9)]
    x = rng.standard_normal((1, C, 300)).astype(np.float32)
    ora = run_oracle(x, units)
    ref = x
    for u in units:
        ref = oracle.ref_voc_resunit(ref, {k: v for k, v in u.items() if k != "dilation"},
                                     u["dilation"])
    assert max_rel_err(run_device(x, units, 3), ora) <= max(TOL_F32, 2 * max_rel_err(ref, ora))


@pytest.mark.skipif(not oracle.have_ref(), reason="reference vocoder ops not built")
def test_resunit_matches_reference_functions():
    # the unit composed from the reference's own compiled voc_snake_beta and
    # voc_conv1d_causal (scalar build), not only the restatement
    rng = np.random.default_rng(11)
    p = make_unit(96, 3, rng)
    x = rng.standard_normal((1, 96, 700)).astype(np.float32)
    ref = oracle.ref_voc_resunit(x, {k: v for k, v in p.items() if k != "dilation"}, 3)
    assert max_rel_err(run_device(x, [p], 3), ref) <= TOL_F32


def test_pack_conv_bit_exact():
    rng = np.random.default_rng(2)
    w = rng.standard_normal((64, 32, 7)).astype(np.float32)
    got = lai.voc_pack_conv(torch.from_numpy(w).to(DEV)).cpu().numpy()
    bits = w.view(np.uint32)
    hi = ((bits + np.uint32(0x1000)) & np.uint32(0xFFFFE000)).view(np.float32)  # TF32, ties away
    lo = w - hi
    want = np.stack([hi.transpose(2, 0, 1), lo.transpose(2, 0, 1)])  # [2, k, c_out, c_in]
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.array_equal((got[0] + got[1]), w.transpose(2, 0, 1))
    # specials: NaN with a full mantissa (CUDA's canonical 0x7fffffff) stays NaN, inf stays
    # inf, a tie rounds away from zero
    sp = np.array([0x7FFFFFFF, 0xFFFFFFFF, 0x7F800000, 0xFF800000, 0x3F801000, 0xBF801000,
                   0x3F800FFF, 0x00000000], np.uint32).view(np.float32)
    w2 = np.zeros((32, 32, 1), np.float32)
    w2[0, :8, 0] = sp
    hi2 = lai.voc_pack_conv(torch.from_numpy(w2).to(DEV)).cpu().numpy()[0, 0, 0, :8]
    assert np.isnan(hi2[:2]).all()
    assert hi2[2] == np.inf and hi2[3] == -np.inf
    assert hi2[4:].view(np.uint32).tolist() == [0x3F802000, 0xBF802000, 0x3F800000, 0]


def test_transpose_round_trip():
    x = torch.randn(3, 77, 45, device=DEV)
    y = lai.voc_transpose(x)
    assert torch.equal(y, x.transpose(1, 2))
    assert torch.equal(lai.voc_transpose(y), x)


def test_resunits_argument_checks():
    L = lai.load()
    import ctypes
    x = torch.zeros(1, 128, 96, device=DEV)
    s = torch.zeros(4 * 128 * 96, device=DEV)
    units = lai.voc_units([to_dev(make_unit(96, 1, np.random.default_rng(0)))])
    arr = ctypes.cast(units[0], ctypes.c_void_p)
    f = L.lai_voc_resunits_f32
    assert f(lai._p(x), lai._p(s), arr, 1, 1, 96, 128, 2, None, None) == lai.LAI_ERR_INVALID
    assert f(lai._p(x), lai._p(s), arr, 1, 1, 80, 128, 3, None, None) == lai.LAI_ERR_INVALID
    assert f(lai._p(x), lai._p(x), arr, 1, 1, 96, 128, 3, None, None) == lai.LAI_ERR_ALIAS
    assert f(lai._p(x), lai._p(s), arr, 0, 1, 96, 128, 3, None, None) == lai.LAI_OK

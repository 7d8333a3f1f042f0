"""The oracle's weight-format restatements, pinned on the CPU against independent numpy.

The reference stores decode weights as FP16 or as INT8 with per-row scales in its GPU
modes (src/tts_pipeline.h:37-40, src/tts_native.c:1185-1240; INT8 recipe
tools/asr_benchmarks.md:342-352). Its conversion code is not vendored, so the oracle's C
restatement is checked here against numpy's own IEEE binary16 rounding and a numpy
restatement of the INT8 recipe (roundf: halves away from zero), bit for bit.
"""
import numpy as np
import pytest

import oracle


def bf16_bits(x):
    """F32 -> BF16 bit patterns, round to nearest even (exact inputs stay exact)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def bf16_vals(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def test_f16_encode_matches_numpy():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e6, -1e6, 2.0 ** -24, 2.0 ** -25,
                  3 * 2.0 ** -26, 2.0 ** -14, 2.0 ** -14 - 2.0 ** -25, np.inf, -np.inf],
                 np.float32)]).astype(np.float32)  # both sides round the same F32 values
    got = oracle.f32_to_f16_bits(x)
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    nan = oracle.f32_to_f16_bits(np.array([np.nan], np.float32))
    assert np.isnan(nan.view(np.float16)).all()


def test_linear_f16_decodes_exactly():
    # every finite binary16 value against numpy's decode
    bits = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    vals = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(vals)
    W = bits[finite][:, None]  # one weight per row, K = 1
    x = np.ones((1, 1), np.float32)
    got = oracle.linear_f16(x, W)[0]
    assert np.array_equal(got, vals[finite])


def quantize_numpy(w_bits):
    w = bf16_vals(w_bits)
    amax = np.abs(w).max(axis=1)
    scale = (amax / np.float32(127)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        qf = (w / scale[:, None]).astype(np.float32)
    r = np.sign(qf) * np.floor(np.abs(qf).astype(np.float64) + 0.5)
    r = np.where(scale[:, None] > 0, np.clip(r, -127, 127), 0)
    return r.astype(np.int8), scale


@pytest.mark.parametrize("N,K", [(64, 1024), (7, 33), (3, 1)])
def test_quantize_rows_matches_recipe(N, K):
    rng = np.random.default_rng(N + K)
    w = bf16_bits(rng.standard_normal((N, K)).astype(np.float32) * 0.05)
    w[0] = 0  # an all-zero row: scale 0, q 0
    if K > 4:  # exact halves after division: 0.5 and -2.5 steps of the scale
        w[1, :4] = bf16_bits(np.array([127.0, 0.5, -2.5, 1.5], np.float32))
    q, s = oracle.quantize_rows_i8_bf16(w)
    qn, sn = quantize_numpy(w)
    assert np.array_equal(s.view(np.uint32), sn.view(np.uint32))
    assert np.array_equal(q, qn)
    assert s[0] == 0 and not q[0].any()
    if K > 4:
        assert q[1, :4].tolist() == [127, 1, -3, 2]  # halves away from zero
    assert np.abs(q).max() <= 127


def test_linear_i8_applies_scale_after_the_sum():
    rng = np.random.default_rng(5)
    q = rng.integers(-127, 128, (16, 96)).astype(np.int8)
    s = rng.uniform(0.001, 0.01, 16).astype(np.float32)
    x = rng.standard_normal((3, 96)).astype(np.float32)
    want = (x.astype(np.float64) @ q.T.astype(np.float64)) * s.astype(np.float64)
    got = oracle.linear_i8(x, q, s)
    assert np.abs(got - want).max() <= 1e-6 * max(1.0, np.abs(want).max())
    Wf = rng.standard_normal((16, 96)).astype(np.float32)
    assert np.allclose(oracle.linear_f32(x, Wf), x.astype(np.float64) @ Wf.T.astype(np.float64),
                       rtol=1e-6, atol=1e-6)

"""The CPU oracle against the reference's own golden vectors (CPU only).

Fixtures in tests/golden/ were produced by tests/golden/make_golden.py from the
reference: its numpy specification functions (tools/verify_xfmr.py,
tools/verify_vocoder.py) and its compiled voc_snake_beta (src/tts_vocoder_ops.c).
"""
import os

import numpy as np
import pytest

import oracle
from conftest import TOL_F32, max_rel_err

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def g(name):
    return np.load(os.path.join(GOLD, f"{name}.npz"))


@pytest.mark.parametrize("tag", ["d1024", "d2048", "d512", "d200"])
def test_rmsnorm_matches_reference_numpy(tag):
    d = g(f"rmsnorm_{tag}")
    y = oracle.rms_norm(d["x"], d["w"], float(d["eps"]))
    assert max_rel_err(y, d["y"]) <= TOL_F32


@pytest.mark.parametrize("tag", ["hd128", "hd64"])
def test_rope_matches_reference_numpy(tag):
    d = g(f"rope_{tag}")
    T, hd, heads = d["x"].shape[0], int(d["hd"]), int(d["heads"])
    c, s = oracle.compute_rope_neox(np.arange(T), hd, float(d["theta"]))
    y = oracle.apply_rope_neox(d["x"], c, s, heads, hd)
    assert max_rel_err(y, d["y"]) <= TOL_F32


def test_rope_position_zero_is_identity():
    x = np.random.default_rng(1).standard_normal((1, 4 * 128), dtype=np.float32)
    c, s = oracle.compute_rope_neox(np.array([0]), 128, 1e6)
    assert np.array_equal(oracle.apply_rope_neox(x, c, s, 4, 128), x)


def test_swiglu_matches_reference_numpy():
    d = g("swiglu")
    y = oracle.swiglu_multiply(d["gate_up"], int(d["inter"]))
    assert max_rel_err(y, d["y"]) <= TOL_F32


def test_swiglu_in_place_matches_out_of_place():
    rng = np.random.default_rng(2)
    gu = rng.standard_normal((7, 2 * 96), dtype=np.float32)
    ref = oracle.swiglu_multiply(gu, 96)
    buf = gu.copy()
    lib = oracle.load()
    lib.oracle_swiglu_multiply(oracle.ptr(buf), oracle.ptr(buf), 7, 96)
    assert np.array_equal(buf.reshape(-1)[: 7 * 96].reshape(7, 96), ref)


def test_silu_matches_reference_numpy():
    d = g("silu")
    assert max_rel_err(oracle.silu(d["x"]), d["y"]) <= TOL_F32


def test_snake_restatement_is_bit_exact_with_reference_build():
    d = g("snake")
    y = oracle.snake_beta(d["x"], d["ea"], d["ieb"])
    assert np.array_equal(y, d["y_ref_scalar"])
    assert max_rel_err(y, d["y_numpy"]) <= TOL_F32


def test_reference_avx2_snake_error_is_the_known_approximation():
    # The shipped AVX2 fast sin is the reference's approximation, ~2e-4 * ieb at most.
    d = g("snake")
    err = np.max(np.abs(d["y_ref_avx2"] - d["y_ref_scalar"]))
    assert 1e-6 < err < 1e-3


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (reference absent)")
def test_snake_against_live_reference_build_ragged():
    rng = np.random.default_rng(3)
    for C, T in [(3, 1), (5, 7), (2, 1001)]:
        x = (3 * rng.standard_normal((C, T))).astype(np.float32)
        ea = np.exp(0.1 * rng.standard_normal(C)).astype(np.float32)
        ieb = (1 / np.exp(0.1 * rng.standard_normal(C))).astype(np.float32)
        assert np.array_equal(oracle.snake_beta(x, ea, ieb), oracle.ref_snake_beta(x, ea, ieb))


def test_bf16_widening_known_answers():
    d = g("bf16_widen")
    table = d["bf16"].reshape(1, -1)
    out = oracle.gather_bf16_to_f32(table, np.array([0], np.int32))
    assert np.array_equal(out.view(np.uint32).reshape(-1), d["f32_bits"])


def test_bf16_rounding_is_rne():
    f = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e38, np.inf, -0.0], np.float32)
    # 1+2^-8 is a tie -> even (1.0); 1+3*2^-8 is a tie -> even (1+2^-6)
    want = np.array([0x3F80, 0x3F80, 0x3F82, 0xC020, 0x7F62, 0x7F80, 0x8000], np.uint16)
    assert np.array_equal(oracle.f32_to_bf16_bits(f), want)
    lib = oracle.load()
    assert [lib.oracle_f32_to_bf16(float(v)) for v in f] == want.tolist()
    assert lib.oracle_f32_to_bf16(float("nan")) == 0x7FFF


def test_fused_oracles_equal_reference_call_sequences():
    rng = np.random.default_rng(4)
    x = rng.standard_normal((4, 256), dtype=np.float32)
    dl = rng.standard_normal((4, 256), dtype=np.float32)
    w = (1 + 0.02 * rng.standard_normal(256)).astype(np.float32)
    xo, y = oracle.add_rms_norm_f32(x, dl, w, 1e-6)
    assert np.array_equal(xo, oracle.add_inplace(x, dl))
    assert np.array_equal(y, oracle.rms_norm(xo, w, 1e-6))
    q = rng.standard_normal((3, 4 * 128), dtype=np.float32)
    wq = (1 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    c, s = oracle.compute_rope_neox(np.arange(3), 128, 1e6)
    qo, _ = oracle.qk_norm_rope(q, None, wq, None, c, s, None, 4, 0, 128, 1e-6, bf16=False)
    ref = oracle.apply_rope_neox(oracle.rms_norm_per_head(q, wq, 4, 128, 1e-6), c, s, 4, 128)
    assert np.array_equal(qo, ref)


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (reference absent)")
@pytest.mark.parametrize("c_in,c_out,T,k,d", [(24, 16, 50, 7, 1), (16, 32, 40, 7, 3),
                                               (8, 8, 30, 7, 9), (32, 24, 17, 1, 1)])
def test_conv1d_restatement_against_reference_build(c_in, c_out, T, k, d):
    # voc_conv1d_causal compiled from the reference source (no BLAS: pad, im2col, float
    # dot products) against the restatement's double sums: F32 round-off only
    rng = np.random.default_rng(c_in + T)
    x = rng.standard_normal((c_in, T)).astype(np.float32)
    w = (rng.standard_normal((c_out, c_in, k)) / np.sqrt(c_in * k)).astype(np.float32)
    b = rng.normal(0, 0.1, c_out).astype(np.float32)
    got = oracle.voc_conv1d_causal(x, w, b, d)
    ref = oracle.ref_voc_conv1d_causal(x, w, b, d)
    assert np.max(np.abs(got - ref)) / max(1.0, np.max(np.abs(ref))) <= 1e-5
    # causality: output t never sees inputs after t
    x2 = x.copy()
    x2[:, T // 2:] += 1.0
    got2 = oracle.voc_conv1d_causal(x2, w, b, d)
    assert np.array_equal(got[:, : T // 2], got2[:, : T // 2])


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (reference absent)")
def test_resunit_restatement_against_reference_functions():
    rng = np.random.default_rng(9)
    C, T = 32, 90
    p = {"ea1": np.exp(rng.normal(0, 0.1, C)), "ieb1": 1 / np.exp(rng.normal(0, 0.1, C)),
         "w1": rng.standard_normal((C, C, 7)) / np.sqrt(7 * C), "b1": rng.normal(0, 0.1, C),
         "ea2": np.exp(rng.normal(0, 0.1, C)), "ieb2": 1 / np.exp(rng.normal(0, 0.1, C)),
         "w2": rng.standard_normal((C, C, 1)) / np.sqrt(C), "b2": rng.normal(0, 0.1, C)}
    p = {k: v.astype(np.float32) for k, v in p.items()}
    x = rng.standard_normal((2, C, T)).astype(np.float32)
    for d in (1, 3, 9):
        got, ref = oracle.voc_resunit(x, p, d), oracle.ref_voc_resunit(x, p, d)
        assert np.max(np.abs(got - ref)) / max(1.0, np.max(np.abs(ref))) <= 1e-5


@pytest.mark.skipif(not oracle.have_ref_sampling(), reason="oracle/_ref not built (reference absent)")
@pytest.mark.parametrize("vocab,top_k,temp", [(3072, 50, 0.9), (2048, 50, 0.7), (3072, 1, 1.0),
                                              (300, 0, 1.3), (3072, 3072, 0.8), (100, 7, 0.5)])
def test_sampling_restatement_matches_reference_build(vocab, top_k, temp):
    # the reference's own tts_sample_topk, its rand() driven by srand(seed), against the
    # restatement given the same draw: identical tokens
    rng = np.random.default_rng(vocab + top_k)
    for trial in range(200):
        logits = (rng.standard_normal(vocab) * (1 + trial % 5)).astype(np.float32)
        if trial % 7 == 0:
            logits[rng.integers(0, vocab, 20)] = logits.max()  # ties at the top
        seed = 1000 + trial
        want = oracle.ref_sample_topk(logits, temp, top_k, seed)
        got, _, _ = oracle.sample_topk(logits, temp, top_k, oracle.ref_rand_draw(seed))
        assert got == want, (trial, got, want)


@pytest.mark.skipif(not oracle.have_ref_sampling(), reason="oracle/_ref not built (reference absent)")
def test_repetition_penalty_matches_reference_build():
    rng = np.random.default_rng(1)
    logits = rng.standard_normal(3072).astype(np.float32)
    hist = rng.integers(-5, 3100, 200).astype(np.int32)  # repeats and out-of-range ids
    for pen in (1.0, 1.05, 1.3):
        assert np.array_equal(oracle.repetition_penalty(logits, hist, pen),
                              oracle.ref_repetition_penalty(logits, hist, pen))


@pytest.mark.skipif(not oracle.have_ref(), reason="oracle/_ref not built (reference absent)")
def test_convnext_restatement_against_reference_functions():
    # run_convnext's sequence composed from the reference's compiled voc_conv1d_causal
    # (depthwise branch and k = 1), voc_layer_norm_channels and voc_gelu
    rng = np.random.default_rng(5)
    C, T = 32, 30
    f = lambda a: np.asarray(a, np.float32)  # noqa: E731
    p = {"dw_w": f(rng.standard_normal((C, 1, 7)) / np.sqrt(7)), "dw_b": f(rng.normal(0, .1, C)),
         "norm_w": f(1 + rng.normal(0, .1, C)), "norm_b": f(rng.normal(0, .1, C)),
         "pw1_w": f(rng.standard_normal((4 * C, C, 1)) / np.sqrt(C)), "pw1_b": f(rng.normal(0, .1, 4 * C)),
         "pw2_w": f(rng.standard_normal((C, 4 * C, 1)) / np.sqrt(4 * C)), "pw2_b": f(rng.normal(0, .1, C)),
         "gamma": f(rng.normal(0, .3, C))}
    x = rng.standard_normal((2, C, T)).astype(np.float32)
    got, ref = oracle.voc_convnext(x, p), oracle.ref_voc_convnext(x, p)
    assert np.max(np.abs(got - ref)) / max(1.0, np.max(np.abs(ref))) <= 1e-5

"""The vocoder front on the device against the oracle: causal prefill attention (plain and
with RoPE folded in over a fused q|k|v output), the RVQ gather, the LayerScale + residual
linear, and the whole front (RVQ decode -> pre_conv -> 8-layer pre-transformer) of
tts_vocoder_run (src/tts_vocoder.c:589-640, src/tts_vocoder_xfmr.c:126-225).

Tolerances: single ops max |d| / max(1, |ref|) <= 1e-5 (F32 paths; the linears are 3xTF32);
the whole front within max(1e-5, 2x the error of the same composition in float arithmetic,
the oracle's timed build) of the double-accumulating checker, as for the decoder.
"""
import numpy as np
import pytest

import lai
import oracle
import runner
from conftest import TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def td(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("T,heads,kv,hd", [(1, 16, 16, 64), (31, 16, 16, 64), (100, 4, 2, 64),
                                           (500, 16, 16, 64), (257, 2, 2, 128), (33, 8, 1, 128)])
def test_prefill_attention(T, heads, kv, hd):
    rng = np.random.default_rng(T + 13 * heads + hd)
    q = rng.standard_normal((T, heads * hd)).astype(np.float32)
    k = rng.standard_normal((T, kv * hd)).astype(np.float32)
    v = rng.standard_normal((T, kv * hd)).astype(np.float32)
    got = lai.prefill_attention(td(q), td(k), td(v), heads, kv, hd).cpu().numpy()
    assert max_rel_err(got, oracle.causal_attention(q, k, v, heads, kv, hd)) <= TOL_F32


@pytest.mark.parametrize("T,heads,hd", [(7, 16, 64), (129, 16, 64), (64, 4, 128)])
def test_prefill_attention_rope_fused_qkv(T, heads, hd):
    rng = np.random.default_rng(T + hd)
    D = heads * hd
    qkv = rng.standard_normal((T, 3 * D)).astype(np.float32)
    cos_t, sin_t = oracle.compute_rope_neox(np.arange(T, dtype=np.int32), hd, 10000.0)
    q = oracle.apply_rope_neox(qkv[:, :D], cos_t, sin_t, heads, hd)
    k = oracle.apply_rope_neox(qkv[:, D:2 * D], cos_t, sin_t, heads, hd)
    want = oracle.causal_attention(q, k, qkv[:, 2 * D:], heads, heads, hd)
    got = lai.prefill_attention_rope(td(qkv), heads, heads, hd, td(cos_t), td(sin_t))
    assert max_rel_err(got.cpu().numpy(), want) <= TOL_F32


def test_prefill_attention_rope_table_too_short():
    qkv = torch.zeros((8, 3 * 64), device="cuda")
    c = torch.zeros((4, 64), device="cuda")
    with pytest.raises(lai.LaiError):
        lai.prefill_attention_rope(qkv, 1, 1, 64, c, c)


def test_rvq_gather_exact_and_out_of_range():
    rng = np.random.default_rng(3)
    books = rng.standard_normal((4, 50, 256)).astype(np.float32)
    codes = rng.integers(0, 50, (9, 4)).astype(np.int64)
    codes[4, 2] = 50  # out of range
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    got = lai.voc_rvq_gather(td(books), td(codes), err=err).cpu().numpy()
    want = np.concatenate([books[cb][np.clip(codes[:, cb], 0, 49)] for cb in range(4)], axis=1)
    want[4, 2 * 256:3 * 256] = 0.0
    assert np.array_equal(got, want)
    assert int(err.item()) == lai.LAI_DEVERR_TOKEN_ID


@pytest.mark.parametrize("rows,c_in,c_out,passes", [(1, 1024, 512, 3), (300, 1024, 512, 3),
                                                     (77, 96, 64, 3), (128, 512, 512, 1)])
def test_linear_scale_residual(rows, c_in, c_out, passes):
    rng = np.random.default_rng(rows + c_in)
    x = rng.standard_normal((rows, c_out)).astype(np.float32)
    inp = rng.standard_normal((rows, c_in)).astype(np.float32)
    W = (rng.standard_normal((c_out, c_in)) / np.sqrt(c_in)).astype(np.float32)
    b = rng.normal(0, .1, c_out).astype(np.float32)
    g = rng.normal(0, .1, c_out).astype(np.float32)
    xd = td(x)
    lai.voc_linear_scale_residual(xd, td(inp), lai.voc_pack_conv(td(W[:, :, None])), td(b), td(g),
                                  passes=passes)
    lin = oracle.linear_f32(inp, W).astype(np.float64) + b
    want = x.astype(np.float64) + g * lin
    tol = TOL_F32 if passes == 3 else 2e-3  # 1 pass is plain TF32 (10-bit mantissa operands)
    assert max_rel_err(xd.cpu().numpy(), want) <= tol


def _front_numpy(front):
    n = lambda t: t.detach().cpu().numpy()  # noqa: E731
    r = front.ref
    p = {k: n(v) for k, v in r.items() if k != "layers"}
    p["layers"] = [{k: n(v) for k, v in L.items()} for L in r["layers"]]
    return p


@pytest.mark.parametrize("T", [40, 129])
def test_front_matches_oracle(T):
    front = runner.VocFront(t_frames=T, seed=31 + T)
    for f in front.launches():
        f()
    torch.cuda.synchronize()
    assert int(front.err.item()) == 0
    got = front.y[0].cpu().numpy()
    p = _front_numpy(front)
    codes = front.codes.cpu().numpy()
    ora = oracle.voc_front(p, codes)
    flt = oracle.voc_front(p, codes, lib=oracle.load("liblai_cpuref.so"))
    e_gpu, e_flt = max_rel_err(got, ora), max_rel_err(flt, ora)
    assert np.isfinite(got).all()
    assert e_gpu <= max(TOL_F32, 2 * e_flt), (e_gpu, e_flt)


def test_codes_to_audio_end_to_end():
    # the whole tts_vocoder_run: the front writes the decoder's input buffer in place
    w = runner.VocCodesToAudio(t_frames=6, seed=3)
    assert w.dec.x_in.data_ptr() == w.front.y.data_ptr()
    for f in w.launches():
        f()
    torch.cuda.synchronize()
    assert int(w.err.item()) == 0 and int(w.dec.err.item()) == 0
    audio = w.audio.cpu().numpy()
    assert audio.shape == (1, w.rows_step)
    assert np.isfinite(audio).all() and np.abs(audio).max() <= 1.0
    # deterministic: a second run from the same codes gives the same samples, and so does
    # the step replayed as one CUDA graph
    w.run()
    assert np.array_equal(w.audio.cpu().numpy(), audio)
    w.run(graph=True)
    torch.cuda.synchronize()
    assert np.array_equal(w.audio.cpu().numpy(), audio)
    # new codes copied into the captured buffer change the replayed output
    w.codes.copy_(torch.flip(w.codes, [0]))
    w.run(graph=True)
    assert not np.array_equal(w.audio.cpu().numpy(), audio)


@pytest.mark.parametrize("T,c_in,c_out,k", [(500, 1024, 512, 1), (200, 512, 1024, 3),
                                            (40, 4096, 512, 1), (130, 512, 3072, 1)])
def test_split_k_conv_deterministic_and_exact(T, c_in, c_out, k):
    # short sequences have few 128-row tiles, so the GEMM runs split-K across a cluster;
    # the partial sums are combined in a fixed order: repeated runs are bit-identical
    rng = np.random.default_rng(T + c_out)
    x = rng.standard_normal((1, T, c_in)).astype(np.float32)
    w = (rng.standard_normal((c_out, c_in, k)) / np.sqrt(c_in * k)).astype(np.float32)
    b = rng.normal(0, .1, c_out).astype(np.float32)
    wp = lai.voc_pack_conv(td(w))
    a = lai.voc_conv1d(td(x), wp, td(b), c_out, k).cpu().numpy()
    for _ in range(3):
        assert np.array_equal(lai.voc_conv1d(td(x), wp, td(b), c_out, k).cpu().numpy(), a)
    want = oracle.voc_conv1d_causal(np.ascontiguousarray(x[0].T), w, b).T
    assert max_rel_err(a[0], want) <= TOL_F32

"""The vocoder decoder's remaining convolutions and the whole decoder against the oracle.

Causal conv1d (voc_conv1d_causal, src/tts_vocoder_ops.c:44-147), transposed conv with
kernel = stride (the ConvNeXt upsample stages, src/tts_vocoder.c:658-667) and 2 stride, the
final SnakeBeta -> conv 96 -> 1 -> clamp (src/tts_vocoder.c:748-758), and tts_vocoder_run
from the pre-transformer's output to audio. Single ops: max |d| / max(1, |ref|) <= 1e-5. The
whole decoder (14 chained convolution stages) is held to twice the drift of the reference's
own F32 functions from the double-precision oracle.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_F32, max_rel_err
from test_gpu_convnext import make_block as make_convnext
from test_gpu_resunit import make_unit

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"


def td(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(DEV)


def cl(x_ct):  # [B, C, T] numpy -> device [B, T, C]
    return td(x_ct).transpose(1, 2).contiguous()


def ct(x_cl):  # device [B, T, C] -> numpy [B, C, T]
    return x_cl.transpose(1, 2).contiguous().cpu().numpy()


@pytest.mark.parametrize("B,c_in,c_out,T,k,d", [(1, 1024, 1536, 60, 7, 1), (2, 64, 96, 200, 3, 2),
                                                (1, 32, 32, 5, 7, 1)])
def test_conv1d(B, c_in, c_out, T, k, d):
    rng = np.random.default_rng(c_in + T)
    w = (rng.standard_normal((c_out, c_in, k)) / np.sqrt(c_in * k)).astype(np.float32)
    b = rng.normal(0, 0.1, c_out).astype(np.float32)
    x = rng.standard_normal((B, c_in, T)).astype(np.float32)
    got = ct(lai.voc_conv1d(cl(x), lai.voc_pack_conv(td(w)), td(b), c_out, k, d))
    want = np.stack([oracle.voc_conv1d_causal(x[i], w, b, d) for i in range(B)])
    assert max_rel_err(got, want) <= TOL_F32


@pytest.mark.parametrize("B,c_in,c_out,T,kernel,stride", [(1, 1024, 1024, 50, 2, 2),
                                                          (2, 64, 32, 33, 3, 3),
                                                          (1, 96, 64, 40, 8, 4)])
def test_conv_transpose1d(B, c_in, c_out, T, kernel, stride):
    rng = np.random.default_rng(kernel + T)
    w = (rng.standard_normal((c_in, c_out, kernel)) / np.sqrt(c_in)).astype(np.float32)
    b = rng.normal(0, 0.1, c_out).astype(np.float32)
    x = rng.standard_normal((B, c_in, T)).astype(np.float32)
    got = ct(lai.voc_conv_transpose1d(cl(x), lai.voc_pack_tconv(td(w), stride), td(b), c_out,
                                      kernel, stride))
    want = np.stack([oracle.voc_conv_transpose1d(x[i], w, b, stride) for i in range(B)])
    assert got.shape == want.shape
    assert max_rel_err(got, want) <= TOL_F32


def final_ref(x, ea, ieb, w, b, ref=False):
    out = []
    for i in range(x.shape[0]):
        if ref:
            s = oracle.ref_snake_beta(x[i], ea, ieb)
            y = oracle.ref_voc_conv1d_causal(s, w, b, 1)
        else:
            s = oracle.snake_beta(x[i], ea, ieb)
            y = oracle.voc_conv1d_causal(s, w, b, 1)
        out.append(np.clip(y[0], -1.0, 1.0))
    return np.stack(out)


@pytest.mark.parametrize("B,T", [(1, 1000), (2, 300), (1, 5)])
def test_final_snake_conv_clamp(B, T):
    rng = np.random.default_rng(T)
    C = 96
    ea = np.exp(rng.normal(0, 0.1, C)).astype(np.float32)
    ieb = (1 / np.exp(rng.normal(0, 0.1, C))).astype(np.float32)
    w = (rng.standard_normal((1, C, 7)) / np.sqrt(C * 7) * 3).astype(np.float32)  # some clamping
    b = rng.normal(0, 0.1, 1).astype(np.float32)
    x = rng.standard_normal((B, C, T)).astype(np.float32)
    got = lai.voc_final(cl(x), td(ea), td(ieb), td(w), td(b)).cpu().numpy()
    assert max_rel_err(got, final_ref(x, ea, ieb, w, b)) <= TOL_F32
    if oracle.have_ref():
        assert max_rel_err(got, final_ref(x, ea, ieb, w, b, ref=True)) <= TOL_F32


@pytest.mark.skipif(not oracle.have_ref(), reason="reference vocoder ops not built")
def test_whole_decoder_as_accurate_as_reference_f32():
    # tts_vocoder_run from the pre-transformer output [1024, T0]: 2 x (transposed conv k=s=2 +
    # ConvNeXt), init conv 1024 -> 1536, 4 BigVGAN blocks (rates 8, 5, 4, 3), final step
    rng = np.random.default_rng(2024)
    T0 = 4
    f = lambda a: np.asarray(a, np.float32)  # noqa: E731
    ups = [{"w": f(rng.standard_normal((1024, 1024, 2)) / np.sqrt(1024)), "b": f(rng.normal(0, .05, 1024)),
            "cn": make_convnext(1024, rng)} for _ in range(2)]
    init_w = f(rng.standard_normal((1536, 1024, 7)) / np.sqrt(7 * 1024))
    init_b = f(rng.normal(0, .05, 1536))
    chans, rates = (1536, 768, 384, 192, 96), (8, 5, 4, 3)
    blocks = []
    for i, r in enumerate(rates):
        c_in, c_out = chans[i], chans[i + 1]
        blocks.append({"ea": f(np.exp(rng.normal(0, .1, c_in))), "ieb": f(1 / np.exp(rng.normal(0, .1, c_in))),
                       "w": f(rng.standard_normal((c_in, c_out, 2 * r)) / np.sqrt(2 * c_in)),
                       "b": f(rng.normal(0, .05, c_out)), "rate": r,
                       "units": [make_unit(c_out, d, rng) for d in (1, 3, 9)]})
    fin = {"ea": f(np.exp(rng.normal(0, .1, 96))), "ieb": f(1 / np.exp(rng.normal(0, .1, 96))),
           "w": f(rng.standard_normal((1, 96, 7)) / np.sqrt(96 * 7)), "b": f(rng.normal(0, .05, 1))}
    x = rng.standard_normal((1, 1024, T0)).astype(np.float32)

    def cpu(ref):
        h = x[0]
        for u in ups:
            h = (oracle.ref_voc_conv_transpose1d if ref else oracle.voc_conv_transpose1d)(h, u["w"], u["b"], 2)
            h = (oracle.ref_voc_convnext if ref else oracle.voc_convnext)(h[None], u["cn"])[0]
        h = (oracle.ref_voc_conv1d_causal if ref else oracle.voc_conv1d_causal)(h, init_w, init_b, 1)
        for blk in blocks:
            if ref:
                h = oracle.ref_voc_conv_transpose1d(oracle.ref_snake_beta(h, blk["ea"], blk["ieb"]),
                                                    blk["w"], blk["b"], blk["rate"])
                for u in blk["units"]:
                    h = oracle.ref_voc_resunit(h, {k: v for k, v in u.items() if k != "dilation"},
                                               u["dilation"])
            else:
                h = oracle.voc_bigvgan_block(h, blk)[0]
        return final_ref(h[None], fin["ea"], fin["ieb"], fin["w"], fin["b"], ref=ref)

    ora, ref = cpu(False), cpu(True)
    # device
    hd = cl(x)
    for u in ups:
        hd = lai.voc_conv_transpose1d(hd, lai.voc_pack_tconv(td(u["w"]), 2), td(u["b"]), 1024, 2, 2)
        lai.voc_convnext(hd, lai.voc_convnext_params({k: td(v) for k, v in u["cn"].items()}))
    hd = lai.voc_conv1d(hd, lai.voc_pack_conv(td(init_w)), td(init_b), 1536, 7)
    for i, blk in enumerate(blocks):
        dev = {k: (td(v) if isinstance(v, np.ndarray) else v) for k, v in blk.items() if k != "units"}
        dev["units"] = [{k: (td(v) if isinstance(v, np.ndarray) else v) for k, v in u.items()}
                        for u in blk["units"]]
        hd = lai.voc_bigvgan_block(hd, lai.voc_block_params(dev), chans[i + 1])
    audio = lai.voc_final(hd, td(fin["ea"]), td(fin["ieb"]), td(fin["w"]), td(fin["b"]))
    got = audio.cpu().numpy()
    assert got.shape == ora.shape
    assert max_rel_err(got, ora) <= max(TOL_F32, 2 * max_rel_err(ref, ora))

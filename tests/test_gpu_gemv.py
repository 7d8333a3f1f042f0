"""Decode-time fused linear layers against the oracle and a plain PyTorch FP32 matmul.

linear_bf16 (src/tts_native.c:66-79) with the ops the decode step runs around it
(src/tts_native.c:637-668): RMSNorm prologue, residual-add epilogue, SwiGLU epilogue
over interleaved gate/up rows. FP32 tolerance: max |d| / max(1, |ref|) <= 1e-5.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"

# (M, K, N): talker-0.6B q / k,v / o / gate_up / down projections, 1.7B gate_up,
# small batches, multi-pass M, and shapes without a 16-byte weight path
SHAPES = [(1, 1024, 2048), (1, 1024, 1024), (1, 2048, 1024), (1, 1024, 6144), (1, 3072, 1024),
          (1, 2048, 12288), (3, 1024, 512), (8, 2048, 64), (13, 512, 96), (1, 100, 37),
          (2, 6144, 2048)]


def make(M, K, N, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    W = (torch.randn(N, K, generator=g) / np.sqrt(K)).to(torch.bfloat16)
    w = 1 + 0.02 * torch.randn(K, generator=g)
    return x, W, w


def wbits(W):
    return W.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("M,K,N", SHAPES)
@pytest.mark.parametrize("norm", [False, True])
def test_gemv(M, K, N, norm):
    x, W, w = make(M, K, N, 1)
    y = lai.gemv(x.to(DEV), W.to(DEV), w.to(DEV) if norm else None, 1e-6)
    torch.cuda.synchronize()
    xn = oracle.rms_norm(x.numpy(), w.numpy(), 1e-6) if norm else x.numpy()
    assert max_rel_err(y.cpu().numpy(), oracle.linear_bf16(xn, wbits(W))) <= TOL_F32
    ref = torch.from_numpy(xn).to(DEV) @ W.to(DEV).float().T  # plain FP32 matmul
    assert max_rel_err(y.cpu().numpy(), ref.cpu().numpy()) <= TOL_F32


@pytest.mark.parametrize("M,K,N", [(1, 2048, 1024), (1, 3072, 1024), (4, 1024, 512), (9, 100, 37)])
def test_gemv_residual(M, K, N):
    a, W, _ = make(M, K, N, 2)
    x = torch.randn(M, N)
    xd = x.to(DEV)
    lai.gemv_residual(xd, a.to(DEV), W.to(DEV))
    torch.cuda.synchronize()
    ref = oracle.add_inplace(x.numpy(), oracle.linear_bf16(a.numpy(), wbits(W)))
    assert max_rel_err(xd.cpu().numpy(), ref) <= TOL_F32


@pytest.mark.parametrize("M,K,inter", [(1, 1024, 3072), (1, 2048, 6144), (5, 512, 96), (1, 40, 7)])
@pytest.mark.parametrize("norm", [False, True])
def test_gemv_swiglu(M, K, inter, norm):
    x, W, w = make(M, K, 2 * inter, 3)
    out = lai.gemv_swiglu(x.to(DEV), W.to(DEV), w.to(DEV) if norm else None, 1e-6)
    torch.cuda.synchronize()
    xn = oracle.rms_norm(x.numpy(), w.numpy(), 1e-6) if norm else x.numpy()
    gate_up = oracle.linear_bf16(xn, wbits(W))  # [M, 2I], interleaved as the fused weight is
    assert max_rel_err(out.cpu().numpy(), oracle.swiglu_multiply(gate_up, inter)) <= TOL_F32


def test_gemv_decode_layer_equals_unfused_sequence():
    # one talker decode layer's linear + elementwise sequence (src/tts_native.c:637-668),
    # fused kernels vs the unfused device kernels (RMSNorm, GEMV, SwiGLU, add)
    D, I, QKV = 1024, 3072, 2048 + 2 * 1024
    g = torch.Generator(device="cpu").manual_seed(4)
    x = torch.randn(1, D, generator=g).to(DEV)
    w_in, w_post = (1 + 0.02 * torch.randn(D, generator=g)).to(DEV), (1 + 0.02 * torch.randn(D, generator=g)).to(DEV)
    Wqkv = (torch.randn(QKV, D, generator=g) / 32).to(torch.bfloat16).to(DEV)
    Wo = (torch.randn(D, 2048, generator=g) / 45).to(torch.bfloat16).to(DEV)
    Wgu = (torch.randn(2 * I, D, generator=g) / 32).to(torch.bfloat16).to(DEV)
    Wd = (torch.randn(D, I, generator=g) / 55).to(torch.bfloat16).to(DEV)
    attn = torch.randn(1, 2048, generator=g).to(DEV)  # stands in for attention's output
    # fused
    xf = x.clone()
    qkv_f = lai.gemv(xf, Wqkv, w_in, 1e-6)
    lai.gemv_residual(xf, attn, Wo)
    act_f = lai.gemv_swiglu(xf, Wgu, w_post, 1e-6)
    lai.gemv_residual(xf, act_f, Wd)
    # unfused: every intermediate through HBM
    xu = x.clone()
    qkv_u = lai.gemv(lai.rmsnorm(xu, w_in, 1e-6), Wqkv)
    lai.add(xu, lai.gemv(attn, Wo))
    act_u = lai.swiglu(lai.gemv(lai.rmsnorm(xu, w_post, 1e-6), Wgu), I)
    lai.add(xu, lai.gemv(act_u, Wd))
    torch.cuda.synchronize()
    for f, u in [(qkv_f, qkv_u), (act_f, act_u), (xf, xu)]:
        assert max_rel_err(f.cpu().numpy(), u.cpu().numpy()) <= TOL_F32


def test_gemv_argument_checks():
    L = lai.load()
    import ctypes
    from conftest import arena_ptr
    P = arena_ptr(256)  # real memory: a regressed check would still stay in bounds
    assert L.lai_gemv_bf16w_f32(P, P, None, 1e-6, P, 1, 64, 8, None) == lai.LAI_ERR_ALIAS
    assert L.lai_gemv_swiglu_bf16w_f32(P, arena_ptr(1 << 20), None, 1e-6, P, 1, 64, 0,
                                       None) == lai.LAI_ERR_INVALID
    assert L.lai_gemv_bf16w_f32(P, arena_ptr(1 << 24), None, 1e-6, P, 1, 60000, 8,
                                None) == lai.LAI_ERR_TOOBIG


# ---- the reference's other GPU weight formats: FP16, INT8 + per-row scale, F32 ----------
def make_fmt(fmt, N, K, seed):
    """Weights in format fmt on the device + their oracle product function."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    Wf = torch.randn(N, K, generator=g) / np.sqrt(K)
    if fmt == "f16":
        W = Wf.to(torch.float16)
        return W.to(DEV), None, lambda xn: oracle.linear_f16(xn, W.view(torch.int16).numpy().view(np.uint16))
    if fmt == "f32":
        return Wf.to(DEV), None, lambda xn: oracle.linear_f32(xn, Wf.numpy())
    Wb = Wf.to(torch.bfloat16)
    q, s = oracle.quantize_rows_i8_bf16(wbits(Wb))
    return (torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV),
            lambda xn: oracle.linear_i8(xn, q, s))


FMT_SHAPES = [(1, 1024, 2048), (1, 2048, 1024), (4, 1024, 512), (8, 2048, 64), (3, 100, 37),
              (1, 40, 24)]


@pytest.mark.parametrize("fmt", ["f16", "i8", "f32"])
@pytest.mark.parametrize("M,K,N", FMT_SHAPES)
@pytest.mark.parametrize("norm", [False, True])
def test_gemv_formats(fmt, M, K, N, norm):
    W, sc, ref = make_fmt(fmt, N, K, M + K)
    x, _, w = make(M, K, N, 7)
    y = lai.gemv(x.to(DEV), W, w.to(DEV) if norm else None, 1e-6, scales=sc)
    torch.cuda.synchronize()
    xn = oracle.rms_norm(x.numpy(), w.numpy(), 1e-6) if norm else x.numpy()
    assert max_rel_err(y.cpu().numpy(), ref(xn)) <= TOL_F32


@pytest.mark.parametrize("fmt", ["f16", "i8", "f32"])
@pytest.mark.parametrize("M,K,N", [(1, 3072, 1024), (5, 512, 96), (2, 48, 17)])
def test_gemv_residual_formats(fmt, M, K, N):
    W, sc, ref = make_fmt(fmt, N, K, 11)
    a, _, _ = make(M, K, N, 12)
    x = torch.randn(M, N)
    xd = x.to(DEV)
    lai.gemv_residual(xd, a.to(DEV), W, scales=sc)
    torch.cuda.synchronize()
    assert max_rel_err(xd.cpu().numpy(), oracle.add_inplace(x.numpy(), ref(a.numpy()))) <= TOL_F32


@pytest.mark.parametrize("fmt", ["f16", "i8", "f32"])
@pytest.mark.parametrize("M,K,inter", [(1, 1024, 3072), (3, 512, 96), (1, 40, 7)])
def test_gemv_swiglu_formats(fmt, M, K, inter):
    W, sc, ref = make_fmt(fmt, 2 * inter, K, 13)
    x, _, w = make(M, K, 2 * inter, 14)
    out = lai.gemv_swiglu(x.to(DEV), W, w.to(DEV), 1e-6, scales=sc)
    torch.cuda.synchronize()
    gate_up = ref(oracle.rms_norm(x.numpy(), w.numpy(), 1e-6))
    assert max_rel_err(out.cpu().numpy(), oracle.swiglu_multiply(gate_up, inter)) <= TOL_F32


@pytest.mark.parametrize("N,K", [(2048, 1024), (37, 100), (5, 1)])
def test_quantize_rows_i8_bit_exact(N, K):
    g = torch.Generator(device="cpu").manual_seed(N)
    Wb = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16)
    Wb[0] = 0  # all-zero row: scale 0
    q, s = lai.quantize_rows_i8(Wb.to(DEV))
    qo, so = oracle.quantize_rows_i8_bf16(wbits(Wb))
    assert np.array_equal(s.cpu().numpy().view(np.uint32), so.view(np.uint32))
    assert np.array_equal(q.cpu().numpy(), qo)


def test_convert_bf16_to_f16_bit_exact():
    g = torch.Generator(device="cpu").manual_seed(3)
    x = torch.randn(1 << 16, generator=g) * torch.pow(10.0, torch.randint(-8, 6, (1 << 16,),
                                                                        generator=g).float())
    x[:6] = torch.tensor([0.0, -0.0, 65504.0, 70000.0, float("inf"), 2.0 ** -24])
    xb = x.to(torch.bfloat16)
    got = lai.convert_bf16_to_f16(xb.to(DEV)).cpu().view(torch.int16).numpy().view(np.uint16)
    want = oracle.f32_to_f16_bits(xb.float().numpy())
    assert np.array_equal(got, want)


def test_i8_decode_layer_tracks_bf16():
    # quantising a layer's weights changes its outputs by the quantisation error only
    # (scale / 2 per weight), the reference's int8 trade-off
    M, K, N = 1, 2048, 2048
    x, W, _ = make(M, K, N, 21)
    q, s = lai.quantize_rows_i8(W.to(DEV))
    y8 = lai.gemv(x.to(DEV), q, scales=s)
    y16 = lai.gemv(x.to(DEV), W.to(DEV))
    torch.cuda.synchronize()
    bound = (s.cpu() / 2)[None, :] * x.abs().sum(1, keepdim=True)  # |sum (w - q s) x| bound
    assert ((y8 - y16).abs().cpu() <= bound + 1e-5).all()

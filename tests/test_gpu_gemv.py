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


# ---- the decode step's GEMVs as one persistent chain kernel (lai_gemv_chain_*) -----------
def chain_layers(L, D, QD, KV, I, seed):
    """L decoder layers' weights and norms (q|k|v rows concatenated, gate/up interleaved)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    mk = lambda n, k: (torch.randn(n, k, generator=g) / np.sqrt(k)).to(torch.bfloat16)  # noqa: E731
    layers = [dict(qkv=mk(QD + 2 * KV, D), o=mk(D, QD), gu=mk(2 * I, D), down=mk(D, I),
                   w_in=1 + 0.02 * torch.randn(D, generator=g),
                   w_post=1 + 0.02 * torch.randn(D, generator=g)) for _ in range(L)]
    x = torch.randn(D, generator=g)
    attn = torch.randn(QD, generator=g)
    return layers, x, attn


def chain_oracle(layers, x, attn, eps):
    """The reference's per-layer decode sequence (src/tts_native.c:637-668) in the oracle."""
    x = x.numpy()[None].copy()
    a = attn.numpy()[None]
    for ly in layers:
        qkv = oracle.linear_bf16(oracle.rms_norm(x, ly["w_in"].numpy(), eps), wbits(ly["qkv"]))
        x = oracle.add_inplace(x, oracle.linear_bf16(a, wbits(ly["o"])))
        gu = oracle.linear_bf16(oracle.rms_norm(x, ly["w_post"].numpy(), eps), wbits(ly["gu"]))
        act = oracle.swiglu_multiply(gu, ly["gu"].shape[0] // 2)
        x = oracle.add_inplace(x, oracle.linear_bf16(act, wbits(ly["down"])))
    return x[0], qkv[0], act[0]


def build_chain(layers, x, attn, eps):
    xd, ad = x.to(DEV), attn.to(DEV)
    qkv = torch.empty(layers[0]["qkv"].shape[0], device=DEV)
    act = torch.empty(layers[0]["gu"].shape[0] // 2, device=DEV)
    dev = [{k: v.to(DEV) for k, v in ly.items()} for ly in layers]
    ops = []
    for ly in dev:
        ops += [(lai.CHAIN_STORE, ly["qkv"], xd, ly["w_in"], qkv, eps),
                (lai.CHAIN_RESIDUAL, ly["o"], ad, None, xd, 0.0),
                (lai.CHAIN_SWIGLU, ly["gu"], xd, ly["w_post"], act, eps),
                (lai.CHAIN_RESIDUAL, ly["down"], act, None, xd, 0.0)]
    return lai.GemvChain(ops), xd, qkv, act


# (layers, hidden, q dim, kv dim, FFN): the 0.6B talker, the 1.7B shapes (down K = 6144), and
# a narrow model (1-3 rows per SM)
CHAIN_SHAPES = [(3, 1024, 2048, 1024, 3072), (2, 2048, 2048, 1024, 6144), (2, 256, 256, 64, 256)]


@pytest.mark.parametrize("L,D,QD,KV,I", CHAIN_SHAPES)
def test_gemv_chain_matches_oracle(L, D, QD, KV, I):
    layers, x, attn = chain_layers(L, D, QD, KV, I, L + D)
    chain, xd, qkv, act = build_chain(layers, x, attn, 1e-6)
    chain.run()
    torch.cuda.synchronize()
    assert int(chain.err.item()) == 0
    rx, rqkv, ract = chain_oracle(layers, x, attn, 1e-6)
    assert max_rel_err(qkv.cpu().numpy(), rqkv) <= TOL_F32
    assert max_rel_err(act.cpu().numpy(), ract) <= TOL_F32
    assert max_rel_err(xd.cpu().numpy(), rx) <= TOL_F32


def test_gemv_chain_ops_with_fewer_rows_than_ctas():
    # most CTAs own no rows of these ops but still take part in every grid barrier
    g = torch.Generator(device="cpu").manual_seed(9)
    K = 512
    x = torch.randn(K, generator=g)
    w = 1 + 0.02 * torch.randn(K, generator=g)
    Ws = (torch.randn(64, K, generator=g) / 23).to(torch.bfloat16)
    Wg = (torch.randn(100, K, generator=g) / 23).to(torch.bfloat16)   # 50 gate/up pairs
    Wr = (torch.randn(20, 256, generator=g) / 16).to(torch.bfloat16)   # residual: 20 rows of K = 256
    r0 = torch.randn(20, generator=g)
    a = torch.randn(256, generator=g)
    xd, wd, ad = x.to(DEV), w.to(DEV), a.to(DEV)
    ys, yg, rr = torch.empty(64, device=DEV), torch.empty(50, device=DEV), r0.to(DEV)
    chain = lai.GemvChain([(lai.CHAIN_STORE, Ws.to(DEV), xd, wd, ys, 1e-5),
                           (lai.CHAIN_SWIGLU, Wg.to(DEV), xd, None, yg, 0.0),
                           (lai.CHAIN_RESIDUAL, Wr.to(DEV), ad, None, rr, 0.0)])
    chain.run()
    torch.cuda.synchronize()
    assert int(chain.err.item()) == 0
    xn = oracle.rms_norm(x.numpy()[None], w.numpy(), 1e-5)
    assert max_rel_err(ys.cpu().numpy(), oracle.linear_bf16(xn, wbits(Ws))[0]) <= TOL_F32
    gu = oracle.linear_bf16(x.numpy()[None], wbits(Wg))
    assert max_rel_err(yg.cpu().numpy(), oracle.swiglu_multiply(gu, 50)[0]) <= TOL_F32
    ref = oracle.add_inplace(r0.numpy()[None], oracle.linear_bf16(a.numpy()[None], wbits(Wr)))
    assert max_rel_err(rr.cpu().numpy(), ref[0]) <= TOL_F32


@pytest.mark.parametrize("name", ["g1", "g2"])
def test_gemv_chain_equals_per_op_launches_over_28_layers(name):
    # a full decode step's linear path: the chain kernel vs one fused-GEMV launch per projection
    import runner
    cfg = runner.DECODE_CONFIGS[name]
    a = runner.DecodeLinear(cfg, seed=11, chain=True)
    b = runner.DecodeLinear(cfg, seed=11)
    for f in a.launches():
        f()
    for f in b.launches():
        f()
    torch.cuda.synchronize()
    assert int(a.chain.err.item()) == 0
    for u, v in [(a.x, b.x), (a.qkv, b.qkv), (a.act, b.act)]:
        assert max_rel_err(u.cpu().numpy(), v.cpu().numpy()) <= 1e-4
    assert torch.isfinite(a.x).all()


def test_gemv_chain_captured_in_a_graph_repeats():
    layers, x, attn = chain_layers(2, 1024, 2048, 1024, 3072, 5)
    chain, xd, qkv, act = build_chain(layers, x, attn, 1e-6)
    x0 = xd.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        chain.run(s)  # warm up outside the capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    once = xd.clone()
    xd.copy_(x0)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        chain.run(torch.cuda.current_stream())
    xd.copy_(x0)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(xd, once)  # same partition, same order: the same bits
    g.replay()  # a second replay re-zeroes the grid counter and continues from the new x
    torch.cuda.synchronize()
    assert int(chain.err.item()) == 0
    del g


def test_gemv_chain_argument_checks():
    import ctypes
    from conftest import arena_ptr
    L = lai.load()
    P = arena_ptr(0)

    def create(**kw):
        op = dict(w=arena_ptr(1 << 20), in_=arena_ptr(4096), norm_w=None, out=arena_ptr(1 << 16),
                  n=8, k=256, epilogue=lai.CHAIN_STORE, eps=1e-6)
        op.update(kw)
        arr = (lai.GemvChainOp * 1)(lai.GemvChainOp(**{k: (v.value if isinstance(v, ctypes.c_void_p)
                                                          else v) for k, v in op.items()}))
        h = ctypes.c_void_p()
        st = L.lai_gemv_chain_create(ctypes.byref(h), arr, 1)
        if h.value:
            L.lai_gemv_chain_destroy(h)
        return st

    assert create(k=100) == lai.LAI_ERR_INVALID         # k not a multiple of 256
    assert create(k=8192) == lai.LAI_ERR_TOOBIG         # a row beyond one stage
    assert create(epilogue=lai.CHAIN_SWIGLU, n=7) == lai.LAI_ERR_INVALID  # odd gate/up rows
    assert create(out=arena_ptr(4096 + 16)) == lai.LAI_ERR_ALIAS  # output over the input
    assert create(n=1 << 20) == lai.LAI_ERR_TOOBIG      # more rows per SM than staged results
    assert create() == lai.LAI_OK
    assert L.lai_gemv_chain_run(None, P, None) == lai.LAI_ERR_INVALID

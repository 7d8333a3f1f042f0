"""CUDA kernels vs the CPU oracle on identical seeded inputs, through the C ABI.

Tolerances (conftest): FP32 paths max |d|/max(1,|ref|) <= 1e-5; BF16 storage
paths <= 1e-2 against the oracle's BF16 variant on the same BF16 inputs; the
gather is bit-exact. Sizes are the configs' shapes cut to what the oracle
finishes in seconds, plus ragged / odd / unaligned edge cases.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_BF16, TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_bits(t):
    return t.detach().view(torch.int16).cpu().numpy().view(np.uint16)


def from_bits(a):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(DEV).view(torch.bfloat16)


def f32(t):
    return t.detach().float().cpu().numpy()


def rand(shape, seed, dtype=torch.float32, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (scale * torch.randn(shape, generator=g)).to(dtype).to(DEV)


def norm_w(n, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (1.0 + 0.02 * torch.randn(n, generator=g)).float().to(DEV)


# ---------------------------------------------------------------- RMSNorm
RMS_SHAPES = [(512, 1024), (64, 2048), (256, 1024), (33, 512), (7, 200), (5, 1000), (3, 4096),
              (1, 1024), (9, 768)]


@pytest.mark.parametrize("rows,dim", RMS_SHAPES)
def test_rmsnorm_f32(rows, dim):
    x, w = rand((rows, dim), 1), norm_w(dim, 2)
    y = lai.rmsnorm(x, w, 1e-6)
    torch.cuda.synchronize()
    assert max_rel_err(f32(y), oracle.rms_norm(f32(x), f32(w), 1e-6)) <= TOL_F32


@pytest.mark.parametrize("rows,dim", RMS_SHAPES)
def test_rmsnorm_bf16(rows, dim):
    x, w = rand((rows, dim), 3, torch.bfloat16), norm_w(dim, 4)
    y = lai.rmsnorm(x, w, 1e-6)
    ref = oracle.rms_norm_bf16(bf16_bits(x), f32(w), 1e-6)
    got = bf16_bits(y)
    assert max_rel_err(oracle.bf16_bits_to_f32(got), oracle.bf16_bits_to_f32(ref)) <= TOL_BF16
    assert np.mean(got == ref) > 0.99  # almost all bit-identical after rounding


def test_rmsnorm_in_place_and_vocoder_eps():
    x, w = rand((40, 512), 5), norm_w(512, 6)
    ref = oracle.rms_norm(f32(x), f32(w), 1e-5)
    lai.rmsnorm(x, w, 1e-5, y=x)  # out == x (src/tts_native.c:674)
    torch.cuda.synchronize()
    assert max_rel_err(f32(x), ref) <= TOL_F32


def test_rmsnorm_unaligned_rows_take_fallback():
    base = rand((17 * 1024 + 1,), 7)
    x = base[1:].view(17, 1024)  # 4-byte offset: not 16-byte aligned
    w = norm_w(1024, 8)
    y = lai.rmsnorm(x, w, 1e-6)
    torch.cuda.synchronize()
    assert max_rel_err(f32(y), oracle.rms_norm(f32(x), f32(w), 1e-6)) <= TOL_F32


# ---------------------------------------------------------- add + RMSNorm
@pytest.mark.parametrize("rows,dim", [(512, 1024), (128, 2048), (13, 200), (256, 1024)])
def test_add_rmsnorm_bf16_equals_reference_sequence(rows, dim):
    x, d, w = rand((rows, dim), 9, torch.bfloat16), rand((rows, dim), 10, torch.bfloat16), norm_w(dim, 11)
    xo_ref, y_ref = oracle.add_rms_norm_bf16(bf16_bits(x), bf16_bits(d), f32(w), 1e-6)
    y = lai.add_rmsnorm(x, d, w, 1e-6)
    assert np.array_equal(bf16_bits(x), xo_ref)  # residual: one RNE rounding, bit-exact
    got = oracle.bf16_bits_to_f32(bf16_bits(y))
    assert max_rel_err(got, oracle.bf16_bits_to_f32(y_ref)) <= TOL_BF16


@pytest.mark.parametrize("rows,dim", [(64, 2048), (40, 512), (9, 100)])
def test_add_rmsnorm_f32(rows, dim):
    x, d, w = rand((rows, dim), 12), rand((rows, dim), 13), norm_w(dim, 14)
    xo_ref, y_ref = oracle.add_rms_norm_f32(f32(x), f32(d), f32(w), 1e-6)
    y = lai.add_rmsnorm(x, d, w, 1e-6)
    assert np.array_equal(f32(x), xo_ref)
    assert max_rel_err(f32(y), y_ref) <= TOL_F32


def test_add_rmsnorm_fused_equals_unfused_bf16():
    x, d, w = rand((300, 2048), 15, torch.bfloat16), rand((300, 2048), 16, torch.bfloat16), norm_w(2048, 17)
    x2 = x.clone()
    y_fused = lai.add_rmsnorm(x, d, w, 1e-6)
    lai.add(x2, d)
    y_unfused = lai.rmsnorm(x2, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(x, x2) and torch.equal(y_fused, y_unfused)


# ------------------------------------------------------- q/k norm + RoPE
def table(rows, hd, theta):
    pos = torch.arange(rows, dtype=torch.int32, device=DEV)
    return lai.rope_table(pos, rows, hd, theta)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,nq,nkv,hd,posmode", [
    (512, 16, 8, 128, "seq"),      # config 1 prefill, positions 0..511
    (256, 16, 8, 128, "random"),   # config 3 decode, positions U[0, 4095]
    (5003, 16, 8, 128, "random"),  # several tiles per persistent CTA, partial last tile
    (64, 16, 16, 64, "seq"),       # vocoder pre-transformer heads (hd 64)
    (7, 3, 1, 128, "random"),      # odd head counts -> generic kernel
    (3001, 32, 8, 128, "random"),  # 32 q heads: the per-warp stream kernel, fewer warps per CTA
    (5, 2, 2, 96, "seq"),          # head_dim without a fast path
])
def test_qk_norm_rope(dtype, rows, nq, nkv, hd, posmode):
    bf = dtype == torch.bfloat16
    q, k = rand((rows, nq * hd), 20, dtype), rand((rows, nkv * hd), 21, dtype)
    wq, wk = norm_w(hd, 22), norm_w(hd, 23)
    cos_t, sin_t = table(4096, hd, 1e6)
    if posmode == "random":
        g = torch.Generator(device="cpu").manual_seed(24)
        pos = torch.randint(0, 4096, (rows,), generator=g, dtype=torch.int32).to(DEV)
    else:
        pos = torch.arange(rows, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    qh, kh = (bf16_bits(q), bf16_bits(k)) if bf else (f32(q), f32(k))
    lai.qk_norm_rope(q, k, wq, wk, cos_t, sin_t, pos, nq, nkv, hd, 1e-6, err=err)
    qr, kr = oracle.qk_norm_rope(qh, kh, f32(wq), f32(wk), f32(cos_t), f32(sin_t),
                                 pos.cpu().numpy(), nq, nkv, hd, 1e-6, bf16=bf)
    assert int(err.item()) == 0
    if bf:
        assert max_rel_err(oracle.bf16_bits_to_f32(bf16_bits(q)), oracle.bf16_bits_to_f32(qr)) <= TOL_BF16
        assert max_rel_err(oracle.bf16_bits_to_f32(bf16_bits(k)), oracle.bf16_bits_to_f32(kr)) <= TOL_BF16
    else:
        assert max_rel_err(f32(q), qr) <= TOL_F32
        assert max_rel_err(f32(k), kr) <= TOL_F32


def test_qk_q_only_bf16_qwen_heads():
    # k = NULL with the Qwen3 16-head q layout (the register kernel without k passes)
    rows, nq, hd = 777, 16, 128
    q = rand((rows, nq * hd), 35, torch.bfloat16)
    wq = norm_w(hd, 36)
    cos_t, sin_t = table(4096, hd, 1e6)
    g = torch.Generator(device="cpu").manual_seed(37)
    pos = torch.randint(0, 4096, (rows,), generator=g, dtype=torch.int32).to(DEV)
    qh = bf16_bits(q)
    lai.qk_norm_rope(q, None, wq, None, cos_t, sin_t, pos, nq, 0, hd, 1e-6)
    qr, _ = oracle.qk_norm_rope(qh, None, f32(wq), None, f32(cos_t), f32(sin_t),
                                pos.cpu().numpy(), nq, 0, hd, 1e-6, bf16=True)
    assert max_rel_err(oracle.bf16_bits_to_f32(bf16_bits(q)), oracle.bf16_bits_to_f32(qr)) <= TOL_BF16


def test_qk_result_does_not_depend_on_batch_size():
    # one large call (persistent ring kernel) vs 100-row calls (warp-per-token kernel)
    rows, nq, nkv, hd = 5000, 16, 8, 128
    q, k = rand((rows, nq * hd), 27, torch.bfloat16), rand((rows, nkv * hd), 28, torch.bfloat16)
    wq, wk = norm_w(hd, 29), norm_w(hd, 30)
    cos_t, sin_t = table(4096, hd, 1e6)
    g = torch.Generator(device="cpu").manual_seed(31)
    pos = torch.randint(0, 4096, (rows,), generator=g, dtype=torch.int32).to(DEV)
    q2, k2 = q.clone(), k.clone()
    lai.qk_norm_rope(q, k, wq, wk, cos_t, sin_t, pos, nq, nkv, hd, 1e-6)
    for r0 in range(0, rows, 100):
        lai.qk_norm_rope(q2[r0:r0 + 100], k2[r0:r0 + 100], wq, wk, cos_t, sin_t, pos[r0:r0 + 100],
                         nq, nkv, hd, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(q, q2) and torch.equal(k, k2)


def test_rope_only_is_bit_exact_f32():
    # separately rounded products, same as the reference's scalar C: bit-exact
    q = rand((64, 16 * 128), 25)
    cos_t, sin_t = table(64, 128, 1e6)
    ref = oracle.apply_rope_neox(f32(q), f32(cos_t), f32(sin_t), 16, 128)
    lai.qk_norm_rope(q, None, None, None, cos_t, sin_t, None, 16, 0, 128, 0.0)
    torch.cuda.synchronize()
    assert np.array_equal(f32(q), ref)


def test_rope_table_matches_reference_builder():
    pos = torch.randint(0, 4096, (300,), dtype=torch.int32).to(DEV)
    for hd, theta in [(128, 1e6), (64, 1e4)]:
        c, s = lai.rope_table(pos, 300, hd, theta)
        cr, sr = oracle.compute_rope_neox(pos.cpu().numpy(), hd, theta)
        torch.cuda.synchronize()
        assert max_rel_err(f32(c), cr) <= TOL_F32 and max_rel_err(f32(s), sr) <= TOL_F32


def test_rope_position_out_of_range_sets_flag_and_skips_row():
    q = rand((4, 2 * 128), 26, torch.bfloat16)
    before = q.clone()
    cos_t, sin_t = table(16, 128, 1e6)
    pos = torch.tensor([0, 16, -1, 3], dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    lai.qk_norm_rope(q, None, None, None, cos_t, sin_t, pos, 2, 0, 128, 0.0, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & lai.LAI_DEVERR_POSITION
    assert torch.equal(q[1], before[1]) and torch.equal(q[2], before[2])
    assert torch.equal(q[0], before[0])  # position 0 is the identity rotation


# ----------------------------------------------------------------- SwiGLU
@pytest.mark.parametrize("rows,inter", [(512, 3072), (64, 6144), (256, 3072), (3, 5), (1, 1), (2, 7)])
def test_swiglu_bf16(rows, inter):
    gu = rand((rows, 2 * inter), 30, torch.bfloat16, scale=2.0)
    out = lai.swiglu(gu, inter)
    ref = oracle.swiglu_bf16(bf16_bits(gu), inter)
    assert max_rel_err(oracle.bf16_bits_to_f32(bf16_bits(out)), oracle.bf16_bits_to_f32(ref)) <= TOL_BF16


@pytest.mark.parametrize("rows,inter", [(64, 3072), (5, 1000), (3, 5), (1, 1)])
def test_swiglu_f32(rows, inter):
    gu = rand((rows, 2 * inter), 31, scale=2.0)
    out = lai.swiglu(gu, inter)
    torch.cuda.synchronize()
    assert max_rel_err(f32(out), oracle.swiglu_multiply(f32(gu), inter)) <= TOL_F32


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("rows,inter", [(1, 4), (3, 5), (16, 3072), (257, 1000), (2048, 3072),
                                        (21000, 3071)])
def test_swiglu_in_place_equals_out_of_place(dtype, rows, inter):
    # (2048, 3072): the cooperative launch's head and waves only; (21000, 3071): waves of
    # 4M+ units as ordinary launches after it, and a ragged tail
    gu = rand((rows, 2 * inter), 32, dtype, scale=2.0)
    ref = lai.swiglu(gu, inter)
    got = lai.swiglu_inplace(gu, inter)
    torch.cuda.synchronize()
    assert torch.equal(got, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_swiglu_in_place_captured_in_a_graph(dtype):
    # the in-place form is a cooperative launch (+ wave launches when large): it must capture
    rows, inter = 4096, 3072
    src = rand((rows, 2 * inter), 38, dtype, scale=2.0)
    ref = lai.swiglu(src, inter)
    buf = src.clone()
    stream, graph = torch.cuda.Stream(), torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        lai.swiglu_inplace(buf.clone(), inter)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=stream):
            lai.swiglu_inplace(buf, inter)
    for _ in range(2):
        buf.copy_(src)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(buf.view(-1)[: rows * inter], ref.view(-1))


def test_swiglu_in_place_unaligned_buffer():
    base = rand((2 * 300 * 7 + 1,), 33, scale=2.0)
    gu = base[1:].view(300, 14)
    ref = oracle.swiglu_multiply(f32(gu), 7)
    got = lai.swiglu_inplace(gu, 7)
    torch.cuda.synchronize()
    assert max_rel_err(f32(got), ref) <= TOL_F32


def test_silu_and_swiglu_separate_f32():
    x = rand((1000 + 3,), 34, scale=4.0)
    ref = oracle.silu(f32(x))
    lai.call("lai_silu_f32", lai._p(x), x.numel(), lai._s(None))
    torch.cuda.synchronize()
    assert max_rel_err(f32(x), ref) <= TOL_F32
    g, u = rand((4099,), 35, scale=3.0), rand((4099,), 36)
    out = torch.empty_like(g)
    lai.call("lai_swiglu_separate_f32", lai._p(out), lai._p(g), lai._p(u), g.numel(), lai._s(None))
    torch.cuda.synchronize()
    assert max_rel_err(f32(out), oracle.swiglu_separate(f32(g), f32(u))) <= TOL_F32


# ------------------------------------------------------------ residual add
@pytest.mark.parametrize("n", [1, 7, 8, 1024 * 256 + 3])
def test_add(n):
    for dt in (torch.bfloat16, torch.float32):
        x, y = rand((n,), 40, dt), rand((n,), 41, dt)
        if dt == torch.bfloat16:
            ref = oracle.add_bf16(bf16_bits(x), bf16_bits(y))
            lai.add(x, y)
            assert np.array_equal(bf16_bits(x), ref)
        else:
            ref = oracle.add_inplace(f32(x), f32(y))
            lai.add(x, y)
            torch.cuda.synchronize()
            assert np.array_equal(f32(x), ref)


# ------------------------------------------------------------------ gather
@pytest.mark.parametrize("vocab,dim,n", [(151936, 1024, 512), (3072, 1024, 256), (2048, 2048, 64),
                                          (100, 12, 9), (50, 1000, 5)])
def test_gather_bit_exact(vocab, dim, n):
    g = torch.Generator(device="cpu").manual_seed(50)
    tbl = torch.randint(-32768, 32768, (vocab, dim), generator=g, dtype=torch.int32)
    tbl = tbl.to(torch.int16).to(DEV).view(torch.bfloat16)
    ids = torch.randint(0, vocab, (n,), generator=g, dtype=torch.int32).to(DEV)
    out16 = lai.embed_gather(tbl, ids, to_f32=False)
    out32 = lai.embed_gather(tbl, ids, to_f32=True)
    th, ih = bf16_bits(tbl), ids.cpu().numpy()
    assert np.array_equal(bf16_bits(out16), oracle.gather_bf16(th, ih))
    ref32 = oracle.gather_bf16_to_f32(th, ih)
    assert np.array_equal(out32.cpu().numpy().view(np.uint32), ref32.view(np.uint32))  # NaN payloads too


def test_gather_out_of_range_ids_flag_and_zero_rows():
    tbl = rand((10, 16), 51, torch.bfloat16)
    ids = torch.tensor([1, 10, -3, 9], dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = lai.embed_gather(tbl, ids, to_f32=True, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & lai.LAI_DEVERR_TOKEN_ID
    assert torch.all(out[1] == 0) and torch.all(out[2] == 0)
    assert torch.equal(out[0], tbl[1].float()) and torch.equal(out[3], tbl[9].float())


# -------------------------------------------------------------- SnakeBeta
@pytest.mark.parametrize("batch,C,T", [(1, 96, 1919), (2, 192, 4000), (1, 1536, 2000), (3, 5, 3),
                                        (1, 7, 1), (2, 768, 15992), (2, 10, 6), (1, 33, 4),
                                        (3, 17, 5)])
def test_snake_beta_vs_reference_build(batch, C, T):
    x = rand((batch, C, T), 60)
    g = torch.Generator(device="cpu").manual_seed(61)
    ea = torch.exp(0.1 * torch.randn(C, generator=g)).float().to(DEV)
    ieb = (1.0 / torch.exp(0.1 * torch.randn(C, generator=g))).float().to(DEV)
    xh = f32(x)
    lai.snake_beta(x, ea, ieb)
    if oracle.have_ref():
        ref = oracle.ref_snake_beta(xh, f32(ea), f32(ieb), "scalar")  # the reference's own C
    else:
        ref = oracle.snake_beta(xh, f32(ea), f32(ieb))
    got = f32(x)
    assert max_rel_err(got, ref) <= TOL_F32


def test_snake_beta_wide_arguments_and_fallback():
    # |ea*x| across the reduction's range, past its 65536 limit (CUDA sinf takes
    # over), zeros, tiny values and infinities; oracle = the reference's scalar build
    g = torch.Generator(device="cpu").manual_seed(63)
    C, T = 6, 4096
    mags = torch.tensor([1.0, 10.0, 1e3, 3e4, 6e4, 2e5])[:, None]
    x = (mags * (2 * torch.rand(C, T, generator=g) - 1)).float()
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-30, -1e-20, 1.5707964, 3.1415927, 65536.0, -65537.0])
    x[5, :2] = torch.tensor([float("inf"), float("-inf")])
    ea = torch.tensor([1.0, 1.3, 0.7, 1.0, 1.1, 1.0])
    ieb = torch.tensor([1.0, 0.8, 1.2, 0.9, 1.0, 1.0])
    xd = x.to(DEV)
    lai.snake_beta(xd, ea.to(DEV), ieb.to(DEV))
    ref = oracle.ref_snake_beta(x.numpy(), ea.numpy(), ieb.numpy()) if oracle.have_ref() \
        else oracle.snake_beta(x.numpy(), ea.numpy(), ieb.numpy())
    got = f32(xd)
    fin = np.isfinite(ref)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    assert max_rel_err(got[fin], ref[fin]) <= TOL_F32
    # the increment itself (x' - x = ieb * sin^2) to absolute 1e-6 where |x| < 2, so
    # that the output's own rounding (ulp <= 2.4e-7) does not swamp it
    small = fin & (np.abs(x.numpy()) < 2)
    inc_err = np.abs((got - x.numpy())[small] - (ref - x.numpy())[small])
    assert inc_err.max() <= 1e-6


def test_snake_beta_unaligned_base():
    base = rand((1 + 4 * 999,), 62)
    x = base[1:].view(4, 999)
    ea = torch.full((4,), 1.1, device=DEV)
    ieb = torch.full((4,), 0.9, device=DEV)
    ref = oracle.snake_beta(f32(x), f32(ea), f32(ieb))
    lai.call("lai_snake_beta_f32", lai._p(x), lai._p(ea), lai._p(ieb), 1, 4, 999, lai._s(None))
    torch.cuda.synchronize()
    assert max_rel_err(f32(x), ref) <= TOL_F32


# ----------------------------------------------------------- synth inputs
def test_synth_is_shard_invariant():
    full = torch.empty(1 << 16, dtype=torch.bfloat16, device=DEV)
    lai.synth_normal(full, seed=7)
    half = torch.empty(1 << 15, dtype=torch.bfloat16, device=DEV)
    lai.synth_normal(half, seed=7, offset=1 << 15)
    torch.cuda.synchronize()
    assert torch.equal(full[1 << 15:], half)
    f = full.float()
    assert abs(f.mean().item()) < 0.05 and abs(f.std().item() - 1.0) < 0.05

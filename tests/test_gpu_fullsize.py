"""Parity at the configs' full sizes through size-independent properties.

The oracle cannot run 65 536-token layers in seconds, so at full size the tests
use properties that hold whatever the size: fused == unfused and in place ==
out of place bit for bit, per-head RMS of a normalised head, RoPE's preservation
of each rotated pair's norm, bit-exact gathers, and sampled rows (rows are
independent) against the oracle.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_BF16, TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"

T2, D2, I2, NQ, NKV, HD = 65536, 2048, 6144, 16, 8, 128  # config 2


def randn(shape, seed, dtype=torch.bfloat16, std=1.0):
    t = torch.empty(shape, dtype=dtype, device=DEV)
    return lai.synth_normal(t, seed=seed, std=std)


def bits(t):
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def sample_rows(n, k, seed):
    return np.sort(np.random.default_rng(seed).choice(n, size=k, replace=False))


def test_add_rmsnorm_fused_equals_unfused_full_size():
    x, d = randn((T2, D2), 1), randn((T2, D2), 2)
    w = randn((D2,), 3, torch.float32, std=0.02) + 1
    x2 = x.clone()
    y = lai.add_rmsnorm(x, d, w, 1e-6)
    lai.add(x2, d)
    y2 = lai.rmsnorm(x2, w, 1e-6)
    torch.cuda.synchronize()
    assert torch.equal(x, x2) and torch.equal(y, y2)
    rows = sample_rows(T2, 64, 4)
    ref = oracle.rms_norm_bf16(bits(x[rows]), w.cpu().numpy(), 1e-6)
    assert max_rel_err(oracle.bf16_bits_to_f32(bits(y[rows])), oracle.bf16_bits_to_f32(ref)) <= TOL_BF16


def test_swiglu_in_place_equals_out_of_place_full_size():
    gu = randn((T2, 2 * I2), 5, std=2.0)
    out = lai.swiglu(gu, I2)
    got = lai.swiglu_inplace(gu.clone(), I2)
    torch.cuda.synchronize()
    assert torch.equal(got, out)
    rows = sample_rows(T2, 32, 6)
    ref = oracle.swiglu_bf16(bits(gu[rows]), I2)
    assert max_rel_err(oracle.bf16_bits_to_f32(bits(out[rows])), oracle.bf16_bits_to_f32(ref)) <= TOL_BF16


def test_qk_norm_rope_full_size_properties():
    q, k = randn((T2, NQ * HD), 7), randn((T2, NKV * HD), 8)
    wq = randn((HD,), 9, torch.float32, std=0.02) + 1
    wk = randn((HD,), 10, torch.float32, std=0.02) + 1
    P = 1024
    cos_t, sin_t = lai.rope_table(torch.arange(P, dtype=torch.int32, device=DEV), P, HD, 1e6)
    pos = (torch.arange(T2, device=DEV) % P).to(torch.int32)
    q0, k0 = q.clone(), k.clone()
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    lai.qk_norm_rope(q, k, wq, wk, cos_t, sin_t, pos, NQ, NKV, HD, 1e-6, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # sampled rows against the oracle
    rows = sample_rows(T2, 48, 11)
    qr, kr = oracle.qk_norm_rope(bits(q0[rows]), bits(k0[rows]), wq.cpu().numpy(), wk.cpu().numpy(),
                                 cos_t.cpu().numpy(), sin_t.cpu().numpy(), pos[rows].cpu().numpy(),
                                 NQ, NKV, HD, 1e-6, bf16=True)
    assert max_rel_err(oracle.bf16_bits_to_f32(bits(q[rows])), oracle.bf16_bits_to_f32(qr)) <= TOL_BF16
    assert max_rel_err(oracle.bf16_bits_to_f32(bits(k[rows])), oracle.bf16_bits_to_f32(kr)) <= TOL_BF16
    # every head of every row, unit weights: RoPE preserves |(x_d, x_{d+64})|, so after
    # norm + RoPE each head's mean square is 1 up to BF16 rounding
    q1 = q0.clone()
    ones = torch.ones(HD, dtype=torch.float32, device=DEV)
    lai.qk_norm_rope(q1, None, ones, None, cos_t, sin_t, pos, NQ, 0, HD, 1e-6)
    h = q1.float().view(T2, NQ, HD)
    ms = (h * h).mean(-1)
    assert torch.all((ms - 1.0).abs() < 1e-2)


def test_rope_only_full_size_pair_norms_and_samples_f32():
    T = 16384  # FP32 q: 128 MiB
    q = randn((T, NQ * HD), 12, torch.float32)
    P = 4096
    cos_t, sin_t = lai.rope_table(torch.arange(P, dtype=torch.int32, device=DEV), P, HD, 1e6)
    g = torch.Generator(device="cpu").manual_seed(13)
    pos = torch.randint(0, P, (T,), generator=g, dtype=torch.int32).to(DEV)
    q0 = q.clone()
    lai.qk_norm_rope(q, None, None, None, cos_t, sin_t, pos, NQ, 0, HD, 0.0)
    torch.cuda.synchronize()
    a0, a1 = q0.view(T, NQ, 2, 64), q.view(T, NQ, 2, 64)
    n0, n1 = (a0 * a0).sum(2), (a1 * a1).sum(2)
    assert torch.all((n1 - n0).abs() <= 1e-5 * torch.clamp(n0, min=1.0))
    rows = sample_rows(T, 64, 14)
    ref = oracle.qk_norm_rope(q0[rows].cpu().numpy(), None, None, None, cos_t.cpu().numpy(),
                              sin_t.cpu().numpy(), pos[rows].cpu().numpy(), NQ, 0, HD, 0.0,
                              bf16=False)[0]
    assert np.array_equal(q[rows].cpu().numpy(), ref)  # separately rounded: bit-exact


def test_gather_full_vocab_bit_exact():
    V, D, N = 151936, 1024, 512  # config 1
    table = randn((V, D), 15)
    ids = torch.empty(N, dtype=torch.int32, device=DEV)
    lai.synth_uniform_i32(ids, seed=16, lo=0, hi=V)
    out = lai.embed_gather(table, ids, to_f32=False)
    out32 = lai.embed_gather(table, ids, to_f32=True)
    ref = table.index_select(0, ids.long())
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    assert torch.equal(out32, ref.float())


def test_snake_largest_stage_sampled_rows():
    B, C, T = 8, 96, 192000  # config 4 stage 5
    x = randn((B, C, T), 17, torch.float32)
    ea = torch.exp(randn((C,), 18, torch.float32, std=0.1))
    ieb = 1.0 / torch.exp(randn((C,), 19, torch.float32, std=0.1))
    rows = sample_rows(B * C, 6, 20)
    before = x.view(B * C, T)[rows].cpu().numpy()
    lai.snake_beta(x, ea, ieb)
    torch.cuda.synchronize()
    got = x.view(B * C, T)[rows].cpu().numpy()
    ch = rows % C
    ea_h, ieb_h = ea.cpu().numpy(), ieb.cpu().numpy()
    for i in range(len(rows)):
        one = before[i:i + 1]
        ref = (oracle.ref_snake_beta(one, ea_h[ch[i]:ch[i] + 1], ieb_h[ch[i]:ch[i] + 1])
               if oracle.have_ref() else oracle.snake_beta(one, ea_h[ch[i]:ch[i] + 1], ieb_h[ch[i]:ch[i] + 1]))
        assert max_rel_err(got[i:i + 1], ref) <= TOL_F32

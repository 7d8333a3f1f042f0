"""Decode attention over the KV cache against the oracle.

The decode step's cache append + qwen_causal_attention with one query token per
sequence (src/tts_native.c:650-656; math of tools/verify_xfmr.py:57-77). The oracle
attends over the cache with row pos replaced by the new k/v, as the reference appends
before attending. FP32: max |d| / max(1, |ref|) <= 1e-5; the cache append is bit-exact.
"""
import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu
DEV = "cuda"
HD = 128


def make(S, H, Hkv, max_seq, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((S, H * HD)).astype(np.float32)
    kn = rng.standard_normal((S, Hkv * HD)).astype(np.float32)
    vn = rng.standard_normal((S, Hkv * HD)).astype(np.float32)
    kc = rng.standard_normal((S, max_seq, Hkv * HD)).astype(np.float32)
    vc = rng.standard_normal((S, max_seq, Hkv * HD)).astype(np.float32)
    return q, kn, vn, kc, vc


def run(q, kn, vn, kc, vc, pos, H, Hkv, scratch=None):
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    kcd, vcd = t(kc), t(vc)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = lai.decode_attention(t(q), t(kn), t(vn), kcd, vcd, t(np.asarray(pos, np.int32)), H,
                               Hkv, scratch=scratch, err=err)
    torch.cuda.synchronize()
    return out.cpu().numpy(), kcd.cpu().numpy(), vcd.cpu().numpy(), int(err.item())


def expected(q, kn, vn, kc, vc, pos, H, Hkv):
    kc2, vc2 = kc.copy(), vc.copy()
    for s, p in enumerate(pos):
        kc2[s, p], vc2[s, p] = kn[s], vn[s]
    return oracle.decode_attention(q, kc2, vc2, np.asarray(pos, np.int32), H, Hkv, HD), kc2, vc2


# (sequences, heads, kv heads, cache rows, positions): one key; the 256-key split edges;
# a full 4096-row cache; GQA groups 1, 2, 4, 8
CASES = [(1, 16, 8, 64, [0]), (4, 16, 8, 1000, [0, 255, 256, 999]), (1, 16, 8, 4096, [4095]),
         (3, 16, 16, 600, [5, 300, 599]), (2, 16, 4, 700, [511, 512]),
         (2, 16, 2, 300, [1, 257])]


@pytest.mark.parametrize("S,H,Hkv,max_seq,pos", CASES)
def test_decode_attention(S, H, Hkv, max_seq, pos):
    q, kn, vn, kc, vc = make(S, H, Hkv, max_seq, S * 31 + max_seq)
    out, kcd, vcd, err = run(q, kn, vn, kc, vc, pos, H, Hkv)
    want, kc2, vc2 = expected(q, kn, vn, kc, vc, pos, H, Hkv)
    assert err == 0
    assert max_rel_err(out, want) <= TOL_F32
    assert np.array_equal(kcd, kc2) and np.array_equal(vcd, vc2)  # append exact, rest untouched


def test_decode_attention_talker_batch_random_positions():
    # the TTS talker decode config's attention: GQA 16/8, random positions up to 4095
    S, H, Hkv, max_seq = 32, 16, 8, 4096
    pos = np.random.default_rng(3).integers(0, max_seq, S)
    q, kn, vn, kc, vc = make(S, H, Hkv, max_seq, 7)
    out, _, _, err = run(q, kn, vn, kc, vc, pos, H, Hkv)
    want, _, _ = expected(q, kn, vn, kc, vc, pos, H, Hkv)
    assert err == 0 and max_rel_err(out, want) <= TOL_F32


def test_decode_attention_scratch_is_reusable():
    # consecutive decode steps share one scratch: the split counters reset themselves
    S, H, Hkv, max_seq = 3, 16, 8, 1200
    scratch = lai.decode_attention_scratch(S, H, Hkv, max_seq)
    for step, pos in enumerate(([700, 3, 1100], [701, 4, 1101], [1199, 900, 256])):
        q, kn, vn, kc, vc = make(S, H, Hkv, max_seq, 100 + step)
        out, _, _, err = run(q, kn, vn, kc, vc, pos, H, Hkv, scratch=scratch)
        want, _, _ = expected(q, kn, vn, kc, vc, pos, H, Hkv)
        assert err == 0 and max_rel_err(out, want) <= TOL_F32
    n_partial = S * H * ((max_seq + 255) // 256) * (HD + 2)  # floats before the counters
    assert not torch.any(scratch[n_partial:n_partial + S * Hkv].view(torch.int32))


def test_decode_attention_position_out_of_range_flags_and_skips():
    S, H, Hkv, max_seq = 2, 16, 8, 300
    q, kn, vn, kc, vc = make(S, H, Hkv, max_seq, 9)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    out = torch.full((S, H * HD), 7.0, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    kcd = t(kc)
    lai.decode_attention(t(q), t(kn), t(vn), kcd, t(vc), t(np.array([10, max_seq], np.int32)),
                         H, Hkv, out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == lai.LAI_DEVERR_POSITION
    assert torch.all(out[1] == 7.0)                      # skipped sequence untouched
    want, _, _ = expected(q[:1], kn[:1], vn[:1], kc[:1], vc[:1], [10], H, Hkv)
    assert max_rel_err(out[:1].cpu().numpy(), want) <= TOL_F32
    assert np.array_equal(kcd[1].cpu().numpy(), kc[1])   # its cache untouched


def test_decode_attention_argument_checks():
    L = lai.load()
    import ctypes
    from conftest import arena_ptr
    P = arena_ptr(1 << 20)  # real memory: a regressed check would still stay in bounds
    f = L.lai_decode_attention_f32
    # head_dim other than 128; heads not a multiple of kv heads; group of 3
    assert f(P, P, P, P, P, P, P, 1, 16, 8, 64, 100, 0.1, P, None, None) == lai.LAI_ERR_INVALID
    assert f(P, P, P, P, P, P, P, 1, 16, 6, 128, 100, 0.1, P, None, None) == lai.LAI_ERR_INVALID
    assert f(P, P, P, P, P, P, P, 1, 12, 4, 128, 100, 0.1, P, None, None) == lai.LAI_ERR_INVALID
    assert f(P, P, P, P, P, P, P, 0, 16, 8, 128, 100, 0.1, P, None, None) == lai.LAI_OK


# ---- the fused entry: per-head q/k RMSNorm + NeoX RoPE at pos folded into the launch -------
def rope_tables(rows, theta=1e6):
    inv = 1.0 / theta ** (np.arange(0, HD, 2, dtype=np.float64) / HD)
    ang = np.arange(rows)[:, None] * inv[None, :]
    c = np.concatenate([np.cos(ang), np.cos(ang)], 1).astype(np.float32)
    s = np.concatenate([np.sin(ang), np.sin(ang)], 1).astype(np.float32)
    return c, s


@pytest.mark.parametrize("S,H,Hkv,max_seq,pos", CASES[:4] + [(2, 16, 8, 300, [7, 299])])
@pytest.mark.parametrize("norm,rope", [(True, True), (True, False), (False, True)])
def test_decode_attention_qk_fused(S, H, Hkv, max_seq, pos, norm, rope):
    q, kn, vn, kc, vc = make(S, H, Hkv, max_seq, S * 7 + max_seq)
    rng = np.random.default_rng(max_seq)
    wq = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32) if norm else None
    wk = (1 + 0.1 * rng.standard_normal(HD)).astype(np.float32) if norm else None
    cos_t, sin_t = rope_tables(max_seq) if rope else (None, None)
    t = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(DEV)  # noqa: E731
    kcd, vcd = t(kc), t(vc)
    qd, knd = t(q), t(kn)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = lai.decode_attention(qd, knd, t(vn), kcd, vcd, t(np.asarray(pos, np.int32)), H, Hkv,
                               err=err, qk=(t(wq), t(wk), t(cos_t), t(sin_t), 1e-6))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(qd.cpu(), torch.from_numpy(q)) and torch.equal(knd.cpu(), torch.from_numpy(kn))
    # oracle: the separate per-head norm + RoPE at each sequence's pos, then attention
    qn, kn2 = oracle.qk_norm_rope(q, kn, wq, wk, cos_t, sin_t, np.asarray(pos, np.int32), H, Hkv,
                                  HD, 1e-6, bf16=False)
    want, kc2, vc2 = expected(qn, kn2, vn, kc, vc, pos, H, Hkv)
    assert max_rel_err(out.cpu().numpy(), want) <= TOL_F32
    assert max_rel_err(kcd.cpu().numpy(), kc2) <= TOL_F32  # the transformed key in the cache
    assert np.array_equal(vcd.cpu().numpy(), vc2)

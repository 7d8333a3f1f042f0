"""The reference-named FP32 drop-ins (qwen_*, voc_snake_beta) against the oracle.

Each function is exercised the way the reference calls it: on host buffers
(pageable malloc-style numpy arrays, and pinned memory), with the reference's
aliasing (out == x for RMSNorm, out == gate_up for SwiGLU), and on device
pointers. Multi-chunk sizes push the staged pipeline through several chunks.
"""
import ctypes

import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_F32, max_rel_err

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

V = ctypes.c_void_p


def hp(a: np.ndarray):
    return V(a.ctypes.data)


def lib():
    return lai.load()


def no_error():
    assert lib().lai_last_error() == lai.LAI_OK


def rng(seed):
    return np.random.default_rng(seed)


@pytest.mark.parametrize("seq,dim", [(1, 1024), (512, 1024), (3000, 2048), (33, 512)])
def test_qwen_rms_norm_host(seq, dim):
    r = rng(1)
    x = r.standard_normal((seq, dim), dtype=np.float32)
    w = (1 + 0.02 * r.standard_normal(dim)).astype(np.float32)
    out = np.empty_like(x)
    lib().qwen_rms_norm(hp(out), hp(x), hp(w), seq, dim, 1e-6)
    no_error()
    assert max_rel_err(out, oracle.rms_norm(x, w, 1e-6)) <= TOL_F32
    # in place, as src/tts_native.c:674 calls it
    ref = oracle.rms_norm(x, w, 1e-6)
    lib().qwen_rms_norm(hp(x), hp(x), hp(w), seq, dim, 1e-6)
    no_error()
    assert max_rel_err(x, ref) <= TOL_F32


def test_qwen_per_head_and_rope_host_prefill_and_decode():
    r = rng(2)
    seq, nq, nkv, hd = 300, 16, 8, 128
    q = r.standard_normal((seq, nq * hd), dtype=np.float32)
    k = r.standard_normal((seq, nkv * hd), dtype=np.float32)
    wq = (1 + 0.02 * r.standard_normal(hd)).astype(np.float32)
    cos_t, sin_t = oracle.compute_rope_neox(np.arange(1024), hd, 1e6)
    qr = oracle.apply_rope_neox(oracle.rms_norm_per_head(q, wq, nq, hd, 1e-6), cos_t[:seq], sin_t[:seq], nq, hd)
    lib().qwen_rms_norm_per_head(hp(q), hp(wq), seq, nq, hd, 1e-6)
    lib().qwen_apply_rope_neox(hp(q), hp(cos_t), hp(sin_t), seq, nq, hd)
    no_error()
    assert max_rel_err(q, qr) <= TOL_F32
    # decode: seq = 1, table pointer offset to row `pos` (src/tts_native.c:647-648)
    pos = 777
    k1 = np.ascontiguousarray(k[:1])
    kr = oracle.apply_rope_neox(k1, cos_t[pos:pos + 1], sin_t[pos:pos + 1], nkv, hd)
    c_row = np.ascontiguousarray(cos_t[pos:pos + 1])
    s_row = np.ascontiguousarray(sin_t[pos:pos + 1])
    lib().qwen_apply_rope_neox(hp(k1), hp(c_row), hp(s_row), 1, nkv, hd)
    no_error()
    assert np.array_equal(k1, kr)  # RoPE alone is bit-exact


def test_qwen_compute_rope_neox_host():
    pos = np.arange(0, 4096, 3, dtype=np.int32)
    c = np.empty((pos.size, 64), np.float32)
    s = np.empty_like(c)
    lib().qwen_compute_rope_neox(hp(c), hp(s), hp(pos), pos.size, 64, 1e4)
    no_error()
    cr, sr = oracle.compute_rope_neox(pos, 64, 1e4)
    assert max_rel_err(c, cr) <= TOL_F32 and max_rel_err(s, sr) <= TOL_F32


@pytest.mark.parametrize("seq,inter", [(1, 3072), (64, 3072), (1500, 6144), (5, 7)])
def test_qwen_swiglu_multiply_host_in_place(seq, inter):
    # out == gate_up, as every reference call site passes it; 1500 x 6144 spans
    # several staging chunks, so the aliasing order between chunks is exercised.
    r = rng(3)
    gu = (2 * r.standard_normal((seq, 2 * inter))).astype(np.float32)
    ref = oracle.swiglu_multiply(gu, inter)
    lib().qwen_swiglu_multiply(hp(gu), hp(gu), seq, inter)
    no_error()
    got = gu.reshape(-1)[: seq * inter].reshape(seq, inter)
    assert max_rel_err(got, ref) <= TOL_F32


def test_qwen_add_and_silu_host():
    r = rng(4)
    x = r.standard_normal(100003, dtype=np.float32)
    y = r.standard_normal(100003, dtype=np.float32)
    ref = oracle.add_inplace(x, y)
    lib().qwen_add_inplace(hp(x), hp(y), x.size)
    no_error()
    assert np.array_equal(x, ref)
    s = (4 * r.standard_normal(5001)).astype(np.float32)
    ref = oracle.silu(s)
    lib().qwen_silu(hp(s), s.size)
    no_error()
    assert max_rel_err(s, ref) <= TOL_F32


@pytest.mark.parametrize("C,T", [(96, 1919), (1536, 2000), (3, 5)])
def test_voc_snake_beta_host(C, T):
    r = rng(5)
    x = r.standard_normal((C, T), dtype=np.float32)
    ea = np.exp(0.1 * r.standard_normal(C)).astype(np.float32)
    ieb = (1 / np.exp(0.1 * r.standard_normal(C))).astype(np.float32)
    ref = oracle.ref_snake_beta(x, ea, ieb) if oracle.have_ref() else oracle.snake_beta(x, ea, ieb)
    lib().voc_snake_beta(hp(x), hp(ea), hp(ieb), C, T)
    no_error()
    assert max_rel_err(x, ref) <= TOL_F32


def test_pinned_host_and_device_pointers():
    seq, dim = 4096, 1024
    x = torch.randn(seq, dim).pin_memory()
    w = (1 + 0.02 * torch.randn(dim)).pin_memory()
    out = torch.empty(seq, dim).pin_memory()
    lib().qwen_rms_norm(V(out.data_ptr()), V(x.data_ptr()), V(w.data_ptr()), seq, dim, 1e-6)
    no_error()
    ref = oracle.rms_norm(x.numpy(), w.numpy(), 1e-6)
    assert max_rel_err(out.numpy(), ref) <= TOL_F32
    # device pointers: queued on the drop-in stream, no host copy
    xd, wd = x.cuda(), w.cuda()
    od = torch.empty_like(xd)
    lib().lai_set_stream(V(torch.cuda.current_stream().cuda_stream))
    lib().qwen_rms_norm(V(od.data_ptr()), V(xd.data_ptr()), V(wd.data_ptr()), seq, dim, 1e-6)
    no_error()
    torch.cuda.synchronize()
    assert max_rel_err(od.cpu().numpy(), ref) <= TOL_F32
    # device in-place SwiGLU through the drop-in (ordered waves, no scratch)
    gu = (2 * torch.randn(257, 2 * 1000)).cuda()
    ref = oracle.swiglu_multiply(gu.cpu().numpy(), 1000)
    lib().qwen_swiglu_multiply(V(gu.data_ptr()), V(gu.data_ptr()), 257, 1000)
    no_error()
    torch.cuda.synchronize()
    got = gu.view(-1)[: 257 * 1000].view(257, 1000).cpu().numpy()
    assert max_rel_err(got, ref) <= TOL_F32
    lib().lai_set_stream(None)


def test_embed_lookup_registered_host_table_and_device_table():
    r = rng(6)
    vocab, dim = 3072, 1024
    # page-aligned host table, as an mmap'd safetensors region would be
    raw = np.empty(vocab * dim * 2 + 8192, np.uint8)
    start = (-raw.ctypes.data) % 4096
    table = raw[start:start + vocab * dim * 2].view(np.uint16).reshape(vocab, dim)
    table[:] = r.integers(0, 1 << 16, size=(vocab, dim), dtype=np.uint32).astype(np.uint16)
    dst = np.empty(dim, np.float32)
    # an unregistered host table is refused with an error (no CPU fallback)
    lib().lai_embed_lookup_bf16(hp(dst), hp(table), 5, dim, vocab)
    assert lib().lai_last_error() == lai.LAI_ERR_INVALID
    assert lib().lai_register_host_table(hp(table), table.nbytes) == lai.LAI_OK
    try:
        for tid in (0, 1234, vocab - 1):
            lib().lai_embed_lookup_bf16(hp(dst), hp(table), tid, dim, vocab)
            no_error()
            want = oracle.gather_bf16_to_f32(table, np.array([tid], np.int32))[0]
            assert np.array_equal(dst.view(np.uint32), want.view(np.uint32))
        lib().lai_embed_lookup_bf16(hp(dst), hp(table), vocab, dim, vocab)
        assert lib().lai_last_error() == lai.LAI_ERR_RANGE
    finally:
        assert lib().lai_unregister_host_table(hp(table)) == lai.LAI_OK
    td = torch.from_numpy(table.view(np.int16)).cuda()
    lib().lai_embed_lookup_bf16(hp(dst), V(td.data_ptr()), 42, dim, vocab)
    no_error()
    want = oracle.gather_bf16_to_f32(table, np.array([42], np.int32))[0]
    assert np.array_equal(dst.view(np.uint32), want.view(np.uint32))


def _bits(t):
    return t.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("pinned", [True, False])
def test_staged_bf16_chain_equals_device_api(pinned):
    """Host-buffer BF16 entries give the device API's bytes (same kernels, staged rows)."""
    g = torch.Generator().manual_seed(21)
    T, D, I, nq, nkv, hd, P = 3000, 2048, 6144, 16, 8, 128, 1024
    bf = torch.bfloat16

    def host(*shape, dtype=bf):
        t = torch.randn(shape, generator=g).to(dtype)
        return t.pin_memory() if pinned else t

    x, dl, q, k, gu = host(T, D), host(T, D), host(T, nq * hd), host(T, nkv * hd), host(T, 2 * I)
    w, wq, wk = (1 + 0.02 * torch.randn(n, generator=g) for n in (D, hd, hd))
    pos = torch.randint(0, P, (T,), generator=g, dtype=torch.int32)
    ct, st = lai.rope_table(torch.arange(P, dtype=torch.int32, device="cuda"), P, hd, 1e6)
    ct_h, st_h = ct.cpu(), st.cpu()
    # device reference results
    xd, dd, qd, kd, gd = (t.cuda() for t in (x, dl, q, k, gu))
    yd = lai.add_rmsnorm(xd, dd, w.cuda(), 1e-6)
    lai.qk_norm_rope(qd, kd, wq.cuda(), wk.cuda(), ct, st, pos.cuda(), nq, nkv, hd, 1e-6)
    ad = lai.swiglu(gd, I)
    torch.cuda.synchronize()
    # staged host calls
    y = torch.empty_like(x)
    act = torch.empty(T, I, dtype=bf)
    L = lib()
    assert L.lai_staged_add_rmsnorm_bf16(V(x.data_ptr()), V(dl.data_ptr()), V(w.data_ptr()),
                                         V(y.data_ptr()), T, D, 1e-6) == lai.LAI_OK
    assert L.lai_staged_qk_norm_rope_bf16(V(q.data_ptr()), V(k.data_ptr()), V(wq.data_ptr()),
                                          V(wk.data_ptr()), V(ct_h.data_ptr()), V(st_h.data_ptr()),
                                          V(pos.data_ptr()), P, T, nq, nkv, hd, 1e-6) == lai.LAI_OK
    assert L.lai_staged_swiglu_bf16(V(act.data_ptr()), V(gu.data_ptr()), T, I) == lai.LAI_OK
    for got, want in [(x, xd), (y, yd), (q, qd), (k, kd), (act, ad)]:
        assert np.array_equal(_bits(got), _bits(want.cpu()))


def test_staged_qk_without_positions_uses_row_index_across_chunks():
    # pos NULL: row r uses table row r, also in chunks after the first
    g = torch.Generator().manual_seed(22)
    T, nq, hd = 20000, 16, 128
    q = torch.randn(T, nq * hd, generator=g).to(torch.bfloat16)
    ct, st = lai.rope_table(torch.arange(T, dtype=torch.int32, device="cuda"), T, hd, 1e6)
    qd = q.cuda()
    lai.qk_norm_rope(qd, None, None, None, ct, st, None, nq, 0, hd, 0.0)
    ct_h, st_h = ct.cpu(), st.cpu()
    assert lib().lai_staged_qk_norm_rope_bf16(V(q.data_ptr()), None, None, None, V(ct_h.data_ptr()),
                                              V(st_h.data_ptr()), None, T, T, nq, 0, hd,
                                              0.0) == lai.LAI_OK
    assert np.array_equal(_bits(q), _bits(qd.cpu()))


def test_staged_swiglu_in_place_host():
    g = torch.Generator().manual_seed(23)
    T, I = 2500, 6144  # several staging chunks; out aliases gate_up
    gu = (2 * torch.randn(T, 2 * I, generator=g)).to(torch.bfloat16)
    want = lai.swiglu(gu.cuda(), I).cpu()
    assert lib().lai_staged_swiglu_bf16(V(gu.data_ptr()), V(gu.data_ptr()), T, I) == lai.LAI_OK
    got = gu.view(-1)[: T * I].view(T, I)
    assert np.array_equal(_bits(got), _bits(want))


def test_invalid_arguments_report_without_launching():
    x = np.zeros(8, np.float32)
    lib().qwen_rms_norm(hp(x), hp(x), None, 1, 8, 1e-6)
    assert lib().lai_last_error() == lai.LAI_ERR_INVALID
    lib().qwen_rms_norm_per_head(hp(x), hp(x), 1, 1, 7, 1e-6)  # odd head_dim
    assert lib().lai_last_error() == lai.LAI_ERR_INVALID

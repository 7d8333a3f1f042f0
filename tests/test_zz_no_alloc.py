"""lai_rmsnorm_f32_host_noalloc: host-buffer RMSNorm that allocates nothing.

For callers that cannot let a library call cudaMalloc (their device memory is
owned by their own pool allocator, or a latency-critical loop must not meet the
allocator's device-wide synchronisation), the entry point stages through a fixed
array compiled into the library instead of allocated staging buffers. Its output
is checked against the oracle's RMSNorm (pinned to the reference's golden
vectors) and against the allocating qwen_rms_norm drop-in. This file sorts last
so that a run stopping at the first failure has already run every other test;
it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import lai
import oracle
from conftest import TOL_F32, max_rel_err

pytestmark = pytest.mark.gpu
V = ctypes.c_void_p
SCRATCH_BYTES = 8 << 20  # the entry point's fixed array


def hp(a):
    return V(a.ctypes.data)


def test_noalloc_matches_oracle_and_drop_in_on_two_calls_in_a_row():
    lib = lai.load()
    rng = np.random.default_rng(11)
    # two different problems back to back: the shared array keeps the first call's
    # bytes, so the second call must not depend on anything left behind
    for seq, dim in [(256, 2048), (300, 1000)]:
        x = rng.standard_normal((seq, dim), dtype=np.float32)
        w = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
        ref = oracle.rms_norm(x, w, 1e-6)
        want = np.empty_like(x)
        lib.qwen_rms_norm(hp(want), hp(x), hp(w), seq, dim, 1e-6)
        assert lib.lai_last_error() == lai.LAI_OK
        got = np.full_like(x, np.nan)
        st = lib.lai_rmsnorm_f32_host_noalloc(hp(got), hp(x), hp(w), seq, dim, 1e-6, None)
        assert st == lai.LAI_OK
        assert max_rel_err(got, ref) <= TOL_F32
        assert max_rel_err(got, want) <= TOL_F32


def test_noalloc_in_place_exact_fit_and_size_limit():
    lib = lai.load()
    rng = np.random.default_rng(12)
    x = rng.standard_normal((64, 1024), dtype=np.float32)
    w = np.ones(1024, np.float32)
    ref = oracle.rms_norm(x, w, 1e-5)
    st = lib.lai_rmsnorm_f32_host_noalloc(hp(x), hp(x), hp(w), 64, 1024, 1e-5, None)
    assert st == lai.LAI_OK
    assert max_rel_err(x, ref) <= TOL_F32
    # weights (8 KiB) + rows (1023 x 2048 x 4 B) fill the array exactly
    seq, dim = 1023, 2048
    assert dim * 4 + seq * dim * 4 == SCRATCH_BYTES
    xf = rng.standard_normal((seq, dim), dtype=np.float32)
    wf = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
    got = np.full_like(xf, np.nan)
    st = lib.lai_rmsnorm_f32_host_noalloc(hp(got), hp(xf), hp(wf), seq, dim, 1e-6, None)
    assert st == lai.LAI_OK
    assert max_rel_err(got, oracle.rms_norm(xf, wf, 1e-6)) <= TOL_F32
    # one row more is over the limit and is rejected before anything is queued
    big = np.zeros((seq + 2, dim), np.float32)
    st = lib.lai_rmsnorm_f32_host_noalloc(hp(big), hp(big), hp(wf), seq + 2, dim, 1e-6, None)
    assert st == lai.LAI_ERR_TOOBIG

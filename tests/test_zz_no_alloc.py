"""lai_rmsnorm_f32_host_noalloc: host-buffer RMSNorm that allocates nothing.

For callers that cannot let a library call cudaMalloc (their device memory is
owned by their own pool allocator, or a latency-critical loop must not meet the
allocator's device-wide synchronisation), the entry point stages through a fixed
array compiled into the library instead of allocated staging buffers. This file
sorts last so that a run stopping at the first failure has already run every
other test; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

import lai
from conftest import TOL_F32, max_rel_err

pytestmark = pytest.mark.gpu
V = ctypes.c_void_p


def hp(a):
    return V(a.ctypes.data)


def test_noalloc_matches_the_allocating_drop_in_on_two_calls_in_a_row():
    lib = lai.load()
    rng = np.random.default_rng(11)
    # two different problems back to back: the shared array keeps the first call's
    # bytes, so the second call must not depend on anything left behind
    for seq, dim in [(256, 2048), (300, 1000)]:
        x = rng.standard_normal((seq, dim), dtype=np.float32)
        w = (1 + 0.02 * rng.standard_normal(dim)).astype(np.float32)
        want = np.empty_like(x)
        lib.qwen_rms_norm(hp(want), hp(x), hp(w), seq, dim, 1e-6)
        assert lib.lai_last_error() == lai.LAI_OK
        got = np.full_like(x, np.nan)
        st = lib.lai_rmsnorm_f32_host_noalloc(hp(got), hp(x), hp(w), seq, dim, 1e-6, None)
        assert st == lai.LAI_OK
        assert max_rel_err(got, want) <= TOL_F32


def test_noalloc_in_place_and_size_limit():
    lib = lai.load()
    rng = np.random.default_rng(12)
    x = rng.standard_normal((64, 1024), dtype=np.float32)
    w = np.ones(1024, np.float32)
    want = np.empty_like(x)
    lib.qwen_rms_norm(hp(want), hp(x), hp(w), 64, 1024, 1e-5)
    st = lib.lai_rmsnorm_f32_host_noalloc(hp(x), hp(x), hp(w), 64, 1024, 1e-5, None)
    assert st == lai.LAI_OK
    assert max_rel_err(x, want) <= TOL_F32
    big = np.zeros((1025, 2048), np.float32)  # 8.0 MiB of rows + weights: over the limit
    st = lib.lai_rmsnorm_f32_host_noalloc(hp(big), hp(big), hp(np.ones(2048, np.float32)),
                                          1025, 2048, 1e-6, None)
    assert st == lai.LAI_ERR_TOOBIG

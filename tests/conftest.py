"""Test configuration: markers, import paths, on-demand builds.

`-m "not gpu"` runs on a CPU-only host: the oracle against the golden fixtures,
host-side logic, the gloo multi-process sharding path, and the C ABI's symbol
table. `-m gpu` runs the CUDA kernels through the C ABI against the oracle.
"""
from __future__ import annotations

import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("local-ai-server_b200", "oracle", ""):
    p = os.path.join(REPO, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session", autouse=True)
def _built_libraries():
    """Build the product library and the oracle if they are absent (no-op when built)."""
    import oracle  # noqa: F401
    lib = os.path.join(REPO, "local-ai-server_b200", "liblai_kernels.so")
    if not os.path.exists(lib):
        import build as lai_build  # local-ai-server_b200/build.py
        lai_build.build()
    if not os.path.exists(os.path.join(REPO, "oracle", "_build", "liblai_oracle.so")):
        oracle.build()
    yield


# ---- tolerances (stated once, used by every parity test) ----
TOL_F32 = 1e-5   # max |got - ref| / max(1, |ref|) for FP32 paths
TOL_BF16 = 1e-2  # same measure for BF16 storage paths


def max_rel_err(got, ref) -> float:
    import numpy as np
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if got.size == 0:
        return 0.0
    return float(np.max(np.abs(got - ref) / np.maximum(1.0, np.abs(ref))))


# ---- real memory for argument-check tests ----
# Calls that must be rejected by a host-side check still get pointers into a real,
# zeroed allocation (on the GPU when there is one), large enough for every size those
# tests pass, so that a regressed check would launch on owned memory, not on a made-up
# address.
ARENA_BYTES = 64 << 20
_arena = None


def arena_ptr(offset: int = 0):
    """ctypes pointer `offset` bytes into the shared argument-check arena."""
    import ctypes
    global _arena
    assert 0 <= offset < ARENA_BYTES
    if _arena is None:
        import torch
        if torch.cuda.is_available():
            _arena = torch.zeros(ARENA_BYTES, dtype=torch.uint8, device="cuda")
        else:
            import numpy as np
            _arena = np.zeros(ARENA_BYTES, np.uint8)
    base = _arena.data_ptr() if hasattr(_arena, "data_ptr") else _arena.ctypes.data
    return ctypes.c_void_p(base + offset)

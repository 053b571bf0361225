"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU.

The oracle (``oracle/``) is the checker: a C restatement of the reference
crate's CPU arms, pinned by the reference's golden vectors.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


def _ensure_built():
    import oracle as O  # noqa: F401  (builds liboracle.so on first use)

    O.lib()
    lib = os.path.join(ROOT, "sparsl_b200", "libsparsl_cuda.so")
    if not os.path.exists(lib):
        from sparsl_b200 import build

        build.build()


_ensure_built()


@pytest.fixture(scope="session")
def O():
    import oracle

    return oracle


@pytest.fixture(scope="session")
def cuda_device():
    from sparsl_b200 import Backend, Device

    return Device.try_new(Backend.Cuda)


# Shapes from the reference's differential suite (tests/common/mod.rs:459-479).
SHAPES = [
    (0, 0, 0), (0, 8, 4), (1, 1, 0), (1, 1, 1), (1, 64, 64), (7, 7, 3), (31, 31, 5), (32, 32, 5), (33, 33, 5),
    (63, 64, 8), (64, 64, 8), (65, 64, 8), (255, 128, 16), (256, 128, 16), (257, 128, 16), (512, 512, 1),
    (1000, 1000, 64), (2048, 512, 3),
]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def assert_bits_equal(got, want, context=""):
    """Bit-for-bit equality; NaNs compare by class (the reference's comparators
    treat NaN payloads as free, tests/common/mod.rs:158-172)."""
    g = np.asarray(got, dtype=np.float32)
    w = np.asarray(want, dtype=np.float32)
    assert g.shape == w.shape, f"{context}: shape {g.shape} vs {w.shape}"
    both_nan = np.isnan(g) & np.isnan(w)
    diff = (bits(g) != bits(w)) & ~both_nan
    if diff.any():
        i = int(np.flatnonzero(diff)[0])
        raise AssertionError(f"{context}: {int(diff.sum())} elements differ; first at {i}: got {g.flat[i]!r} "
                             f"(0x{bits(g).flat[i]:08x}) want {w.flat[i]!r} (0x{bits(w).flat[i]:08x})")

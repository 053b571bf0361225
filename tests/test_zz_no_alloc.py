"""The allocation-free scan entry point, for callers that cannot allocate.

A host whose allocator already owns all of the GPU's memory (or that only lends
this library buffers it holds) cannot let the library call cudaMalloc.  For it,
sparsl_dev_assoc_scan_noalloc keeps the scan's scratch in a static device array
and takes only caller-owned input and output buffers.  This file checks it
through the C ABI against the ordinary scan entry point, bit for bit, on two
calls in a row (the array keeps the previous call's contents, so the second
call proves the clearing), and checks that sizes past its maximum are refused.

It is collected last on purpose (tests/test_zz_*), so a run that stops at the
first failure has already run everything else; it also passes on its own.
"""
import ctypes

import numpy as np
import pytest

import sparsl_b200 as S
from sparsl_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_MAPS = 1 << 22


def _maps(n, seed):
    r = np.random.default_rng(seed)
    return np.stack([r.uniform(0.9, 1.0, n), r.standard_normal(n)], 1).astype(np.float32)


def test_allocation_free_scan_matches_the_ordinary_entry_point():
    import torch

    dev = S.Device.try_new(S.Backend.Cuda, 0)
    L = _lib.load()
    stream = torch.cuda.Stream()
    # Two calls in a row with different sizes and data; the second call must
    # not see anything the first left in the shared static scratch.
    for n, seed in ((1_000_003, 11), (MAX_MAPS, 12)):
        xs = _maps(n, seed)
        with torch.cuda.stream(stream):
            d_in = torch.from_numpy(xs).cuda()
            d_got = torch.full_like(d_in, float("nan"))
            d_want = torch.full_like(d_in, float("nan"))
        stream.synchronize()
        rc = L.sparsl_dev_assoc_scan_noalloc(0, d_in.data_ptr(), n, d_got.data_ptr(), stream.cuda_stream, 60000)
        assert rc == 0, _lib.last_error()
        rc = L.sparsl_dev_assoc_scan_device(dev.handle, d_in.data_ptr(), n, d_want.data_ptr(), stream.cuda_stream)
        assert rc == 0, _lib.last_error()
        stream.synchronize()
        got = d_got.cpu().numpy().view(np.uint32)
        want = d_want.cpu().numpy().view(np.uint32)
        assert np.array_equal(got, want), f"n={n}: {int((got != want).sum())} words differ"


def test_allocation_free_scan_refuses_sizes_past_its_maximum():
    L = _lib.load()
    rc = L.sparsl_dev_assoc_scan_noalloc(0, ctypes.c_void_p(16), MAX_MAPS + 1, ctypes.c_void_p(16), None, 1000)
    assert rc == _lib.SPARSL_ERR_LENGTH
    assert "maximum" in _lib.last_error()
    assert L.sparsl_dev_assoc_scan_noalloc(0, None, 0, None, None, 1000) == 0  # empty is a no-op


def test_allocation_free_scan_follows_the_quarantine_rules():
    """A call whose bounded wait runs out quarantines the backend like every
    other entry point: later calls are refused until the caller's stream has
    drained and sparsl_device_reset has cleared the quarantine.  The slow
    work is a bounded busy kernel queued ahead of the scan on the caller's
    stream."""
    import time

    import torch

    L = _lib.load()
    dev = S.Device.try_new(S.Backend.Cuda, 0)
    n = 100_000
    xs = _maps(n, 13)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        d_in = torch.from_numpy(xs).cuda()
        d_got = torch.empty_like(d_in)
        d_want = torch.empty_like(d_in)
    stream.synchronize()
    try:
        with torch.cuda.stream(stream):
            torch.cuda._sleep(1_000_000_000)  # ~0.5 s, bounded
        rc = L.sparsl_dev_assoc_scan_noalloc(0, d_in.data_ptr(), n, d_got.data_ptr(), stream.cuda_stream, 20)
        assert rc == _lib.SPARSL_ERR_EXECUTION, _lib.last_error()
        assert "quarantined" in _lib.last_error()
        assert L.sparsl_quarantined() == 1
        rc = L.sparsl_dev_assoc_scan_noalloc(0, d_in.data_ptr(), n, d_got.data_ptr(), stream.cuda_stream, 60000)
        assert rc == _lib.SPARSL_ERR_BACKEND
        stream.synchronize()  # the timed-out scan completes behind the busy kernel
    finally:
        t0 = time.time()
        while L.sparsl_device_reset() != 0:
            assert time.time() - t0 < 30, _lib.last_error()
            time.sleep(0.02)
    assert L.sparsl_quarantined() == 0
    rc = L.sparsl_dev_assoc_scan_noalloc(0, d_in.data_ptr(), n, d_got.data_ptr(), stream.cuda_stream, 0)
    assert rc == 0, _lib.last_error()
    rc = L.sparsl_dev_assoc_scan_device(dev.handle, d_in.data_ptr(), n, d_want.data_ptr(), stream.cuda_stream)
    assert rc == 0, _lib.last_error()
    stream.synchronize()
    assert np.array_equal(d_got.cpu().numpy().view(np.uint32), d_want.cpu().numpy().view(np.uint32))


def test_allocation_free_scan_checks_the_caller_buffers():
    """Buffers must be device memory of the named GPU and hold n maps inside
    their allocation; a short buffer is refused before anything runs."""
    import torch

    L = _lib.load()
    short = torch.zeros((1000, 2), dtype=torch.float32, device="cuda")
    out = torch.zeros((4096, 2), dtype=torch.float32, device="cuda")
    # 2^21 maps (16 MiB) cannot fit the small allocation behind `short`.
    rc = L.sparsl_dev_assoc_scan_noalloc(0, short.data_ptr(), 1 << 21, out.data_ptr(), None, 1000)
    assert rc == _lib.SPARSL_ERR_INVALID, _lib.last_error()
    host = np.zeros((16, 2), np.float32)
    rc = L.sparsl_dev_assoc_scan_noalloc(0, host.ctypes.data, 16, out.data_ptr(), None, 1000)
    assert rc == _lib.SPARSL_ERR_INVALID, _lib.last_error()
    assert L.sparsl_quarantined() == 0

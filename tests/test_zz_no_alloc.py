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

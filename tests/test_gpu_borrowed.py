"""sparsl_op_prepare_device_borrowed: an f32 operator that uses the caller's
device CSR arrays in place instead of copying them.

It must give the same products as sparsl_op_prepare_device on the same arrays
(and so the oracle's, bit for bit), on the generic path and on the TMA path
for equal rows; it must read the caller's memory (a weight changed in place
shows in the next product), write set_weights into it, refuse arrays that do
not meet the alignment and slack that the operator's own arrays guarantee
every kernel, and leave the arrays to the caller when it is destroyed.
"""
import ctypes
import gc

import numpy as np
import pytest
import torch

from conftest import assert_bits_equal

import sparsl_b200 as S
from sparsl_b200 import _lib

pytestmark = pytest.mark.gpu

PARAMS = S.LifParams.new(0.9, 0.0, 0.1)


def _lent(a, dtype):
    """A CUDA tensor holding `a`, cut from a larger one so that 256 bytes of
    the same allocation follow it (the storage start is 256-byte aligned)."""
    a = np.ascontiguousarray(a)
    t = torch.empty(a.size + 64, dtype=dtype, device="cuda")
    t[: a.size].copy_(torch.from_numpy(a.view(np.int32 if dtype == torch.int32 else np.float32)))
    return t[: a.size]


def _csr(O, kind, seed):
    if kind == "uniform":  # equal rows of 64: the TMA-streamed path
        rng = O.Rng(seed)
        return O.random_csr(20_000, 20_000, 64, rng), rng
    r = np.random.default_rng(seed)
    nrows, ncols = 6000, 7000
    lens = np.minimum(r.zipf(1.5, nrows), 3000)
    lens[::53] = 0
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(ncols, k, replace=False)) for k in lens]).astype(np.uint32)
    return O.Csr(rp.astype(np.uint32), col, ncols), O.Rng(seed)


@pytest.mark.parametrize("kind", ["uniform", "power_law"])
def test_borrowed_products_match_copying_prepare(O, cuda_device, kind):
    csr, rng = _csr(O, kind, 0xB0 + len(kind))
    nrows, ncols = csr.row_ptr.size - 1, csr.ncols
    w = O.random_vec(csr.nnz, 1.0, rng)
    rp_t, col_t, w_t = _lent(csr.row_ptr, torch.int32), _lent(csr.col, torch.int32), _lent(w, torch.float32)
    lent = cuda_device.prepare_device_borrowed(rp_t, col_t, ncols, w_t, transpose=True)
    owned = cuda_device.prepare_device(rp_t, col_t, ncols, w_t, transpose=True)
    assert lent.shape() == owned.shape() and lent.has_transpose()
    x = O.random_vec(ncols, 1.0, rng)
    xt = O.random_vec(nrows, 1.0, rng)
    y0 = O.random_vec(nrows, 1.0, rng)
    xs = (np.random.default_rng(5).random(ncols) < 0.3).astype(np.uint8)
    packed = O.pack_spikes(xs)
    csc = O.csc_from_csr(csr, ncols)
    for op in (lent, owned):
        got = y0.copy()
        op.spmv(x, got)
        assert_bits_equal(got, O.spmv(csr, w, x, y0.copy()), f"spmv {kind}")
        gt = np.zeros(ncols, np.float32)
        op.spmv_t(xt, gt)
        assert_bits_equal(gt, O.spmv_t(csc, w, xt, np.zeros(ncols, np.float32)), f"spmv_t {kind}")
        got = y0.copy()
        op.spmv_spikes(packed, got)
        assert_bits_equal(got, O.spmv_spikes(csr, w, packed, y0.copy()), f"spikes {kind}")
    if nrows == ncols:  # fused spike LIF on the square operator
        v = O.random_vec(nrows, 1.0, rng)
        th = np.ones(nrows, np.float32)
        res = []
        for op in (lent, owned):
            vv, tt, sp = v.copy(), th.copy(), np.zeros(nrows, np.uint8)
            op.fused_spmv_spikes_lif(packed, vv, tt, sp, PARAMS)
            res.append((vv, tt, sp))
        assert_bits_equal(res[0][0], res[1][0], "fused v")
        assert np.array_equal(res[0][2], res[1][2])


def test_borrowed_arrays_are_read_in_place_and_set_weights_writes_them(O, cuda_device):
    csr, rng = _csr(O, "uniform", 0xB1)
    ncols = csr.ncols
    w = O.random_vec(csr.nnz, 1.0, rng)
    rp_t, col_t, w_t = _lent(csr.row_ptr, torch.int32), _lent(csr.col, torch.int32), _lent(w, torch.float32)
    lent = cuda_device.prepare_device_borrowed(rp_t, col_t, ncols, w_t)
    owned = cuda_device.prepare_device(rp_t, col_t, ncols, w_t)
    x = O.random_vec(ncols, 1.0, rng)
    y0 = np.zeros(csr.row_ptr.size - 1, np.float32)
    w_t.mul_(2.0)  # doubling is exact: the borrowed operator now folds 2w
    torch.cuda.synchronize()
    got = y0.copy()
    lent.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, w * np.float32(2), x, y0.copy()), "borrowed weights read in place")
    got = y0.copy()
    owned.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, w, x, y0.copy()), "the copying operator kept its own weights")
    w3 = O.random_vec(csr.nnz, 3.0, rng)
    lent.set_weights(w3)
    torch.cuda.synchronize()
    assert_bits_equal(w_t.cpu().numpy(), w3, "set_weights writes into the borrowed array")
    got = y0.copy()
    lent.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, w3, x, y0.copy()))
    # Destroying the operator leaves the arrays to the caller.
    del lent
    gc.collect()
    torch.cuda.synchronize()
    assert np.array_equal(col_t.cpu().numpy().view(np.uint32), csr.col)
    w_t.add_(1.0)
    torch.cuda.synchronize()


def test_borrowed_refuses_unaligned_short_and_host_arrays(O, cuda_device):
    csr, rng = _csr(O, "uniform", 0xB2)
    ncols = csr.ncols
    w = O.random_vec(csr.nnz, 1.0, rng)
    rp_t, col_t, w_t = _lent(csr.row_ptr, torch.int32), _lent(csr.col, torch.int32), _lent(w, torch.float32)
    lib = _lib.load()
    sh = _lib.Shape()
    h = ctypes.c_void_p()

    def call(rp, rp_len, col, col_len, wp, w_len):
        h.value = None
        return lib.sparsl_op_prepare_device_borrowed(cuda_device.handle, rp, rp_len, col, col_len, ncols, ncols, wp,
                                                     w_len, 0, ctypes.byref(sh), ctypes.byref(h))

    n_rp, nnz = rp_t.numel(), col_t.numel()
    # a start off the 256-byte boundary
    shifted = torch.empty(nnz + 128, dtype=torch.int32, device="cuda")
    shifted[1:nnz + 1].copy_(col_t)
    rc = call(rp_t.data_ptr(), n_rp, shifted[1:].data_ptr(), nnz, w_t.data_ptr(), nnz)
    assert rc == _lib.SPARSL_ERR_INVALID and not h.value and "256-byte boundary" in _lib.last_error()
    # a length that runs past the allocation
    rc = call(rp_t.data_ptr(), n_rp, col_t.data_ptr(), 1 << 40, w_t.data_ptr(), nnz)
    assert rc == _lib.SPARSL_ERR_INVALID and not h.value
    # host memory
    host_w = np.zeros(nnz + 64, np.float32)
    rc = call(rp_t.data_ptr(), n_rp, col_t.data_ptr(), nnz, host_w.ctypes.data, nnz)
    assert rc == _lib.SPARSL_ERR_INVALID and not h.value and _lib.last_reason() == "not device memory"
    # and the same arrays, lent properly, make an operator
    op = cuda_device.prepare_device_borrowed(rp_t, col_t, ncols, w_t)
    assert op.shape().nnz() == nnz

"""sparsl_op_prepare_device: an operator built from arrays already in HBM.

It must be indistinguishable from sparsl_op_prepare on the same values: the
same gate (validate_csr, src/backend/mod.rs:2116-2182) with the same first
failure and payload, the same quantised weights (src/half.rs:49-219), and so
bit-identical products.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import SHAPES, assert_bits_equal

import sparsl_b200 as S
from sparsl_b200 import _lib

pytestmark = pytest.mark.gpu

PRECISIONS = [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16]


def _dev(a, dtype=torch.int32):
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32 if dtype == torch.int32 else np.float32)).cuda()


def _both(dev, rp, col, csr_ncols, ncols, w, precision=S.WeightPrecision.F32, transpose=False):
    """(host result, device result): an operator or the SparsePlanError raised."""
    out = []
    rp = np.asarray(rp, np.uint32)
    col = np.asarray(col, np.uint32)
    w = np.asarray(w, np.float32)
    try:
        out.append(S.SparseOp._prepare(dev, S.Csr(rp, col, csr_ncols), ncols, w, transpose, precision))
    except S.SparsePlanError as e:
        out.append(e)
    try:
        out.append(dev.prepare_device(_dev(rp), _dev(col), ncols, _dev(w, torch.float32), precision, transpose,
                                      csr_ncols=csr_ncols))
    except S.SparsePlanError as e:
        out.append(e)
    return out


def _same_error(h, d):
    assert isinstance(h, S.SparsePlanError) and isinstance(d, S.SparsePlanError), (h, d)
    assert h.kind == d.kind and h.fields == d.fields and str(h) == str(d), (h.kind, h.fields, d.kind, d.fields)
    return h.kind


@pytest.mark.parametrize(
    "case",
    [
        # (row_ptr, col, csr_ncols, ncols, weights_len, expected kind)
        ([], [], 4, 4, 0, "EmptyRowPtr"),
        ([3, 4], [0, 1, 2, 3], 4, 4, 4, "NonZeroStart"),
        ([0, 2, 1, 4], [0, 1, 2, 3], 4, 4, 4, "NotMonotonic"),
        ([0, 2, 1, 0, 4], [0, 1, 2, 3], 4, 4, 4, "NotMonotonic"),
        ([0, 2, 5], [0, 1, 2, 3], 4, 4, 4, "NnzMismatch"),
        ([0, 2, 4], [0, 1, 2, 3], 5, 4, 4, "NcolsMismatch"),
        ([0, 2, 4], [0, 9, 2, 7], 4, 4, 4, "ColumnOutOfRange"),
        ([0, 2, 4, 6], [0, 1, 3, 2, 1, 0], 4, 4, 6, "RowUnsorted"),
        ([0, 3, 6], [0, 0, 1, 3, 3, 3], 4, 4, 5, "WeightsLen"),
        ([0, 2, 4], [0, 1, 2, 3], 2**32 + 5, 2**32 + 5, 4, "TooLarge"),
        # Order: an unsorted row and an out-of-range column -> the column check first.
        ([0, 2, 4], [1, 0, 2, 9], 4, 4, 4, "ColumnOutOfRange"),
    ],
)
def test_gate_matches_host_prepare(cuda_device, case):
    rp, col, csr_ncols, ncols, wlen, kind = case
    h, d = _both(cuda_device, rp, col, csr_ncols, ncols, np.ones(wlen, np.float32))
    assert _same_error(h, d) == kind


def test_first_failure_over_many_blocks(O, cuda_device):
    """Failures spread over a large CSR: the lowest edge / row wins on the GPU
    as in the reference's sequential scan."""
    rng = O.Rng(0x9A7E)
    nrows, ncols, deg = 200_000, 50_000, 16
    csr = O.random_csr(nrows, ncols, deg, rng)
    w = O.random_vec(csr.nnz, 1.0, rng)
    col = csr.col.copy()
    r = np.random.default_rng(3)
    bad = np.sort(r.choice(csr.nnz, 40, replace=False))
    col[bad] = ncols + np.arange(40, dtype=np.uint32)
    h, d = _both(cuda_device, csr.row_ptr, col, ncols, ncols, w)
    assert _same_error(h, d) == "ColumnOutOfRange"
    assert d.fields["edge"] == int(bad[0]) and d.fields["col"] == ncols
    # Unsorted rows: swap the first two entries of several rows with distinct columns.
    col = csr.col.copy()
    rows = [r_ for r_ in range(1000, nrows, 7919) if csr.row_ptr[r_ + 1] - csr.row_ptr[r_] >= 2][:25]
    for row in rows:
        b = csr.row_ptr[row]
        seg = col[b:csr.row_ptr[row + 1]]
        k = int(np.argmax(seg[1:] > seg[:-1])) if np.any(seg[1:] > seg[:-1]) else None
        if k is not None:
            seg[k], seg[k + 1] = seg[k + 1], seg[k]
    h, d = _both(cuda_device, csr.row_ptr, col, ncols, ncols, w)
    assert _same_error(h, d) == "RowUnsorted" and d.fields["row"] == rows[0]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("precision", PRECISIONS)
def test_products_bit_identical(O, cuda_device, shape, precision):
    nrows, ncols, deg = shape
    rng = O.Rng(0x0DE7 + nrows + 3 * ncols)
    csr = O.random_csr(nrows, ncols, deg, rng)
    w = O.random_vec(csr.nnz, 1.0, rng)
    x = O.random_vec(ncols, 1.0, rng)
    xt = O.random_vec(nrows, 1.0, rng)
    y0 = O.random_vec(nrows, 1.0, rng)
    h, d = _both(cuda_device, csr.row_ptr, csr.col, ncols, ncols, w, precision, transpose=True)
    assert d.weight_precision() is precision and d.has_transpose()
    assert d.shape() == h.shape()
    wq = O.quantise(int(precision), w)
    csc = O.csc_from_csr(csr, ncols)
    for op in (h, d):
        got = y0.copy()
        op.spmv(x, got)
        assert_bits_equal(got, O.spmv(csr, wq, x, y0.copy()), f"spmv {shape}")
        gt = np.zeros(ncols, np.float32)
        op.spmv_t(xt, gt)
        assert_bits_equal(gt, O.spmv_t(csc, wq, xt, np.zeros(ncols, np.float32)), f"spmv_t {shape}")
        xs = (np.random.default_rng(nrows).random(ncols) < 0.3).astype(np.uint8)
        got = y0.copy()
        op.spmv_spikes(O.pack_spikes(xs), got)
        assert_bits_equal(got, O.spmv_spikes(csr, wq, O.pack_spikes(xs), y0.copy()), f"spikes {shape}")


@pytest.mark.parametrize("precision", [S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_device_encoder_matches_host_encoder(O, cuda_device, precision):
    """A diagonal operator reads each quantised weight back as y_i = 0 + w_i * 1.
    Inputs: every rounding boundary of the narrow format (each representable
    value and the f32 patterns either side of each midpoint), the specials,
    and 2^20 random patterns."""
    if precision is S.WeightPrecision.F16:
        narrow = np.arange(0x10000, dtype=np.uint32)
        narrow = narrow[((narrow >> 10) & 0x1F) != 0x1F].astype(np.uint16)
        wide = narrow.view(np.float16).astype(np.float32)
    else:
        narrow = np.arange(0x10000, dtype=np.uint32)
        wide = (narrow << 16).view(np.float32)
        wide = wide[np.isfinite(wide)]
    wide = np.sort(np.unique(wide.astype(np.float64))).astype(np.float32)
    mid = ((wide[:-1].astype(np.float64) + wide[1:].astype(np.float64)) / 2).astype(np.float32)
    mb = mid.view(np.uint32)
    pats = [wide.view(np.uint32), mb, mb - 1, mb + 1,
            np.array([0x7F800000, 0xFF800000, 0x7FC00000, 0xFFC00001, 0x7F7FFFFF, 0xFF7FFFFF, 0x00000001,
                      0x80000001, 0x477FF000, 0x477FEFFF, 0x47800000], np.uint32),
            np.random.default_rng(11).integers(0, 2**32, 2**20, dtype=np.uint64).astype(np.uint32)]
    w = np.concatenate(pats).view(np.float32)
    n = w.size
    rp = np.arange(n + 1, dtype=np.uint32)
    col = np.arange(n, dtype=np.uint32)
    h, d = _both(cuda_device, rp, col, n, n, w, precision)
    ones = np.ones(n, np.float32)
    yh = np.zeros(n, np.float32)
    yd = np.zeros(n, np.float32)
    h.spmv(ones, yh)
    d.spmv(ones, yd)
    assert_bits_equal(yd, yh, "device vs host encoder")
    want = O.quantise(int(precision), w)
    assert_bits_equal(yd, np.where(want == 0, np.float32(0), want).astype(np.float32), "against the oracle codec")


def test_rejects_host_and_short_arrays(cuda_device):
    """Arguments that are not this GPU's memory, or claim more elements than
    their allocation holds, are refused before any kernel reads them."""
    rp = torch.tensor([0, 2, 4], dtype=torch.int32, device="cuda")
    col = torch.tensor([0, 1, 2, 3], dtype=torch.int32, device="cuda")
    w = torch.ones(4, dtype=torch.float32, device="cuda")
    lib = _lib.load()
    sh = _lib.Shape()
    h = ctypes.c_void_p()
    host_col = np.array([0, 1, 2, 3], np.uint32)
    rc = lib.sparsl_op_prepare_device(cuda_device.handle, rp.data_ptr(), 3, host_col.ctypes.data, 4, 4, 4,
                                      w.data_ptr(), 4, 0, 0, ctypes.byref(sh), ctypes.byref(h))
    assert rc == _lib.SPARSL_ERR_INVALID and not h.value and "not device memory" in _lib.last_reason()
    rc = lib.sparsl_op_prepare_device(cuda_device.handle, rp.data_ptr(), 3, col.data_ptr(), 1 << 40, 4, 4,
                                      w.data_ptr(), 4, 0, 0, ctypes.byref(sh), ctypes.byref(h))
    assert rc == _lib.SPARSL_ERR_INVALID and not h.value and "too short" in _lib.last_reason()
    rc = lib.sparsl_op_prepare_device(cuda_device.handle, 0, 3, col.data_ptr(), 4, 4, 4, w.data_ptr(), 4, 0, 0,
                                      ctypes.byref(sh), ctypes.byref(h))
    assert rc == _lib.SPARSL_ERR_INVALID and not h.value
    # The arrays stay the caller's: the operator holds copies.
    op = cuda_device.prepare_device(rp, col, 4, w)
    rp.fill_(7)
    col.fill_(9)
    w.fill_(-1.0)
    y = np.zeros(2, np.float32)
    op.spmv(np.array([1, 2, 3, 4], np.float32), y)
    assert y.tolist() == [3.0, 7.0]

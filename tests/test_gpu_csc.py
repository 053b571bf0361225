"""The stable reverse index built on the GPU against the oracle's
Csc::from_csr_slices (src/sparse.rs:361-427): identical col_ptr, row and
edge_idx arrays, including every radix pass count (ncols up to 2^25),
duplicate columns within a row, empty rows and columns, and hub columns."""
import numpy as np
import pytest
import torch

from conftest import SHAPES

import sparsl_b200 as S

pytestmark = pytest.mark.gpu


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def _gpu_csc(dev, rp, col, ncols):
    nnz = len(col)
    cp = torch.full((ncols + 1,), -1, dtype=torch.int32, device="cuda")
    row = torch.full((max(nnz, 1),), -1, dtype=torch.int32, device="cuda")
    eidx = torch.full((max(nnz, 1),), -1, dtype=torch.int32, device="cuda")
    dev.csc_from_csr_device(_t(rp), _t(col), ncols, cp, row, eidx)
    u = lambda t, n: t.cpu().numpy().view(np.uint32)[:n]  # noqa: E731
    return u(cp, ncols + 1), u(row, nnz), u(eidx, nnz)


def _check(O, dev, rp, col, ncols):
    csr = O.Csr(rp, col, ncols)
    want = O.csc_from_csr(csr, ncols)
    got = _gpu_csc(dev, csr.row_ptr, csr.col, ncols)
    for name, g, w in zip(("col_ptr", "row", "edge_idx"), got, want):
        assert np.array_equal(g, w), f"{name} differs at {np.flatnonzero(g != w)[:5]}"


@pytest.mark.parametrize("shape", SHAPES)
def test_matches_oracle_on_reference_shapes(O, cuda_device, shape):
    nrows, ncols, deg = shape
    csr = O.random_csr(nrows, ncols, deg, O.Rng(0xC5C + nrows * 31 + ncols))
    _check(O, cuda_device, csr.row_ptr, csr.col, ncols)


def _rows_from_lists(rows):
    rp = np.zeros(len(rows) + 1, np.uint64)
    rp[1:] = np.cumsum([len(r) for r in rows])
    col = np.concatenate([np.asarray(r, np.uint32) for r in rows]) if rows else np.zeros(0, np.uint32)
    return rp.astype(np.uint32), col.astype(np.uint32)


# ncols chosen at every radix pass boundary: 1, 2, 3 and 4 passes of 8 bits.
@pytest.mark.parametrize("ncols", [1, 2, 256, 257, 65536, 65537, 1 << 24, (1 << 24) + 3, 20_000_000])
def test_every_pass_count(O, cuda_device, ncols):
    r = np.random.default_rng(ncols)
    nrows = 5000
    rows = []
    for i in range(nrows):
        k = int(r.integers(0, 40))
        if i % 97 == 0:
            k = 0  # empty rows
        rows.append(np.sort(r.integers(0, ncols, k)))  # duplicates allowed (non-decreasing)
    rp, col = _rows_from_lists(rows)
    _check(O, cuda_device, rp, col, ncols)


def test_many_tiles_hub_and_duplicates(O, cuda_device):
    """3.2M edges (hundreds of radix tiles, tens of scan tiles); one hub
    column that every row touches, repeated columns, empty columns."""
    r = np.random.default_rng(7)
    nrows, ncols = 40_000, 300_000
    deg = r.integers(0, 160, nrows)
    rows = []
    for i in range(nrows):
        c = r.integers(0, ncols, int(deg[i]))
        c = np.concatenate([c, [12345, 12345]])  # hub column, twice per row
        c[c % 1000 == 999] = 998  # columns ending in 999 stay empty
        rows.append(np.sort(c))
    rp, col = _rows_from_lists(rows)
    assert len(col) > 3_000_000
    _check(O, cuda_device, rp, col, ncols)


def test_no_edges(O, cuda_device):
    _check(O, cuda_device, np.zeros(6, np.uint32), np.zeros(0, np.uint32), 9)
    _check(O, cuda_device, np.zeros(1, np.uint32), np.zeros(0, np.uint32), 0)


def test_gate_errors(cuda_device):
    with pytest.raises(S.SparsePlanError) as ei:
        _gpu_csc(cuda_device, np.array([0, 2, 4], np.uint32), np.array([0, 5, 1, 2], np.uint32), 4)
    assert ei.value.kind == "ColumnOutOfRange" and ei.value.fields["edge"] == 1
    with pytest.raises(S.SparsePlanError) as ei:
        _gpu_csc(cuda_device, np.array([0, 2, 4], np.uint32), np.array([0, 1, 3, 2], np.uint32), 4)
    assert ei.value.kind == "RowUnsorted" and ei.value.fields["row"] == 1 and ei.value.fields["edge"] == 3

"""Dense-x SpMV with x in shared-memory panels (uniform rows, x of at most
4 x 55,296 floats) against the oracle and the generic row fold, bit for bit.

Covers one to four panels, several row waves, ragged last tiles, columns at
and around the panel edges (rows that stop in one panel and resume in the
next, rows that skip whole panels, duplicate columns), the three weight
precisions, new weights after prepare, an x that is not 16-byte aligned, and
the widest x that still takes the TMA stream instead.  The transpose product
over the same panels (built from the sliced-ELL reverse index, x indexed by
row) is checked the same way against the oracle and the reverse-index fold,
and so is the ordered copy that skewed operators use for dense-x SpMV."""
import numpy as np
import pytest

from conftest import assert_bits_equal

import sparsl_b200 as S

pytestmark = pytest.mark.gpu

PANELS = 16  # SPARSL_LAYOUT_X_PANELS
ELL = 1      # SPARSL_LAYOUT_ELL
MAX_PANEL = 55296


def _uniform(O, nrows, ncols, L, seed):
    r = np.random.default_rng(seed)
    col = np.sort(r.integers(0, ncols, size=(nrows, L), dtype=np.uint32), axis=1).reshape(-1)
    rp = (np.arange(nrows + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = r.uniform(-1, 1, nrows * L).astype(np.float32)
    return O.Csr(rp, col, ncols), w


def _check(O, dev, csr, w, precision, seed, panels=True):
    wq = O.quantise(int(precision), w)
    op = dev.prepare_with(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w, precision)
    assert bool(op.layouts() & PANELS) == panels
    ref = dev.prepare_with(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w, precision)
    ref.force_plain_row_fold()
    assert not ref.layouts() & (PANELS | ELL)
    r = np.random.default_rng(seed)
    x = r.uniform(-1, 1, csr.ncols).astype(np.float32)
    nrows = len(csr.row_ptr) - 1
    y0 = r.uniform(-1, 1, nrows).astype(np.float32)
    got, gen = y0.copy(), y0.copy()
    op.spmv(x, got)
    ref.spmv(x, gen)
    want = O.spmv(csr, wq, x, y0.copy())
    assert_bits_equal(got, want, "panel spmv vs oracle")
    assert_bits_equal(gen, want, "generic row fold vs oracle")
    return op, x, y0


@pytest.mark.parametrize("nrows,ncols,L", [
    (1, 64, 8),             # one row, one panel
    (33, 1000, 40),         # ragged last tile
    (5000, 60000, 64),      # two panels (the config-1 geometry, smaller)
    (3000, 150000, 32),     # three panels
    (2000, 4 * MAX_PANEL, 16),  # four full panels, the widest x
    (130_000, 2000, 8),     # two waves of tiles (more tiles than warps in flight)
    (777, 110593, 3),       # odd panel width rounding, short rows
])
@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_panel_spmv_bit_exact(O, cuda_device, nrows, ncols, L, precision):
    csr, w = _uniform(O, nrows, ncols, L, nrows * 13 + L)
    _check(O, cuda_device, csr, w, precision, L)


def test_panel_edges_and_skipped_panels(O, cuda_device):
    """Rows whose entries sit on the panel edges, repeat a column, start in a
    later panel, or end before the last one."""
    ncols = 3 * MAX_PANEL  # three panels of 55,296
    wdt = MAX_PANEL
    edges = [0, 1, wdt - 2, wdt - 1, wdt, wdt + 1, 2 * wdt - 1, 2 * wdt, 2 * wdt + 1, ncols - 2, ncols - 1]
    r = np.random.default_rng(5)
    L = 12
    rows = []
    for i in range(700):
        kind = i % 7
        if kind == 0:
            c = r.choice(edges, L)
        elif kind == 1:
            c = np.full(L, edges[i % len(edges)])                   # one column, repeated
        elif kind == 2:
            c = r.integers(2 * wdt, ncols, L)                        # third panel only
        elif kind == 3:
            c = r.integers(0, wdt, L)                                # first panel only
        elif kind == 4:
            c = np.concatenate([r.integers(0, 10, L // 2), r.integers(ncols - 10, ncols, L - L // 2)])
        elif kind == 5:
            c = r.integers(wdt, 2 * wdt, L)                          # middle panel only
        else:
            c = r.integers(0, ncols, L)
        rows.append(np.sort(c).astype(np.uint32))
    col = np.concatenate(rows)
    rp = (np.arange(len(rows) + 1, dtype=np.uint64) * L).astype(np.uint32)
    w = r.standard_normal(col.size).astype(np.float32)
    _check(O, cuda_device, O.Csr(rp, col, ncols), w, S.WeightPrecision.F32, 6)


def test_panel_single_entry_rows(O, cuda_device):
    csr, w = _uniform(O, 4097, 90000, 1, 3)
    _check(O, cuda_device, csr, w, S.WeightPrecision.F16, 4)


@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.Bf16])
def test_panel_copy_follows_new_weights(O, cuda_device, precision):
    csr, w = _uniform(O, 2000, 70000, 24, 11)
    op, x, y0 = _check(O, cuda_device, csr, w, precision, 12)
    w2 = np.random.default_rng(13).uniform(-2, 2, w.size).astype(np.float32)
    op.set_weights(w2)
    got = y0.copy()
    op.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, O.quantise(int(precision), w2), x, y0.copy()), "spmv after set_weights")


def test_panel_unaligned_bound_x(O, cuda_device):
    """A bound x that starts 4 bytes past a 16-byte boundary: the panel load
    takes its 4-byte path."""
    import torch

    csr, w = _uniform(O, 3000, 65000, 16, 21)
    op = cuda_device.prepare(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w)
    assert op.layouts() & PANELS
    r = np.random.default_rng(22)
    x = r.uniform(-1, 1, csr.ncols).astype(np.float32)
    xt = torch.zeros(csr.ncols + 4, dtype=torch.float32, device="cuda")
    xt[1:1 + csr.ncols] = torch.from_numpy(x).cuda()
    xv = xt[1:]
    assert xv.data_ptr() % 16 == 4
    op.bind_cuda_x(xv)
    y0 = r.uniform(-1, 1, 3000).astype(np.float32)
    got = y0.copy()
    op.spmv(x, got)  # the host slice is ignored while x is bound
    torch.cuda.synchronize()
    op.unbind_cuda_x()
    assert_bits_equal(got, O.spmv(csr, w, x, y0.copy()), "unaligned bound x")


def test_widest_x_past_the_panels_takes_the_stream(O, cuda_device):
    csr, w = _uniform(O, 1500, 4 * MAX_PANEL + 1, 16, 31)
    op, _, _ = _check(O, cuda_device, csr, w, S.WeightPrecision.F32, 32, panels=False)
    assert op.layouts() & ELL


T_PANELS = 32  # SPARSL_LAYOUT_T_X_PANELS
SLICED = 4     # SPARSL_LAYOUT_SLICED_REVERSE


def _check_t(O, dev, csr, w, precision, seed, panels=True):
    """spmv_t through the transpose x panels against the oracle and against
    the sliced-ELL fold of the same operator."""
    wq = O.quantise(int(precision), w)
    nrows = len(csr.row_ptr) - 1
    op = dev.prepare_with_transpose_precision(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w, precision)
    # The panel copy is built from the sliced-ELL reverse index; an operator
    # whose slices would pad too much keeps the plain reverse index instead.
    lay = op.layouts()
    assert bool(lay & T_PANELS) == (panels and bool(lay & SLICED))
    ref = dev.prepare_with_transpose_precision(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w, precision)
    ref.force_plain_row_fold()
    assert not ref.layouts() & T_PANELS
    r = np.random.default_rng(seed)
    xt = r.uniform(-1, 1, nrows).astype(np.float32)
    yt0 = r.uniform(-1, 1, csr.ncols).astype(np.float32)
    got, alt = yt0.copy(), yt0.copy()
    op.spmv_t(xt, got)
    ref.spmv_t(xt, alt)
    want = O.spmv_t(O.csc_from_csr(csr, csr.ncols), wq, xt, yt0.copy())
    assert_bits_equal(got, want, "transpose panels vs oracle")
    assert_bits_equal(alt, want, "reverse-index fold vs oracle")
    return op, xt, yt0


@pytest.mark.parametrize("nrows,ncols,L", [
    (40, 33, 5),              # one slice, ragged last slice
    (100_000, 100_000, 64),   # config 1's shape: two panels over the rows
    (150_000, 2000, 16),      # three panels, long columns (~1,200 entries)
    (4 * MAX_PANEL, 5000, 4), # four full panels
])
@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16])
def test_transpose_panels_bit_exact(O, cuda_device, nrows, ncols, L, precision):
    csr, w = _uniform(O, nrows, ncols, L, nrows + 3 * L)
    op, _, _ = _check_t(O, cuda_device, csr, w, precision, L)
    if nrows >= 100_000:
        assert op.layouts() & T_PANELS


def test_transpose_panels_ragged_slices(O, cuda_device):
    """Rows of 1 to 40 entries and columns whose popularity grows sixfold
    across the matrix: every slice is padded to its own longest column, so
    the tiles have different depths, and short columns finish early."""
    r = np.random.default_rng(17)
    nrows, ncols = 120_000, 3000
    pop = 1.0 + 5.0 * np.arange(ncols) / ncols
    pop /= pop.sum()
    lens = r.integers(1, 41, nrows)
    rows = [np.sort(r.choice(ncols, k, replace=False, p=pop)) for k in lens]
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate(rows).astype(np.uint32)
    w = r.standard_normal(col.size).astype(np.float32)
    csr = O.Csr(rp.astype(np.uint32), col, ncols)
    op, _, _ = _check_t(O, cuda_device, csr, w, S.WeightPrecision.F32, 18)
    assert op.layouts() & T_PANELS


def test_transpose_panel_copy_follows_new_weights(O, cuda_device):
    csr, w = _uniform(O, 70_000, 5000, 12, 41)
    op, xt, yt0 = _check_t(O, cuda_device, csr, w, S.WeightPrecision.Bf16, 42)
    w2 = np.random.default_rng(43).uniform(-2, 2, w.size).astype(np.float32)
    op.set_weights(w2)
    got = yt0.copy()
    op.spmv_t(xt, got)
    want = O.spmv_t(O.csc_from_csr(csr, csr.ncols), O.quantise(int(S.WeightPrecision.Bf16), w2), xt, yt0.copy())
    assert_bits_equal(got, want, "spmv_t after set_weights")


def test_transpose_rows_past_the_panels_keep_the_reverse_index(O, cuda_device):
    csr, w = _uniform(O, 4 * MAX_PANEL + 1, 3000, 2, 51)
    op, _, _ = _check_t(O, cuda_device, csr, w, S.WeightPrecision.F32, 52, panels=False)
    assert op.layouts() & SLICED


ORDERED = 64  # SPARSL_LAYOUT_ORDERED_COPY
ROW_ORDER = 2  # SPARSL_LAYOUT_ROW_ORDER


def _skewed(O, nrows, ncols, seed, cap=3000, empty_every=0):
    r = np.random.default_rng(seed)
    lens = np.minimum(r.zipf(1.5, nrows), min(cap, ncols))
    if empty_every:
        lens[::empty_every] = 0
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(ncols, k, replace=False)) if k else np.zeros(0, np.int64)
                          for k in lens]).astype(np.uint32)
    w = (r.standard_normal(col.size) * 0.5).astype(np.float32)
    return O.Csr(rp.astype(np.uint32), col, ncols), w


@pytest.mark.parametrize("nrows,ncols,empty_every", [(40, 50, 7), (20_000, 300_000, 0), (200_000, 50_000, 13)])
@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_ordered_copy_spmv_bit_exact(O, cuda_device, nrows, ncols, empty_every, precision):
    """Skewed rows (Zipf lengths, some empty): dense-x SpMV over the ordered
    copy against the oracle and the generic row fold; y holds -0.0 values so
    an empty row's y + 0.0 is checked too."""
    csr, w = _skewed(O, nrows, ncols, nrows + ncols, empty_every=empty_every)
    wq = O.quantise(int(precision), w)
    op = cuda_device.prepare_with(S.Csr(csr.row_ptr, csr.col, ncols), ncols, w, precision)
    lay = op.layouts()
    assert bool(lay & ORDERED) == bool(lay & ROW_ORDER)
    if nrows >= 20_000:
        assert lay & ORDERED
    ref = cuda_device.prepare_with(S.Csr(csr.row_ptr, csr.col, ncols), ncols, w, precision)
    ref.force_plain_row_fold()
    assert not ref.layouts() & (ORDERED | ROW_ORDER)
    r = np.random.default_rng(3)
    x = r.uniform(-1, 1, ncols).astype(np.float32)
    y0 = r.uniform(-1, 1, nrows).astype(np.float32)
    y0[::5] = -0.0
    got, gen = y0.copy(), y0.copy()
    op.spmv(x, got)
    ref.spmv(x, gen)
    want = O.spmv(csr, wq, x, y0.copy())
    assert_bits_equal(got, want, "ordered copy vs oracle")
    assert_bits_equal(gen, want, "generic row fold vs oracle")


def test_ordered_copy_follows_new_weights(O, cuda_device):
    csr, w = _skewed(O, 50_000, 20_000, 77)
    op = cuda_device.prepare(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w)
    assert op.layouts() & ORDERED
    r = np.random.default_rng(78)
    x = r.uniform(-1, 1, csr.ncols).astype(np.float32)
    y0 = r.uniform(-1, 1, 50_000).astype(np.float32)
    w2 = r.uniform(-2, 2, w.size).astype(np.float32)
    op.set_weights(w2)
    got = y0.copy()
    op.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, w2, x, y0.copy()), "ordered spmv after set_weights")

"""CUDA path against the CPU oracle, bit for bit, through the C ABI.

The reference's differential suite compares every available backend with
CpuSequential (tests/differential.rs); the CUDA substrate is held to the
stronger rule the oracle makes checkable: identical bits (NaN payloads aside).
"""
import numpy as np
import pytest
import torch

from conftest import SHAPES, assert_bits_equal

import sparsl_b200 as S
from sparsl_b200 import _lib

pytestmark = pytest.mark.gpu

PARAMS = S.LifParams.new(0.9, 0.0, 0.1)  # tests/common/mod.rs:304-306


def _fixture(O, shape, seed):
    nrows, ncols, deg = shape
    rng = O.Rng(seed)
    csr = O.random_csr(nrows, ncols, deg, rng)
    w = O.random_vec(csr.nnz, 1.0, rng)
    x = O.random_vec(ncols, 1.0, rng)
    y = O.random_vec(nrows, 1.0, rng)
    return csr, w, x, y


def _scsr(csr):
    return S.Csr(csr.row_ptr, csr.col, csr.ncols)


def test_gpu_reproduces_reference_fingerprint(O, cuda_device):
    """tests/golden.rs:30-77 computed on the GPU: the reference's own hash."""
    h = 0xCBF29CE484222325
    mask = (1 << 64) - 1

    def fnv(bits_iter):
        nonlocal h
        for b in bits_iter:
            h ^= int(b)
            h = (h * 0x100000001B3) & mask

    rng = O.Rng(0x00601DE1)
    for nrows, ncols, deg in SHAPES:
        csr = O.random_csr(nrows, ncols, deg, rng)
        w = O.random_vec(csr.nnz, 1.0, rng)
        x = O.random_vec(ncols, 1.0, rng)
        op = cuda_device.prepare(_scsr(csr), ncols, w)
        y = O.random_vec(nrows, 1.0, rng)
        op.spmv(x, y)
        fnv(y.view(np.uint32))
        v = O.random_vec(nrows, 0.5, rng)
        th = np.abs(O.random_vec(nrows, 0.5, rng))
        sp = np.zeros(nrows, np.bool_)
        op.fused_spmv_lif(x, v, th, sp, PARAMS)
        for a, b in zip(v.view(np.uint32), th.view(np.uint32)):
            fnv((a, b))
        fnv(sp.astype(np.uint32))
    assert h == 0x2D29670756DFC8D6


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_spmv_family_bit_exact(O, cuda_device, shape, precision):
    nrows, ncols, deg = shape
    csr, w, x, y0 = _fixture(O, shape, 0xD1FF + nrows * 7 + ncols)
    op = cuda_device.prepare_with_transpose_precision(_scsr(csr), ncols, w, precision)
    assert op.weight_precision() is precision
    wq = O.quantise(int(precision), w)  # the operator holds the quantised values (mod.rs:1333)
    # y += A x
    got = y0.copy()
    op.spmv(x, got)
    want = O.spmv(csr, wq, x, y0.copy())
    assert_bits_equal(got, want, f"spmv {shape}")
    # packed spikes == dense 0/1 (spikes_backend.rs:91-129)
    r = np.random.default_rng(nrows + ncols)
    s = (r.random(ncols) < 0.3).astype(np.uint8)
    packed = O.pack_spikes(s)
    got = y0.copy()
    op.spmv_spikes(packed, got)
    want = O.spmv_spikes(csr, wq, packed, y0.copy())
    assert_bits_equal(got, want, f"spmv_spikes {shape}")
    # y += A^T x
    csc = O.csc_from_csr(csr, ncols)
    xt = O.random_vec(nrows, 1.0, O.Rng(nrows))
    yt0 = O.random_vec(ncols, 1.0, O.Rng(ncols + 1))
    got = yt0.copy()
    op.spmv_t(xt, got)
    want = O.spmv_t(csc, wq, xt, yt0.copy())
    assert_bits_equal(got, want, f"spmv_t {shape}")


@pytest.mark.parametrize("shape", [(1, 64, 64), (33, 33, 5), (257, 128, 16), (1000, 1000, 64)])
@pytest.mark.parametrize("n_vec", [1, 2, 3, 16, 33, 64, 70])
def test_spmm_bit_exact_and_columns_match_spmv(O, cuda_device, shape, n_vec):
    nrows, ncols, deg = shape
    csr, w, _, _ = _fixture(O, shape, 0x5A11 + n_vec)
    rng = O.Rng(n_vec * 31 + nrows)
    X = O.random_vec(ncols * n_vec, 1.0, rng)
    Y0 = O.random_vec(nrows * n_vec, 1.0, rng)
    for p in (S.WeightPrecision.F32, S.WeightPrecision.F16):
        op = cuda_device.prepare_with(_scsr(csr), ncols, w, p)
        got = Y0.copy()
        op.spmm(X, n_vec, got)
        want = O.spmm(csr, O.quantise(int(p), w), X, n_vec, Y0.copy())
        assert_bits_equal(got, want, f"spmm {shape} n_vec={n_vec} {p}")
        # each column equals its own SpMV (tests/spmm.rs:104-135)
        for v in {0, n_vec - 1}:
            yv = Y0.reshape(nrows, n_vec)[:, v].copy()
            op.spmv(np.ascontiguousarray(X.reshape(ncols, n_vec)[:, v]), yv)
            assert_bits_equal(got.reshape(nrows, n_vec)[:, v], yv, f"column {v}")


@pytest.mark.parametrize("shape", SHAPES)
def test_fused_lif_bit_exact(O, cuda_device, shape):
    nrows, ncols, deg = shape
    csr, w, x, _ = _fixture(O, shape, 0xF05E + nrows)
    op = cuda_device.prepare(_scsr(csr), ncols, w)
    rng = O.Rng(0x77 + nrows)
    v0 = O.random_vec(nrows, 0.5, rng)
    th0 = np.abs(O.random_vec(nrows, 0.5, rng))
    v, th, sp = v0.copy(), th0.copy(), np.zeros(nrows, np.bool_)
    op.fused_spmv_lif(x, v, th, sp, PARAMS)
    vw, tw, sw = v0.copy(), th0.copy(), np.zeros(nrows, np.uint8)
    O.fused_lif(csr, w, x, vw, tw, sw, 0.9, 0.0, 0.1)
    assert_bits_equal(v, vw, "v")
    assert_bits_equal(th, tw, "theta")
    assert np.array_equal(sp.astype(np.uint8), sw)
    # spike-vector variant
    s = (np.random.default_rng(nrows).random(ncols) < 0.4).astype(np.uint8)
    packed = O.pack_spikes(s)
    v, th, sp = v0.copy(), th0.copy(), np.zeros(nrows, np.bool_)
    op.fused_spmv_spikes_lif(packed, v, th, sp, PARAMS)
    vw, tw, sw = v0.copy(), th0.copy(), np.zeros(nrows, np.uint8)
    O.fused_spikes_lif(csr, w, packed, vw, tw, sw, 0.9, 0.0, 0.1)
    assert_bits_equal(v, vw, "v spikes")
    assert_bits_equal(th, tw, "theta spikes")
    assert np.array_equal(sp.astype(np.uint8), sw)


def test_lif_integrate_and_fma_counterexample(O, cuda_device):
    """Separate roundings on the GPU: v*decay+cur == 0.0 exactly (mod.rs:517-521)."""
    v = np.array([0.99999106], np.float32)
    th = np.array([10.0], np.float32)
    sp = np.zeros(1, np.bool_)
    cuda_device.lif_integrate(v, th, np.array([-1.0999901], np.float32), sp, S.LifParams.new(1.1, 0.0, 0.0))
    assert v[0] == 0.0
    r = np.random.default_rng(9)
    n = 100_003
    v0 = r.standard_normal(n).astype(np.float32)
    t0 = np.abs(r.standard_normal(n)).astype(np.float32)
    cur = r.standard_normal(n).astype(np.float32)
    v, t, s = v0.copy(), t0.copy(), np.zeros(n, np.bool_)
    cuda_device.lif_integrate(v, t, cur, s, S.LifParams.new(0.95, -0.25, 0.05))
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(n, np.uint8)
    O.lif_integrate(vw, tw, cur, sw, np.float32(0.95), np.float32(-0.25), np.float32(0.05))
    assert_bits_equal(v, vw)
    assert_bits_equal(t, tw)
    assert np.array_equal(s.astype(np.uint8), sw)
    # the device-array entry point, on a torch stream
    L = _lib.load()
    dv, dt, dc = (torch.from_numpy(a.copy()).cuda() for a in (v0, t0, cur))
    ds = torch.zeros(n, dtype=torch.uint8, device="cuda")
    st = torch.cuda.Stream()
    torch.cuda.synchronize()
    assert L.sparsl_dev_lif_integrate_device(cuda_device.handle, dv.data_ptr(), dt.data_ptr(), dc.data_ptr(),
                                             ds.data_ptr(), n, 0.95, -0.25, 0.05, st.cuda_stream) == 0
    st.synchronize()
    assert_bits_equal(dv.cpu().numpy(), vw)
    assert_bits_equal(dt.cpu().numpy(), tw)
    assert np.array_equal(ds.cpu().numpy(), sw)
    host = np.zeros(n, np.float32)
    assert L.sparsl_dev_lif_integrate_device(cuda_device.handle, host.ctypes.data, dt.data_ptr(), dc.data_ptr(),
                                             ds.data_ptr(), n, 0.95, -0.25, 0.05, None) == _lib.SPARSL_ERR_INVALID
    # arrays off the 16-byte grid take the cell-by-cell kernel: same bits
    m = n - 1
    dv2, dt2, dc2 = (torch.from_numpy(np.concatenate([[0], a])).float().cuda()[1:] for a in (v0[:m], t0[:m], cur[:m]))
    ds2 = torch.zeros(m + 1, dtype=torch.uint8, device="cuda")[1:]
    torch.cuda.synchronize()
    assert L.sparsl_dev_lif_integrate_device(cuda_device.handle, dv2.data_ptr(), dt2.data_ptr(), dc2.data_ptr(),
                                             ds2.data_ptr(), m, 0.95, -0.25, 0.05, None) == 0
    assert L.sparsl_dev_wait(cuda_device.handle) == 0
    assert_bits_equal(dv2.cpu().numpy(), vw[:m])
    assert np.array_equal(ds2.cpu().numpy(), sw[:m])


def test_resident_api_equals_slice_api(O, cuda_device):
    """tests/wave3_usefulness.rs: write_* / *_resident / sync_* == slice calls."""
    csr, w, x, y0 = _fixture(O, (300, 300, 20), 0xAE5)
    op = cuda_device.prepare(_scsr(csr), 300, w)
    op.write_x(x)
    op.write_y(y0)
    op.spmv_resident()
    got = np.zeros(300, np.float32)
    op.sync_y(got)
    assert_bits_equal(got, O.spmv(csr, w, x, y0.copy()))
    v0 = O.random_vec(300, 0.5, O.Rng(1))
    t0 = np.abs(O.random_vec(300, 0.5, O.Rng(2)))
    op.write_lif_state(v0, t0)
    op.fused_spmv_lif_resident(PARAMS)
    v, t, sp = np.zeros(300, np.float32), np.zeros(300, np.float32), np.zeros(300, np.bool_)
    op.sync_lif_state(v, t, sp)
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(300, np.uint8)
    O.fused_lif(csr, w, x, vw, tw, sw, 0.9, 0.0, 0.1)
    assert_bits_equal(v, vw)
    assert np.array_equal(sp.astype(np.uint8), sw)
    # pack + spikes resident
    op.pack_resident_spikes_to_x_spikes()
    assert np.array_equal(op.sync_x_spikes(), O.pack_spikes(sw))
    op.fused_spmv_spikes_lif_resident(PARAMS)
    O.fused_spikes_lif(csr, w, O.pack_spikes(sw), vw, tw, sw, 0.9, 0.0, 0.1)
    op.sync_lif_state(v, t, sp)
    assert_bits_equal(v, vw)
    assert_bits_equal(t, tw)


@pytest.mark.parametrize("n,deg,density", [(31, 5, 0.3), (1000, 64, 0.05), (4096, 100, 0.02), (20000, 300, 0.02)])
def test_recurrent_steps_trace_and_state_bit_exact(O, cuda_device, n, deg, density):
    rng = O.Rng(0x71C + n)
    csr = O.random_csr(n, n, deg, rng)
    w = O.random_vec(csr.nnz, 0.6, rng)
    v0 = O.random_vec(n, 1.0, rng)
    t0 = np.full(n, 0.4, np.float32)
    s0 = (np.random.default_rng(n).random(n) < density).astype(np.uint8)
    xs0 = O.pack_spikes(s0)
    params = S.LifParams.new(0.95, 0.0, 0.0)
    op = cuda_device.prepare(_scsr(csr), n, w)
    op.write_x_spikes(xs0)
    op.write_lif_state(v0, t0)
    steps = 25
    op.fused_spmv_spikes_lif_recurrent_steps(params, steps)
    vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(n, np.uint8), xs0.copy()
    trace_w = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, steps)
    assert np.array_equal(op.spike_trace(), trace_w)
    v, t, sp = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.bool_)
    op.sync_lif_state(v, t, sp)
    assert_bits_equal(v, vw)
    assert_bits_equal(t, tw)
    assert np.array_equal(sp.astype(np.uint8), sw)
    assert np.array_equal(op.sync_x_spikes(), xw)
    # device-compacted index list == ascending positions of the last tick
    assert np.array_equal(op.spike_indices(), np.flatnonzero(sw).astype(np.uint32))


def _leak_steps(n, seed):
    r = np.random.default_rng(seed)
    tau = (2.0 + r.random(n) * 8.0).astype(np.float32)
    inp = (r.random(n) * 2.0 - 1.0).astype(np.float32)
    alpha = (np.float32(1.0) / tau).astype(np.float32)
    return np.stack([np.float32(1.0) - alpha, alpha * inp], 1).astype(np.float32)


@pytest.mark.parametrize("n", [1, 2, 17, 33, 255, 4095, 4096, 4097, 8192 + 129, 100_000, 1_000_003])
def test_scan_bit_exact_leak_steps(O, cuda_device, n):
    xs = _leak_steps(n, n)
    got = cuda_device.assoc_scan(xs)
    assert_bits_equal(got, O.scan_sequential(xs), f"n={n}")
    assert_bits_equal(cuda_device.assoc_scan(xs), got, "repeat is byte-identical")


@pytest.mark.parametrize("n", [4096 * 3 + 5, 1 << 20])
def test_scan_bit_exact_decay_workload(O, cuda_device, n):
    """a ~ U[0.9, 1], b ~ N(0, 1): the multiplier sticks at a denormal fixed point."""
    r = np.random.default_rng(2)
    xs = np.stack([r.uniform(0.9, 1.0, n), r.standard_normal(n)], 1).astype(np.float32)
    got = cuda_device.assoc_scan(xs)
    assert_bits_equal(got, O.scan_sequential(xs))
    rep, seg = cuda_device.scan_stats()
    assert rep < n // 4, f"scan replayed {rep} of {n} elements serially"


@pytest.mark.parametrize("n", [2 << 22, 3 << 22 | 4097])
def test_scan_host_buffers_chunked_pipeline(O, cuda_device, n):
    """Host buffers of at least two 2^22-map chunks are uploaded, scanned and
    downloaded chunk by chunk, each chunk continuing from the last state the
    previous one wrote: the result is still the one sequential fold, equal to
    the single-pass device entry point, and only the very first map is copied
    (a first map of (inf, -0.0) survives bit for bit)."""
    r = np.random.default_rng(n)
    xs = np.stack([r.uniform(0.9, 1.0, n), r.standard_normal(n)], 1).astype(np.float32)
    xs[0] = (np.inf, -0.0)
    xs[(1 << 22) - 1] = (1.0, 0.0)  # identity on a chunk's last map
    xs[1 << 22] = (0.5, 7.0)  # and a plain map on the next chunk's first
    got = cuda_device.assoc_scan(xs)
    assert_bits_equal(got, O.scan_sequential(xs), f"n={n}")
    d_in = torch.from_numpy(xs).cuda()
    d_out = torch.empty_like(d_in)
    cuda_device.assoc_scan_from_device(d_in, n, d_out)
    cuda_device.wait()
    assert_bits_equal(got, d_out.cpu().numpy(), "chunked host path vs one device pass")
    assert_bits_equal(cuda_device.assoc_scan(xs), got, "repeat is byte-identical")


def test_scan_known_answers(O, cuda_device):
    """tests/scan_backend.rs:274-419."""
    for n in (1, 1023, 1024, 1025, 5000, 60_000):
        got = cuda_device.assoc_scan(np.tile(np.array([1.0, 1.0], np.float32), (n, 1)))
        assert np.array_equal(got[:, 1], np.arange(1, n + 1, dtype=np.float32))
        assert np.all(got[:, 0] == 1.0)
    got = cuda_device.assoc_scan(np.tile(np.array([2.0, 0.0], np.float32), (100, 1)))
    assert np.array_equal(got[:, 0], np.float32(2.0) ** np.arange(1, 101, dtype=np.float32))
    cyc = np.array([[2.0, 1.0], [0.5, 0.5], [1.0, 1.0]], np.float32)
    xs = cyc[np.arange(4 * 1024 + 33) % 3]
    assert_bits_equal(cuda_device.assoc_scan(xs), O.scan_sequential(xs))
    first = np.array([[np.inf, -0.0]], np.float32)
    assert_bits_equal(cuda_device.assoc_scan(first), first)
    assert cuda_device.assoc_scan(np.zeros((0, 2), np.float32)).shape == (0, 2)
    growth = np.tile(np.array([1.1, 0.0], np.float32), (100, 1))
    assert_bits_equal(cuda_device.assoc_scan(growth), O.scan_sequential(growth))


def test_scan_identity_padding(O, cuda_device):
    xs = _leak_steps(2000, 0x1DEA)
    plain = cuda_device.assoc_scan(xs)
    padded = np.concatenate([np.array([[1.0, 0.0]], np.float32), xs])
    assert_bits_equal(cuda_device.assoc_scan(padded)[1:], plain)  # the fold treats identity as a no-op
    for extra in (1, 31, 724, 800, 5000):
        tail = np.concatenate([xs[:300], np.tile(np.array([1.0, 0.0], np.float32), (extra, 1))])
        assert_bits_equal(cuda_device.assoc_scan(tail)[:300], plain[:300])


def test_cleared_spike_still_multiplies_non_finite_weights(O, cuda_device):
    """tests/spikes_backend.rs:48-89: inf * 0.0 is NaN, never skipped."""
    rng = O.Rng(0x5B18)
    for nrows, ncols, deg in [(48, 64, 4), (48, 64, 40), (48, 64, 160)]:
        csr = O.random_csr(nrows, ncols, deg, rng)
        for poison in (np.inf, -np.inf, np.nan):
            w = O.random_vec(csr.nnz, 1.0, rng)
            w[0] = poison
            s = np.array([c != csr.col[0] for c in range(ncols)], np.uint8)
            packed = O.pack_spikes(s)
            op = cuda_device.prepare(_scsr(csr), ncols, w)
            a = np.zeros(nrows, np.float32)
            op.spmv(s.astype(np.float32), a)
            b = np.zeros(nrows, np.float32)
            op.spmv_spikes(packed, b)
            assert_bits_equal(b, a)
            row = int(np.searchsorted(csr.row_ptr, 0, side="right")) - 1  # row holding edge 0
            assert np.isnan(b[row])


def test_subnormals_and_non_finite_propagate(O, cuda_device):
    """tests/stress.rs:324-384: no flush to zero, NaN/inf by class."""
    csr = O.Csr.from_adjacency([[0, 1, 2], [1], [0, 2], []])
    tiny = np.float32(1e-40)
    w = np.array([tiny, 2.0, -3.0, tiny, np.inf, 1.0], np.float32)
    x = np.array([1.0, 0.5, tiny], np.float32)
    op = cuda_device.prepare(_scsr(csr), 4, w)
    got = np.zeros(4, np.float32)
    op.spmv(np.concatenate([x, [0.0]]).astype(np.float32), got)
    want = O.spmv(csr, w, np.concatenate([x, [0.0]]).astype(np.float32), np.zeros(4, np.float32))
    assert_bits_equal(got, want)
    assert got[1] != 0.0  # tiny * 0.5 survived as a subnormal


def test_long_row_and_degenerate_shapes(O, cuda_device):
    """tests/stress.rs:391-458: a 200k-nnz single row, empty rows and columns."""
    n = 200_000
    csr = O.Csr(np.array([0, n], np.uint32), np.arange(n, dtype=np.uint32), n)
    w = O.random_vec(n, 1.0, O.Rng(3))
    x = O.random_vec(n, 1.0, O.Rng(4))
    op = cuda_device.prepare(_scsr(csr), n, w)
    got = np.zeros(1, np.float32)
    op.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, w, x, np.zeros(1, np.float32)))
    for nrows, ncols in [(0, 0), (0, 5), (5, 0), (3, 3)]:
        e = S.Csr.empty(nrows, ncols)
        op = cuda_device.prepare(e, ncols, np.zeros(0, np.float32))
        y = np.ones(nrows, np.float32)
        op.spmv(np.zeros(ncols, np.float32), y)
        assert np.all(y == 1.0)
        assert op.shape().nnz() == 0


def test_errors_mirror_the_reference(cuda_device):
    csr = S.Csr.from_adjacency([[1], [0]])
    op = cuda_device.prepare(csr, 2, np.ones(2, np.float32))
    with pytest.raises(S.OpError) as ei:
        op.spmv_t(np.zeros(2, np.float32), np.zeros(2, np.float32))
    assert ei.value.kind == "TransposeNotPrepared"
    with pytest.raises(S.OpError) as ei:
        op.spmv(np.zeros(1, np.float32), np.zeros(2, np.float32))
    assert ei.value.kind == "TooShort" and ei.value.fields["what"] == "x"
    with pytest.raises(S.OpError) as ei:
        op.spmv(np.zeros(2, np.float32), np.zeros(3, np.float32))
    assert ei.value.kind == "Length"
    with pytest.raises(S.OpError) as ei:
        op.spmm(np.zeros(2, np.float32), 0, np.zeros(0, np.float32))
    assert ei.value.kind == "Length" and ei.value.fields["what"] == "n_vec"
    with pytest.raises(S.SparsePlanError) as ei:
        cuda_device.prepare(csr, 2, np.ones(3, np.float32))
    assert ei.value.kind == "WeightsLen"
    with pytest.raises(S.SparsePlanError) as ei:
        cuda_device.prepare(S.Csr.from_parts_unchecked([0, 1], [7], 2), 2, np.ones(1, np.float32))
    assert ei.value.kind == "ColumnOutOfRange" and ei.value.fields["col"] == 7
    with pytest.raises(S.SparsePlanError) as ei:
        cuda_device.prepare(csr, 3, np.ones(2, np.float32))
    assert ei.value.kind == "NcolsMismatch"


def test_set_weights_keeps_precision(O, cuda_device):
    csr, w, x, y0 = _fixture(O, (257, 128, 16), 0x5E7)
    op = cuda_device.prepare_bf16(_scsr(csr), 128, w)
    w2 = O.random_vec(csr.nnz, 2.0, O.Rng(99))
    op.set_weights(w2)
    got = y0.copy()
    op.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, O.quantise(2, w2), x, y0.copy()))


def test_device_reports_b200(cuda_device):
    assert cuda_device.label() == "CUDA GPU"
    assert cuda_device.backend() is S.Backend.Cuda
    assert "B200" in cuda_device.device_name()
    assert S.Backend.Cuda in S.available_backends()


@pytest.mark.parametrize("kind", ["power_law", "uniform"])
@pytest.mark.parametrize("n_vec", [3, 64, 100])
def test_spmm_work_units_bit_exact(O, cuda_device, kind, n_vec):
    """Rows handed out in work units (longest rows first, or runs of equal
    rows): empty and 2000-entry rows, -0.0 outputs, and two launches in a row
    (the unit counters must rewind)."""
    r = np.random.default_rng(n_vec + len(kind))
    nrows, ncols = 3000, 5000
    if kind == "power_law":
        lens = np.minimum(r.zipf(1.5, nrows), 2000)
        lens[::97] = 0
    else:
        lens = np.full(nrows, 8)
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(ncols, k, replace=False)) for k in lens]).astype(np.uint32)
    csr = O.Csr(rp.astype(np.uint32), col, ncols)
    w = r.uniform(-1, 1, col.size).astype(np.float32)
    X = r.uniform(-1, 1, ncols * n_vec).astype(np.float32)
    Y0 = r.uniform(-1, 1, nrows * n_vec).astype(np.float32)
    Y0[::5] = -0.0
    op = cuda_device.prepare(_scsr(csr), ncols, w)
    got = Y0.copy()
    op.spmm(X, n_vec, got)
    op.spmm(X, n_vec, got)
    want = O.spmm(csr, w, X, n_vec, Y0.copy())
    want = O.spmm(csr, w, X, n_vec, want)
    assert_bits_equal(got, want, f"spmm {kind} n_vec={n_vec}")
    empty = np.flatnonzero(lens == 0)
    if empty.size:  # -0.0 + 0.0 + 0.0 is +0.0 on an empty row
        row = got.reshape(nrows, n_vec)[empty]
        assert not np.any(np.signbit(row) & (row == 0))


@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
def test_set_weights_refreshes_the_transpose(O, cuda_device, precision):
    """The transpose product reads the weights in reverse-index order; after
    set_weights both directions must use the new weights (mod.rs:1397)."""
    nrows, ncols, deg = 1000, 700, 40
    csr, w, x, y0 = _fixture(O, (nrows, ncols, deg), 0x7A11 + int(precision))
    op = cuda_device.prepare_with_transpose_precision(_scsr(csr), ncols, w, precision)
    w2 = O.random_vec(csr.nnz, 3.0, O.Rng(0x33 + int(precision)))
    w2[::97] = np.inf
    op.set_weights(w2)
    wq = O.quantise(int(precision), w2)
    csc = O.csc_from_csr(csr, ncols)
    rng = O.Rng(0x44)
    xt = O.random_vec(nrows, 1.0, rng)
    yt0 = O.random_vec(ncols, 1.0, rng)
    got = yt0.copy()
    op.spmv_t(xt, got)
    assert_bits_equal(got, O.spmv_t(csc, wq, xt, yt0.copy()), "spmv_t after set_weights")
    got = y0.copy()
    op.spmv(x, got)
    assert_bits_equal(got, O.spmv(csr, wq, x, y0.copy()), "spmv after set_weights")


@pytest.mark.parametrize("hub", [False, True])
def test_spmv_t_sliced_and_hub_layouts(O, cuda_device, hub):
    """The transpose product runs over a sliced-ELL copy of the reverse index;
    a hub column (here in every row) would pad that copy beyond twice the
    nonzeros, so such operators keep the CSC row-fold path.  Both must equal
    the reference's col_dot fold bit for bit, in every precision."""
    r = np.random.default_rng(7 + hub)
    nrows, ncols = 3000, 2000
    rows = []
    for i in range(nrows):
        k = int(r.integers(0, 12))
        cols = set(r.choice(ncols, k, replace=False).tolist())
        if hub:
            cols.add(5)
        rows.append(sorted(cols))
    lens = np.array([len(c) for c in rows])
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.array([c for row in rows for c in row], np.uint32)
    csr = O.Csr(rp.astype(np.uint32), col, ncols)
    w = r.uniform(-1, 1, col.size).astype(np.float32)
    w[::41] = np.inf
    csc = O.csc_from_csr(csr, ncols)
    xt = r.uniform(-1, 1, nrows).astype(np.float32)
    xt[::13] = 0.0
    yt0 = r.uniform(-1, 1, ncols).astype(np.float32)
    yt0[::7] = -0.0
    for p in (S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16):
        op = cuda_device.prepare_with_transpose_precision(_scsr(csr), ncols, w, p)
        # SPARSL_LAYOUT_CSC (8) for the hub, SPARSL_LAYOUT_SLICED_REVERSE (4) otherwise
        assert op.layouts() & (8 if hub else 4) and not op.layouts() & (4 if hub else 8)
        got = yt0.copy()
        op.spmv_t(xt, got)
        want = O.spmv_t(csc, O.quantise(int(p), w), xt, yt0.copy())
        assert_bits_equal(got, want, f"spmv_t hub={hub} {p}")


@pytest.mark.parametrize("kind", ["power_law", "uniform"])
@pytest.mark.parametrize("n_vec", [3, 64])
def test_spmm_row_range_pipeline_bit_exact(O, cuda_device, kind, n_vec):
    """Operators of 65,536 rows or more run the host-buffer SpMM one row
    range at a time, with each range's Y rows copied in and out around its own
    launch.  The result is the oracle's bit for bit, and equals the device
    entry point, which runs all rows in one launch."""
    r = np.random.default_rng(n_vec * 7 + len(kind))
    nrows, ncols = 70_001, 5000
    if kind == "power_law":
        lens = np.minimum(r.zipf(1.5, nrows), 1000)
        lens[::97] = 0
    else:
        lens = np.full(nrows, 5)
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(ncols, k, replace=False)) for k in lens]).astype(np.uint32)
    csr = O.Csr(rp.astype(np.uint32), col, ncols)
    w = r.uniform(-1, 1, col.size).astype(np.float32)
    X = r.uniform(-1, 1, ncols * n_vec).astype(np.float32)
    Y0 = r.uniform(-1, 1, nrows * n_vec).astype(np.float32)
    Y0[::5] = -0.0
    op = cuda_device.prepare(_scsr(csr), ncols, w)
    want = O.spmm(csr, w, X, n_vec, Y0.copy())
    got = Y0.copy()
    op.spmm(X, n_vec, got)
    assert_bits_equal(got, want, f"spmm ranges {kind} n_vec={n_vec}")
    dx = torch.from_numpy(X).cuda()
    dy = torch.from_numpy(Y0).cuda()
    assert _lib.load().sparsl_op_spmm_device(op.handle, dx.data_ptr(), n_vec, dy.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert_bits_equal(dy.cpu().numpy(), want, "device entry point, one launch")
    op.spmm(X, n_vec, got)  # again: the unit counters rewound after every range
    assert_bits_equal(got, O.spmm(csr, w, X, n_vec, want.copy()), "second call")


def _skewed(O, nrows, ncols, seed, cap=3000):
    """Zipf(1.5) row lengths clipped to [0, cap], a few empty rows and one hub
    row of `cap` entries: the shape that takes the descending-length order."""
    r = np.random.default_rng(seed)
    lens = np.minimum(r.zipf(1.5, nrows), cap)
    lens[::53] = 0
    lens[nrows // 3] = cap
    rp = np.zeros(nrows + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(ncols, k, replace=False)) for k in lens]).astype(np.uint32)
    return O.Csr(rp.astype(np.uint32), col, ncols), r


@pytest.mark.parametrize("precision", [S.WeightPrecision.F32, S.WeightPrecision.F16, S.WeightPrecision.Bf16])
@pytest.mark.parametrize("nrows,ncols", [(5000, 6000), (40000, 700_000)])
def test_skewed_rows_take_the_length_order_bit_exact(O, cuda_device, precision, nrows, ncols):
    """Power-law rows fold in descending-length order (warps of similar
    rows); every product still equals the reference's per-row left fold, and
    the natural-order engine on the same operator."""
    csr, r = _skewed(O, nrows, ncols, nrows + int(precision))
    w = r.uniform(-1, 1, csr.nnz).astype(np.float32)
    wq = O.quantise(int(precision), w)
    op = cuda_device.prepare_with(_scsr(csr), ncols, w, precision)
    assert op.layouts() & 2, "skewed rows should take the descending-length order"
    plain = cuda_device.prepare_with(_scsr(csr), ncols, w, precision)
    plain.force_plain_row_fold()
    assert not plain.layouts() & 2
    x = r.uniform(-1, 1, ncols).astype(np.float32)
    y0 = r.uniform(-1, 1, nrows).astype(np.float32)
    y0[::7] = -0.0
    got, ref = y0.copy(), y0.copy()
    op.spmv(x, got)
    plain.spmv(x, ref)
    want = O.spmv(csr, wq, x, y0.copy())
    assert_bits_equal(got, want, "spmv")
    assert_bits_equal(ref, want, "spmv, natural order")
    pk = O.pack_spikes((r.random(ncols) < 0.2).astype(np.uint8))
    got = y0.copy()
    op.spmv_spikes(pk, got)
    assert_bits_equal(got, O.spmv_spikes(csr, wq, pk, y0.copy()), "spmv_spikes")
    v0 = r.uniform(-1, 1, nrows).astype(np.float32)
    t0 = np.abs(r.uniform(0, 1, nrows)).astype(np.float32)
    v, t, sp = v0.copy(), t0.copy(), np.zeros(nrows, np.bool_)
    op.fused_spmv_lif(x, v, t, sp, PARAMS)
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(nrows, np.uint8)
    O.fused_lif(csr, wq, x, vw, tw, sw, 0.9, 0.0, 0.1)
    assert_bits_equal(v, vw, "fused v")
    assert_bits_equal(t, tw, "fused theta")
    assert np.array_equal(sp.astype(np.uint8), sw)
    v, t, sp = v0.copy(), t0.copy(), np.zeros(nrows, np.bool_)
    op.fused_spmv_spikes_lif(pk, v, t, sp, PARAMS)
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(nrows, np.uint8)
    O.fused_spikes_lif(csr, wq, pk, vw, tw, sw, 0.9, 0.0, 0.1)
    assert_bits_equal(v, vw, "fused spikes v")
    assert np.array_equal(sp.astype(np.uint8), sw)


@pytest.mark.parametrize("n", [3000, 70_001])
def test_skewed_recurrent_ticks_pack_and_compact_bit_exact(O, cuda_device, n):
    """Recurrent ticks on a square skewed operator: the ordered fold, then the
    packing and the index list from the spike bytes."""
    csr, r = _skewed(O, n, n, n, cap=1500)
    w = (r.standard_normal(csr.nnz) * 0.3).astype(np.float32)
    v0 = r.uniform(0, 1, n).astype(np.float32)
    t0 = np.full(n, 0.5, np.float32)
    xs0 = O.pack_spikes((r.random(n) < 0.1).astype(np.uint8))
    op = cuda_device.prepare(_scsr(csr), n, w)
    assert op.layouts() & 2
    op.write_x_spikes(xs0)
    op.write_lif_state(v0, t0)
    steps = 12
    op.fused_spmv_spikes_lif_recurrent_steps(S.LifParams.new(0.95, 0.0, 0.0), steps)
    vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(n, np.uint8), xs0.copy()
    trace_w = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, steps)
    assert trace_w.sum() > 0
    assert np.array_equal(op.spike_trace(), trace_w)
    v, t, sp = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.bool_)
    op.sync_lif_state(v, t, sp)
    assert_bits_equal(v, vw)
    assert_bits_equal(t, tw)
    assert np.array_equal(op.sync_x_spikes(), xw)
    assert np.array_equal(op.spike_indices(), np.flatnonzero(sw).astype(np.uint32))

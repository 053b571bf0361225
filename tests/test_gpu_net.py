"""The network tick runtime (row-block operators + all-gather + trace) against
the oracle's recurrent ticks, and the GPU workload generator against its
definition.  Single GPU: one rank, several row blocks."""
import ctypes

import numpy as np
import pytest

from conftest import assert_bits_equal

import sparsl_b200 as S
from sparsl_b200 import _lib

pytestmark = pytest.mark.gpu


def _check(rc):
    assert rc == 0, _lib.last_error()


def _make_net(dev, ops, row0, n):
    L = _lib.load()
    arr = (ctypes.c_void_p * len(ops))(*[op.handle.value for op in ops])
    h = ctypes.c_void_p()
    _check(L.sparsl_net_create(dev.handle, arr, len(ops), row0, n, 0, 1, None, ctypes.byref(h)))
    return h


def _skewed_csr(O, n, seed):
    r = np.random.default_rng(seed)
    lens = np.minimum(r.zipf(1.5, n), 1200)
    lens[n // 2] = 1200
    rp = np.zeros(n + 1, np.uint64)
    np.cumsum(lens, out=rp[1:])
    col = np.concatenate([np.sort(r.choice(n, k, replace=False)) for k in lens]).astype(np.uint32)
    return O.Csr(rp.astype(np.uint32), col, n)


NETS = [(4096, 64, [2048, 2048]), (6016, 200, [1024, 32, 4960]), (8192, 0, [4096, 4096])]


def _net_case(O, dev, n, deg, splits):
    """A network of row blocks and its initial state (deg 0: power-law rows,
    whose blocks fold in descending-length order)."""
    rng = O.Rng(0xE7 + n)
    csr = O.random_csr(n, n, deg, rng) if deg else _skewed_csr(O, n, n)
    w = O.random_vec(csr.nnz, 0.5, rng)
    v0 = O.random_vec(n, 1.0, rng)
    t0 = np.full(n, 0.45, np.float32)
    xs0 = O.pack_spikes((np.random.default_rng(n).random(n) < 0.03).astype(np.uint8))
    ops, r = [], 0
    for k in splits:
        rp = (csr.row_ptr[r:r + k + 1] - csr.row_ptr[r]).astype(np.uint32)
        col = csr.col[csr.row_ptr[r]:csr.row_ptr[r + k]]
        ww = w[csr.row_ptr[r]:csr.row_ptr[r + k]]
        ops.append(dev.prepare(S.Csr(rp, col, n), n, ww))
        r += k
    return csr, w, v0, t0, xs0, ops


@pytest.mark.parametrize("n,deg,splits", NETS)
def test_net_ticks_match_oracle_recurrent_steps(O, cuda_device, n, deg, splits):
    csr, w, v0, t0, xs0, ops = _net_case(O, cuda_device, n, deg, splits)
    L = _lib.load()
    net = _make_net(cuda_device, ops, 0, n)
    try:
        _check(L.sparsl_net_write_state(net, xs0.ctypes.data, xs0.size, v0.ctypes.data, t0.ctypes.data, n))
        steps = 30
        _check(L.sparsl_net_steps(net, 0.95, 0.0, 0.0, steps))
        trace = np.zeros(steps, np.uint32)
        cnt = ctypes.c_uint64()
        _check(L.sparsl_net_trace(net, trace.ctypes.data, steps, ctypes.byref(cnt)))
        vw, tw, sw, xw = v0.copy(), t0.copy(), np.zeros(n, np.uint8), xs0.copy()
        want = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, steps)
        assert np.array_equal(trace, want)
        xs, v, t = np.zeros_like(xs0), np.zeros(n, np.float32), np.zeros(n, np.float32)
        _check(L.sparsl_net_read_state(net, xs.ctypes.data, xs.size, v.ctypes.data, t.ctypes.data, n))
        assert np.array_equal(xs, xw)
        assert_bits_equal(v, vw)
        assert_bits_equal(t, tw)
    finally:
        L.sparsl_net_destroy(net)


class _Host:
    """Host arrays for the state: pinned (sparsl_host_alloc) or pageable."""

    def __init__(self, L, pinned, like):
        self.L, self.ptr = L, None
        if pinned:
            self.ptr = L.sparsl_host_alloc(max(like.nbytes, 16))
            buf = (ctypes.c_char * like.nbytes).from_address(self.ptr)
            self.a = np.frombuffer(buf, dtype=like.dtype, count=like.size)
        else:
            self.a = np.empty_like(like)
        self.a[:] = like

    def free(self):
        if self.ptr:
            self.L.sparsl_host_free(self.ptr)


@pytest.mark.parametrize("n,deg,splits", NETS)
@pytest.mark.parametrize("pinned", [True, False])
def test_net_steps_host_matches_oracle_recurrent_steps(O, cuda_device, n, deg, splits, pinned):
    """State in from host buffers, ticks, state back into the same buffers,
    each block's copies on their own streams: one-tick and four-tick calls
    against the oracle's ticks, the trace of each call, and a call made while
    ticks of sparsl_net_steps_async are still in flight (its copies must wait
    for them)."""
    csr, w, v0, t0, xs0, ops = _net_case(O, cuda_device, n, deg, splits)
    L = _lib.load()
    net = _make_net(cuda_device, ops, 0, n)
    hx, hv, ht = _Host(L, pinned, xs0), _Host(L, pinned, v0), _Host(L, pinned, t0)
    xw, vw, tw, sw = xs0.copy(), v0.copy(), t0.copy(), np.zeros(n, np.uint8)
    try:
        for k in (1, 1, 1, 4):
            _check(L.sparsl_net_steps_host(net, hx.a.ctypes.data, hx.a.size, hv.a.ctypes.data, ht.a.ctypes.data, n,
                                           0.95, 0.0, 0.0, k))
            want = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, k)
            trace = np.zeros(k, np.uint32)
            cnt = ctypes.c_uint64()
            _check(L.sparsl_net_trace(net, trace.ctypes.data, k, ctypes.byref(cnt)))
            assert cnt.value == k and np.array_equal(trace, want)
            assert np.array_equal(hx.a, xw)
            assert_bits_equal(hv.a, vw)
            assert_bits_equal(ht.a, tw)
        # Two ticks from the device state, not waited for; then one tick from
        # the host state, which must replace the device state only after them.
        _check(L.sparsl_net_steps_async(net, 0.95, 0.0, 0.0, 2))
        _check(L.sparsl_net_steps_host(net, hx.a.ctypes.data, hx.a.size, hv.a.ctypes.data, ht.a.ctypes.data, n,
                                       0.95, 0.0, 0.0, 1))
        O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, 1)
        assert np.array_equal(hx.a, xw)
        assert_bits_equal(hv.a, vw)
        assert_bits_equal(ht.a, tw)
    finally:
        L.sparsl_net_destroy(net)
        for h in (hx, hv, ht):
            h.free()


def test_workload_generator_matches_its_definition(O, cuda_device):
    """Row r's columns are gen_index(ncols) draws of ChaCha12 seeded with
    seed ^ (r * 0x9E3779B97F4A7C15), sorted -- checked with the oracle's Rng;
    the whole (col, w) block and the LIF state equal the host definition
    (oracle wl_*) bit for bit."""
    L = _lib.load()
    seed, row0, nrows, ncols, fan_in = 0x1234, 77, 300, 1_000_003, 300
    dcol = L.sparsl_device_alloc(cuda_device.handle, nrows * fan_in * 4)
    dw = L.sparsl_device_alloc(cuda_device.handle, nrows * fan_in * 4)
    try:
        _check(L.sparsl_workload_fixed_fanin(seed, row0, nrows, ncols, fan_in, 0.05, dcol, dw, None))
        col = np.zeros(nrows * fan_in, np.uint32)
        w = np.zeros(nrows * fan_in, np.float32)
        _check(L.sparsl_memcpy(col.ctypes.data, dcol, col.nbytes))
        _check(L.sparsl_memcpy(w.ctypes.data, dw, w.nbytes))
    finally:
        L.sparsl_device_free(dcol)
        L.sparsl_device_free(dw)
    for i in range(5):
        r = row0 + i
        rng = O.Rng(seed ^ ((r * 0x9E3779B97F4A7C15) & (2 ** 64 - 1)))
        want = np.sort(np.array([rng.gen_index(ncols) for _ in range(fan_in)], np.uint32))
        assert np.array_equal(col[i * fan_in:(i + 1) * fan_in], want)
    hcol, hw = O.wl_fixed_fanin(seed, row0, nrows, ncols, fan_in, 0.05)
    assert np.array_equal(col, hcol)
    assert_bits_equal(w, hw, "weights vs the host definition")
    assert abs(float(w.std()) - 0.05) < 0.002 and abs(float(w.mean())) < 0.002


@pytest.mark.parametrize("fan_in,ncols", [(1024, 4_194_304), (512, 262_144), (1, 7), (33, 1 << 31)])
def test_workload_generator_bit_identical_to_host(O, cuda_device, fan_in, ncols):
    L = _lib.load()
    seed, row0, nrows = 0x5EED0005, 2_097_152 - 40, 96
    n = nrows * fan_in
    dcol = L.sparsl_device_alloc(cuda_device.handle, n * 4)
    dw = L.sparsl_device_alloc(cuda_device.handle, n * 4)
    try:
        _check(L.sparsl_workload_fixed_fanin(seed, row0, nrows, ncols, fan_in, 0.03, dcol, dw, None))
        col = np.zeros(n, np.uint32)
        w = np.zeros(n, np.float32)
        _check(L.sparsl_memcpy(col.ctypes.data, dcol, col.nbytes))
        _check(L.sparsl_memcpy(w.ctypes.data, dw, w.nbytes))
    finally:
        L.sparsl_device_free(dcol)
        L.sparsl_device_free(dw)
    hcol, hw = O.wl_fixed_fanin(seed, row0, nrows, ncols, fan_in, 0.03)
    assert np.array_equal(col, hcol)
    assert_bits_equal(w, hw, "weights")


def test_lif_state_generator_bit_identical_to_host(O, cuda_device):
    L = _lib.load()
    seed, cell0, n = 0x5EED0005 ^ 0x57A7E, 64, 100_000
    dv = L.sparsl_device_alloc(cuda_device.handle, n * 4)
    dt = L.sparsl_device_alloc(cuda_device.handle, n * 4)
    dp = L.sparsl_device_alloc(cuda_device.handle, (n + 31) // 32 * 4)
    try:
        _check(L.sparsl_workload_lif_state(seed, cell0, n, 0.0, 1.0, 1.0, 0.01, dv, dt, dp, None))
        v, t = np.zeros(n, np.float32), np.zeros(n, np.float32)
        pk = np.zeros((n + 31) // 32, np.uint32)
        for h, d in ((v, dv), (t, dt), (pk, dp)):
            _check(L.sparsl_memcpy(h.ctypes.data, d, h.nbytes))
    finally:
        for d in (dv, dt, dp):
            L.sparsl_device_free(d)
    hv, ht, hs = O.wl_lif_state(seed, cell0, n, 0.0, 1.0, 1.0, 0.01)
    assert_bits_equal(v, hv, "v")
    assert_bits_equal(t, ht, "theta")
    assert np.array_equal(pk, O.pack_spikes(hs))

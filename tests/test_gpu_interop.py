"""Zero-copy interop: caller device buffers bound as an operator's x / y and
CUDA-event handoff, the CUDA analogue of bind_mtl_x / bind_mtl_y /
wait_shared_event / signal_shared_event (src/backend/mod.rs:1975-2098,
metal.rs:1805-1955).  Results stay bit-identical to the oracle."""
import numpy as np
import pytest
import torch

from conftest import assert_bits_equal

import sparsl_b200 as S

pytestmark = pytest.mark.gpu

PARAMS = S.LifParams.new(0.9, 0.0, 0.1)


def _setup(O, seed=0xB1D, nrows=3000, ncols=2000, deg=40):
    rng = O.Rng(seed)
    csr = O.random_csr(nrows, ncols, deg, rng)
    w = O.random_vec(csr.nnz, 1.0, rng)
    x = O.random_vec(ncols, 1.0, rng)
    y0 = O.random_vec(nrows, 1.0, rng)
    return csr, w, x, y0


def _op(dev, csr, w):
    return dev.prepare(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w)


def test_bound_x_replaces_the_slice(O, cuda_device):
    csr, w, x, y0 = _setup(O)
    op = _op(cuda_device, csr, w)
    dx = torch.from_numpy(x).cuda()
    op.bind_cuda_x(dx)
    assert op.cuda_x_gpu_address() == dx.data_ptr()
    y = y0.copy()
    op.spmv(np.zeros_like(x), y)  # the slice is ignored while x is bound
    assert_bits_equal(y, O.spmv(csr, w, x, y0.copy()), "bound x")
    op.unbind_cuda_x()
    assert op.cuda_x_gpu_address() != dx.data_ptr()
    y = y0.copy()
    op.spmv(np.zeros_like(x), y)
    assert_bits_equal(y, y0, "unbound: the zero slice is used again")


def test_bound_y_accumulates_in_place(O, cuda_device):
    csr, w, x, y0 = _setup(O, 0xB1E)
    op = _op(cuda_device, csr, w)
    dy = torch.from_numpy(y0.copy()).cuda()
    op.bind_cuda_y(dy)
    host_y = np.zeros_like(y0)
    op.spmv(x, host_y)
    want = O.spmv(csr, w, x, y0.copy())
    torch.cuda.synchronize()
    assert_bits_equal(dy.cpu().numpy(), want, "bound y on the device")
    assert_bits_equal(host_y, want, "bound y copied to the slice")
    # resident: x and y both bound; sync_y reads the bound y
    dx = torch.from_numpy(x).cuda()
    op.bind_cuda_x(dx)
    op.spmv_resident()
    out = np.zeros_like(y0)
    op.sync_y(out)
    assert_bits_equal(out, O.spmv(csr, w, x, want.copy()), "resident with bound x and y")


def test_writes_refused_while_bound(O, cuda_device):
    csr, w, x, y0 = _setup(O, 0xB1F, 64, 64, 8)
    op = _op(cuda_device, csr, w)
    buf = op.alloc_cuda_f32(x)
    assert np.array_equal(buf.to_numpy(), x)
    op.bind_cuda_x(buf)
    with pytest.raises(S.OpError) as ei:
        op.write_x(x)
    assert ei.value.kind == "Backend" and "unbind first" in str(ei.value)
    ybuf = op.alloc_cuda_f32(y0)
    op.bind_cuda_y(ybuf)
    with pytest.raises(S.OpError) as ei:
        op.write_y(y0)
    assert ei.value.kind == "Backend"
    op.unbind_cuda_x()
    op.unbind_cuda_y()
    op.write_x(x)
    op.write_y(y0)
    buf.free()
    ybuf.free()


def test_fused_lif_reads_bound_x(O, cuda_device):
    csr, w, x, _ = _setup(O, 0xB20, 500, 500, 30)
    op = _op(cuda_device, csr, w)
    dx = torch.from_numpy(x).cuda()
    op.bind_cuda_x(dx)
    v = O.random_vec(500, 0.5, O.Rng(1))
    th = np.abs(O.random_vec(500, 0.5, O.Rng(2)))
    sp = np.zeros(500, np.bool_)
    vv, tt = v.copy(), th.copy()
    op.fused_spmv_lif(np.zeros_like(x), vv, tt, sp, PARAMS)
    wv, wt, ws = v.copy(), th.copy(), np.zeros(500, np.uint8)
    O.fused_lif(csr, w, x, wv, wt, ws, 0.9, 0.0, 0.1)
    assert_bits_equal(vv, wv, "v")
    assert_bits_equal(tt, wt, "theta")
    assert np.array_equal(sp.astype(np.uint8), ws)


def test_bind_checks(O, cuda_device):
    """validate_external_vec (metal.rs:1805-1832): too short -> Length, not
    this GPU's memory -> Backend."""
    rp = np.array([0, 2, 3], np.uint32)
    col = np.array([5, 999_999, 7], np.uint32)
    op = cuda_device.prepare(S.Csr(rp, col, 1_000_000), 1_000_000, np.ones(3, np.float32))
    raw = op.alloc_cuda_f32(np.zeros(1000, np.float32))  # 4 KB: far short of 1M f32
    with pytest.raises(S.OpError) as ei:
        op.bind_cuda_x(raw)
    assert ei.value.kind == "Length"
    host = np.zeros(4, np.float32)

    class HostPtr:
        def data_ptr(self):
            return host.ctypes.data

    with pytest.raises(S.OpError) as ei:
        op.bind_cuda_y(HostPtr())
    assert ei.value.kind == "Backend"
    big = torch.zeros(1_000_000, dtype=torch.float32, device="cuda")
    big[5], big[7], big[999_999] = 1.0, 2.0, 4.0
    op.bind_cuda_x(big)
    y = np.zeros(2, np.float32)
    op.spmv(np.zeros(1_000_000, np.float32), y)
    assert y.tolist() == [5.0, 2.0]
    raw.free()


def test_event_handoff(O, cuda_device):
    csr, w, x, y0 = _setup(O, 0xB22)
    op = _op(cuda_device, csr, w)
    src = torch.from_numpy(x).cuda()
    torch.cuda.synchronize()
    # A peer (torch) produces x on its own stream, after a bounded busy
    # kernel of about 50 ms, then records an event.  Everything the peer
    # needs is allocated first: an allocation inside the block could make
    # the host wait for the busy kernel before the wait below is tried.
    peer = torch.cuda.Stream()
    done = torch.cuda.Event()
    dx = torch.empty_like(src)
    done.record(peer)  # creates the event before the busy kernel
    torch.cuda.synchronize()
    with torch.cuda.stream(peer):
        torch.cuda._sleep(100_000_000)
        dx.copy_(src)
        done.record(peer)
    with pytest.raises(S.OpError) as ei:
        op.wait_cuda_event(done, 0)  # not complete yet: the bounded wait runs out
    assert ei.value.kind == "Execution"
    op.wait_cuda_event(done, 10_000)
    op.bind_cuda_x(dx)
    op.spmv_resident()
    # The operator signals; the peer waits for it before reading y.
    ready = torch.cuda.Event()
    ready.record(peer)  # creates the event
    op.signal_cuda_event(ready)
    ready.synchronize()
    out = np.zeros_like(y0)
    op.sync_y(out)
    assert_bits_equal(out, O.spmv(csr, w, x, np.zeros_like(y0)), "after handoff")
    op.wait_cuda_event(None, 0)  # nothing to wait for

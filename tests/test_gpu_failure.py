"""Failure detection on the GPU, in forms that neither fault nor hang it.

The library follows the reference's fail-closed contract
(src/backend/metal.rs:346-445, Device::reset_metal mod.rs:825-843):

* a host-facing wait that runs past its deadline quarantines the backend,
  and every new call is refused with ``Backend`` until ``sparsl_device_reset``;
* the reset is refused while a call is admitted or while the dispatch that
  timed out is still running on the GPU;
* every device-side spin has an iteration cap: when it runs out the kernel
  records a bit in the device error word and returns, and the call reports
  ``Execution`` with the device still usable;
* an overwritten canary tail is reported as ``Execution``.

The slow dispatch is a bounded busy kernel (``torch.cuda._sleep``, about half
a second) that the operator's stream is made to wait behind; the expired
device wait is a look-back over a predecessor that never publishes, which the
spin cap ends after about 0.1 s.  Nothing here faults, traps or hangs a GPU.
"""
import time

import numpy as np
import pytest
import torch

from conftest import assert_bits_equal

import sparsl_b200 as S
from sparsl_b200 import _lib

pytestmark = pytest.mark.gpu

SLEEP_CYCLES = 1_000_000_000  # ~0.5 s at 1.9 GHz, longer at lower clocks


def _reset_when_idle(limit_s=30.0):
    """Poll sparsl_device_reset until the timed-out work has drained."""
    L = _lib.load()
    t0 = time.time()
    while L.sparsl_device_reset() != 0:
        assert time.time() - t0 < limit_s, "reset still refused: " + _lib.last_error()
        time.sleep(0.02)


@pytest.fixture
def restore_backend():
    L = _lib.load()
    yield
    torch.cuda.synchronize()
    _reset_when_idle()
    L.sparsl_set_timeout_ms(60000)
    assert L.sparsl_quarantined() == 0


def _small_op(O, dev, seed):
    rng = O.Rng(seed)
    csr = O.random_csr(500, 400, 20, rng)
    w = O.random_vec(csr.nnz, 1.0, rng)
    x = O.random_vec(400, 1.0, rng)
    op = dev.prepare(S.Csr(csr.row_ptr, csr.col, csr.ncols), csr.ncols, w)
    return op, csr, w, x


def test_timeout_quarantines_until_the_timed_out_dispatch_completes(O, cuda_device, restore_backend):
    L = _lib.load()
    op, csr, w, x = _small_op(O, cuda_device, 0xFA11)
    y = np.zeros(500, np.float32)
    op.spmv(x, y)  # warm: the operator works
    # A peer stream runs a bounded busy kernel, then records `done`.  The
    # operator's stream is made to wait for `done` on the device; the host
    # side of that wait is given no time and reports Execution (this alone
    # does not quarantine: nothing of the operator's own work timed out).
    peer = torch.cuda.Stream()
    done = torch.cuda.Event()
    done.record(peer)
    torch.cuda.synchronize()
    with torch.cuda.stream(peer):
        torch.cuda._sleep(SLEEP_CYCLES)
        done.record(peer)
    with pytest.raises(S.OpError) as ei:
        op.wait_cuda_event(done, 0)
    assert ei.value.kind == "Execution"
    assert L.sparsl_quarantined() == 0
    # The operator's next wait runs out behind the busy kernel.
    L.sparsl_set_timeout_ms(20)
    rc = L.sparsl_op_wait(op.handle)
    assert rc == _lib.SPARSL_ERR_EXECUTION, _lib.last_error()
    assert "quarantined" in _lib.last_error()
    assert L.sparsl_quarantined() == 1
    # Every new call is refused, on any operator or device entry point.
    with pytest.raises(S.OpError) as ei:
        op.spmv(x, y)
    assert ei.value.kind == "Backend" and "quarantined" in str(ei.value)
    with pytest.raises(S.OpError) as ei:
        cuda_device.assoc_scan(np.ones((4, 2), np.float32))
    assert ei.value.kind == "Backend"
    assert L.sparsl_cuda_probe(None) == _lib.SPARSL_ERR_BACKEND
    # The reset is refused while the timed-out dispatch is still running.
    assert not done.query(), "the busy kernel finished too early for this test"
    assert L.sparsl_device_reset() == _lib.SPARSL_ERR_BACKEND
    assert "timed out" in _lib.last_error()
    assert L.sparsl_quarantined() == 1
    # Once it has drained, the reset clears the quarantine and work resumes.
    done.synchronize()
    _reset_when_idle()
    L.sparsl_set_timeout_ms(60000)
    assert L.sparsl_quarantined() == 0
    y = np.zeros(500, np.float32)
    op.spmv(x, y)
    assert_bits_equal(y, O.spmv(csr, w, x, np.zeros(500, np.float32)), "after reset")


def test_expired_device_wait_reports_execution_and_leaves_the_device_usable(O, cuda_device, restore_backend):
    L = _lib.load()
    t0 = time.time()
    rc = L.sparsl_dev_test_expired_wait(cuda_device.handle)
    dt = time.time() - t0
    assert rc == _lib.SPARSL_ERR_EXECUTION
    assert "bounded look-back wait expired" in _lib.last_error()
    assert dt < 10.0
    assert L.sparsl_quarantined() == 0
    # The error word was cleared and the context is intact.
    xs = np.random.default_rng(5).standard_normal((10_000, 2)).astype(np.float32)
    xs[:, 0] = np.abs(xs[:, 0]) * 0.1 + 0.9
    assert np.array_equal(cuda_device.assoc_scan(xs).view(np.uint32), O.scan_sequential(xs).view(np.uint32))
    op, csr, w, x = _small_op(O, cuda_device, 0xFA12)
    y = np.zeros(500, np.float32)
    op.spmv(x, y)
    assert_bits_equal(y, O.spmv(csr, w, x, np.zeros(500, np.float32)), "after the expired wait")


def test_overwritten_canary_is_reported(O, cuda_device, restore_backend):
    L = _lib.load()
    op, csr, w, x = _small_op(O, cuda_device, 0xFA13)
    y = np.zeros(500, np.float32)
    op.spmv(x, y)
    assert L.sparsl_op_test_mark_canary(op.handle) == _lib.SPARSL_ERR_EXECUTION
    assert "canary" in _lib.last_error()
    # The tail stays marked: the next dispatch on this operator reports it too.
    with pytest.raises(S.OpError) as ei:
        op.spmv(x, y)
    assert ei.value.kind == "Execution" and "canary" in str(ei.value)
    # Other operators are unaffected.
    op2, csr2, w2, x2 = _small_op(O, cuda_device, 0xFA14)
    y2 = np.zeros(500, np.float32)
    op2.spmv(x2, y2)
    assert_bits_equal(y2, O.spmv(csr2, w2, x2, np.zeros(500, np.float32)), "another operator")

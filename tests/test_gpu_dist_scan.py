"""The pieces of the sharded exact scan on the GPU (scan with an entry
state, serial fold, rejoin) against the oracle's sequential fold
(src/scan.rs:298-313), and the whole sharded driver with P runs emulated as
threads on one GPU (one run per thread, the boundary exchange through
shared memory instead of a process group)."""
import threading

import numpy as np
import pytest
import torch

from test_dist_scan_cpu import _comb, _data

from sparsl_b200 import dist_scan

pytestmark = pytest.mark.gpu


def _seq(O, x, entry=None):
    x2 = x.copy()
    if entry is not None:
        x2[0] = _comb(entry, x[0])
    return O.scan_sequential(x2)


@pytest.mark.parametrize("n", [1, 2, 4095, 4096, 4097, 100_003])
def test_scan_from_entry(O, cuda_device, n):
    x = _data("contracting", n)
    entry = np.array([0.5, -2.25], np.float32)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    cuda_device.assoc_scan_from_device(dx, n, dy, entry)
    cuda_device.wait()
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), _seq(O, x, entry).view(np.uint32))
    cuda_device.assoc_scan_from_device(dx, n, dy, None)
    cuda_device.wait()
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), _seq(O, x).view(np.uint32))


def test_table_and_settle(O, cuda_device):
    from test_dist_scan_cpu import OracleRun

    for kind, n in (("contracting", 50_000), ("contracting", 3), ("flat", 1000)):
        x = _data(kind, n)
        dx = torch.from_numpy(x).cuda()
        ref = OracleRun(O, x)
        for k in (0, 1, n // 3):
            got = cuda_device.scan_table_device(dx[k:], n - k)
            assert got == ref.table(k), (kind, n, k, hex(got), hex(ref.table(k)))
        a, i = cuda_device.scan_settle_device(dx, n)
        ra, ri = ref.settle()
        assert i == ri and np.float32(a).view(np.uint32) == np.float32(ra).view(np.uint32)


def test_fold_and_rejoin(O, cuda_device):
    n = 20_000
    x = _data("contracting", n)
    dx = torch.from_numpy(x).cuda()
    st = cuda_device.scan_fold_device(dx, n)
    assert np.array_equal(st.view(np.uint32), _seq(O, x)[-1].view(np.uint32))
    e = np.array([2.0, 7.0], np.float32)
    st = cuda_device.scan_fold_device(dx, n, e)
    assert np.array_equal(st.view(np.uint32), _seq(O, x, e)[-1].view(np.uint32))
    # Rejoin: the stored run was computed from a wrong entry.
    dy = torch.empty_like(dx)
    cuda_device.assoc_scan_from_device(dx, n, dy, np.array([1.0, 0.0], np.float32))
    cuda_device.wait()
    ex, k = cuda_device.scan_rejoin_device(dx, dy, n, e)
    want = _seq(O, x, e)
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert 0 < k < n and np.array_equal(ex.view(np.uint32), want[-1].view(np.uint32))
    # Nothing to rewrite when the run is already exact.
    ex, k = cuda_device.scan_rejoin_device(dx, dy, n, e)
    assert k == 0


class _Gather:
    def __init__(self, world):
        self.world = world
        self.bar = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def for_rank(self, r):
        def gather(a):
            self.slots[r] = np.array(a, np.float32, copy=True)
            self.bar.wait()
            out = [s.copy() for s in self.slots]
            self.bar.wait()
            return out

        return gather


class _PlantedRun(dist_scan.DeviceRun):
    def fold(self, prefix):
        return super().fold(prefix) + np.float32(1.0)


@pytest.mark.parametrize("world,kind,n,plant,halo", [
    (4, "contracting", (1 << 22) + 12_345, -1, 2048),
    (3, "contracting", 300_000, 1, 2048),
    (3, "flat", 5_000, -1, 256),
])
def test_sharded_driver_on_one_gpu(O, cuda_device, world, kind, n, plant, halo):
    x = _data(kind, n)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    torch.cuda.synchronize()
    g = _Gather(world)
    stats, errs = [None] * world, []

    def rank_main(r):
        try:
            lo, hi = r * n // world, (r + 1) * n // world
            cls = _PlantedRun if r == plant else dist_scan.DeviceRun
            run = cls(cuda_device, dx[lo:hi], dy[lo:hi], hi - lo)
            stats[r] = dist_scan.sharded_scan(run, r, world, g.for_rank(r), halo=halo)
        except Exception as e:  # noqa: BLE001
            errs.append(e)
            g.bar.abort()

    th = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    assert not errs, errs
    cuda_device.wait()
    want = O.scan_sequential(x)
    got = dy.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert len({s.rounds for s in stats}) == 1
    if plant >= 0:
        assert stats[plant].rewritten > 0
    elif kind == "contracting":
        assert all(s.entry_exact for s in stats) and stats[0].rounds == 0


class _DevGather:
    """all_gather_dev for threads sharing one GPU: every rank's tensor is
    stacked on the caller's current stream (all are on the device's stream,
    in enqueue order)."""

    def __init__(self, world):
        self.bar = threading.Barrier(world, timeout=120)
        self.slots = [None] * world

    def for_rank(self, r):
        def gather(t):
            self.slots[r] = t
            self.bar.wait()
            out = torch.stack(self.slots)
            self.bar.wait()
            return out

        return gather


@pytest.mark.parametrize("world,kind,n,halo", [
    (4, "contracting", (1 << 22) + 12_345, 2048),
    (3, "contracting", 3_000, 2048),        # short runs: the halo spans several runs, the whole prefix
    (3, "flat", 5_000, 256),                # no contraction: guesses off, host rejoin rounds
])
def test_device_pipeline_on_one_gpu(O, cuda_device, world, kind, n, halo):
    x = _data(kind, n)
    dx = torch.from_numpy(x).cuda()
    dy = torch.empty_like(dx)
    torch.cuda.synchronize()
    g = _DevGather(world)
    stats, errs = [None] * world, []

    def rank_main(r):
        try:
            lo, hi = r * n // world, (r + 1) * n // world
            stats[r] = dist_scan.sharded_scan_device(cuda_device, dx[lo:hi], dy[lo:hi], hi - lo, r, world,
                                                     g.for_rank(r), halo=halo)
        except Exception as e:  # noqa: BLE001
            errs.append(e)
            g.bar.abort()

    th = [threading.Thread(target=rank_main, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join(timeout=300)
    assert not errs, errs
    cuda_device.wait()
    torch.cuda.synchronize()
    want = O.scan_sequential(x)
    assert np.array_equal(dy.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert len({s.rounds for s in stats}) == 1
    if kind == "contracting":
        assert all(s.entry_exact for s in stats) and stats[0].rounds == 0
    else:
        assert stats[0].rounds >= 1

"""The network tick across two GPUs, one process per GPU, as bench.py runs it.

Each rank prepares the row blocks of its half of a recurrent network and the
ranks exchange the spike vector after every tick: by default through peer
memory (the TMA tick kernel stores its packed words straight into the other
GPU's copy, a small kernel publishes a flag and the count and waits for the
peer's), or through an in-place ncclAllGather.  Both must give the oracle's
recurrent ticks bit for bit: the global spike trace, every rank's membrane
and threshold, and the final spike vector.

A last test lets one rank skip its ticks: the other rank's bounded wait for
the peer's flag runs out, the device error word records it and the call
reports Execution -- nothing hangs.  NVLS is off (NCCL_NVLS_ENABLE=0) and the
kernels use plain peer stores, no multicast.

Needs two GPUs; skipped otherwise.
"""
import ctypes
import os
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

N_GPUS = 2


def _gpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


needs_two = pytest.mark.skipif(_gpus() < N_GPUS, reason="needs two GPUs")


def _network(kind):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    n = 8192
    if kind == "uniform":  # TMA path: the tick kernel pushes its words
        col, w = O.wl_fixed_fanin(0xD1, 0, n, n, 96, 0.35)
        rp = (np.arange(n + 1, dtype=np.uint64) * 96).astype(np.uint32)
    else:  # power-law rows: the generic engine, the exchange step pushes
        r = np.random.default_rng(7)
        lens = np.minimum(r.zipf(1.5, n), 900)
        rp = np.zeros(n + 1, np.uint64)
        np.cumsum(lens, out=rp[1:])
        col = np.concatenate([np.sort(r.choice(n, k, replace=False)) for k in lens]).astype(np.uint32)
        rp = rp.astype(np.uint32)
        w = (r.standard_normal(col.size) * 0.3).astype(np.float32)
    v0, t0, s0 = O.wl_lif_state(0xD2, 0, n, 0.0, 1.0, 0.6, 0.05)
    return O, n, rp, col, w, v0, t0, O.pack_spikes(s0)


def _rank(rank, kind, mode, steps, skip_rank, q_id, q_out, q_done, via_host=False):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, ROOT)
    import torch

    import sparsl_b200 as S
    from sparsl_b200 import _lib

    torch.cuda.set_device(rank)
    L = _lib.load()
    res = {"rank": rank}
    try:
        dev = S.Device.try_new(S.Backend.Cuda, rank)
        O, n, rp, col, w, v0, t0, xs0 = _network(kind)
        local = n // N_GPUS
        r0 = rank * local
        # two row blocks per rank
        ops = []
        for a, b in ((r0, r0 + local // 2), (r0 + local // 2, r0 + local)):
            brp = (rp[a:b + 1] - rp[a]).astype(np.uint32)
            ops.append(dev.prepare(S.Csr(brp, col[rp[a]:rp[b]], n), n, w[rp[a]:rp[b]]))
        buf = (ctypes.c_uint8 * 128)()
        if rank == 0:
            assert L.sparsl_nccl_unique_id(buf) == 0, _lib.last_error()
            for _ in range(N_GPUS - 1):
                q_id.put(bytes(buf))
        else:
            buf = (ctypes.c_uint8 * 128).from_buffer_copy(q_id.get(timeout=120))
        arr = (ctypes.c_void_p * len(ops))(*[op.handle.value for op in ops])
        h = ctypes.c_void_p()
        assert L.sparsl_net_create(dev.handle, arr, len(ops), r0, n, rank, N_GPUS, buf, ctypes.byref(h)) == 0, \
            _lib.last_error()
        try:
            assert L.sparsl_net_set_exchange(h, mode) == 0
            vl, tl = v0[r0:r0 + local].copy(), t0[r0:r0 + local].copy()
            assert L.sparsl_net_write_state(h, xs0.ctypes.data, xs0.size, vl.ctypes.data, tl.ctypes.data, local) == 0
            if rank == skip_rank:
                res["skipped"] = True
            elif via_host:
                # The same ticks as calls of sparsl_net_steps_host, the state
                # going through host buffers between calls: pinned buffers
                # (read and written by the tick kernels over PCIe) or
                # pageable ones (copied on the copy streams).
                xs, trace, rc = xs0.copy(), [], 0
                if via_host == "pinned":
                    pins = [L.sparsl_host_alloc(local * 4) for _ in range(2)]
                    hv, ht = (np.frombuffer((ctypes.c_char * (local * 4)).from_address(q), np.float32, local)
                              for q in pins)
                    hv[:], ht[:] = vl, tl
                    vl, tl = hv, ht
                for k in (1, 2, steps - 3):
                    rc = L.sparsl_net_steps_host(h, xs.ctypes.data, xs.size, vl.ctypes.data, tl.ctypes.data, local,
                                                 0.95, 0.0, 0.0, k)
                    if rc:
                        break
                    tr = np.zeros(k, np.uint32)
                    cnt = ctypes.c_uint64()
                    assert L.sparsl_net_trace(h, tr.ctypes.data, k, ctypes.byref(cnt)) == 0
                    trace += tr.tolist()
                res["rc"] = rc
                res["err"] = _lib.last_error() if rc else ""
                res.update(trace=trace, v=vl.tobytes(), t=tl.tobytes(), xs=xs.tobytes())
                if via_host == "pinned":
                    for q in pins:
                        L.sparsl_host_free(q)
            else:
                if skip_rank is not None:
                    L.sparsl_set_timeout_ms(3000)
                rc = L.sparsl_net_steps(h, 0.95, 0.0, 0.0, steps)
                res["rc"] = rc
                res["err"] = _lib.last_error() if rc else ""
                if rc == 0:
                    trace = np.zeros(steps, np.uint32)
                    cnt = ctypes.c_uint64()
                    assert L.sparsl_net_trace(h, trace.ctypes.data, steps, ctypes.byref(cnt)) == 0
                    xs = np.zeros_like(xs0)
                    v, t = np.zeros(local, np.float32), np.zeros(local, np.float32)
                    assert L.sparsl_net_read_state(h, xs.ctypes.data, xs.size, v.ctypes.data, t.ctypes.data,
                                                   local) == 0
                    res.update(trace=trace.tolist(), v=v.tobytes(), t=t.tobytes(), xs=xs.tobytes())
            res["quarantined"] = L.sparsl_quarantined()
        finally:
            # A rank that skipped its ticks keeps its memory mapped until the
            # other rank's calls (which store into it) have returned.
            if skip_rank is not None:
                if rank == skip_rank:
                    q_done.get(timeout=120)
                else:
                    q_done.put(True)
            L.sparsl_net_destroy(h)
    except Exception as e:  # reported to the parent
        res["exc"] = repr(e)
    q_out.put(res)


def _run(kind, mode, steps=30, skip_rank=None, via_host=False):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q_id, q_out, q_done = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, kind, mode, steps, skip_rank, q_id, q_out, q_done, via_host))
             for r in range(N_GPUS)]
    for p in procs:
        p.start()
    res = sorted((q_out.get(timeout=300) for _ in procs), key=lambda d: d["rank"])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in res:
        assert "exc" not in r, r["exc"]
    return res


@needs_two
@pytest.mark.parametrize("kind", ["uniform", "power_law"])
@pytest.mark.parametrize("mode", [0, 1], ids=["peer", "nccl"])
@pytest.mark.parametrize("via_host", [None, "pinned", "pageable"], ids=["resident", "host_pinned", "host_pageable"])
def test_two_gpu_ticks_match_the_oracle(O, kind, mode, via_host):
    res = _run(kind, mode, via_host=via_host)
    O_, n, rp, col, w, v0, t0, xs0 = _network(kind)
    v, t, sp, xs = v0.copy(), t0.copy(), np.zeros(n, np.uint8), xs0.copy()
    want = O.recurrent_steps(O.Csr(rp, col, n), w, xs, v, t, sp, 0.95, 0.0, 0.0, 30, par=True)
    assert want.sum() > 0 and want[-1] > 0, "the test network should keep spiking"
    local = n // N_GPUS
    for r in res:
        assert r["rc"] == 0, r["err"]
        assert r["trace"] == want.tolist()
        assert np.frombuffer(r["xs"], np.uint32).tolist() == xs.tolist()
        lo = r["rank"] * local
        assert np.array_equal(np.frombuffer(r["v"], np.uint32), v[lo:lo + local].view(np.uint32))
        assert np.array_equal(np.frombuffer(r["t"], np.uint32), t[lo:lo + local].view(np.uint32))


@needs_two
def test_peer_that_never_ticks_expires_the_bounded_wait():
    res = _run("uniform", 0, steps=3, skip_rank=1)
    r0 = res[0]
    assert r0["rc"] == 2, "the waiting rank must report Execution"
    assert "peer GPU did not publish" in r0["err"]
    assert res[1].get("skipped")

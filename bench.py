#!/usr/bin/env python
"""Benchmark of the sparsl CUDA substrate on B200.

Headline workload (``--workload lif_net``, the default): the recurrent LIF
network tick -- 4,194,304 neurons, fixed fan-in 1,024 (4.29e9 synapses, f32
weights N(0, 0.03^2)), decay 0.95, threshold 1.0, reset 0, Bernoulli(0.01)
initial spikes.  One step is one tick of the whole network: the fused
spike-SpMV + LIF kernel over every row block, the exchange of the packed spike
words across ranks (by default the tick kernel stores them into every peer
GPU's copy over NVLink and one small kernel per tick trades flags and spike
counts; --net-exchange nccl uses an in-place NCCL all-gather instead), and the
global spike count.  Neurons are
row-block sharded over the ranks, so the total work is fixed as N grows
(strong scaling).  Rows are split into operators of at most 2^31 synapses
(u32 offsets), so one GPU holds two blocks.

Inputs are generated on the GPU from seeded ChaCha12 streams (one per row),
resident in HBM before timing; each rank's synapse arrays (34.4 GB / N) far
exceed the 126 MB L2, so no flush is needed between ticks.  Before timing,
every rank copies its blocks to host memory and the first ticks (by default
every warm-up and timed tick, up to --check-ticks) are compared bit for bit
with the oracle's CpuParallel tick over the same arrays: the global spike
trace, each rank's final membrane state and the final spike words.  At N=1
that CPU run over the whole network is also the reported CPU baseline.

``e2e`` is the same tick through the C ABI from host state: every step,
``sparsl_net_steps_host`` takes the spike vector and this rank's membrane
state from pinned host buffers, runs one tick and returns them (the tick
kernels read and write the state over PCIe; the spike vector is copied).

Other workloads (``--workload``): ``spmv`` (100k x 100k, 64 distinct sorted
columns per row), ``scan`` (2^26 affine maps, a ~ U[0.9, 1], b ~ N(0, 1)),
``lif`` (262,144 neurons x fan-in 512, 1000-tick network on one GPU),
``spmm`` (1M x 1M Zipf(1.5) rows clipped to [1, 4096], 64 vectors).

``--impl reference`` times the CPU restatement of the reference crate's
CpuParallel arm (the oracle) on this host's cores: full ticks of the whole
config network, drawn on the host from the workload definition (the same
arrays the GPU arm draws).
"""
from __future__ import annotations

import argparse
import ctypes
import datetime
import faulthandler
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_FALLBACK = {"hbm_gbs": 6650.0}

# Workload constants (see module docstring)
NET_N = 4_194_304
NET_FANIN = 1024
NET_SIGMA = 0.03
NET_DECAY, NET_VRESET, NET_DTHETA = 0.95, 0.0, 0.0
NET_THETA0 = 1.0
NET_DENSITY = 0.01
NET_SEED = 0x5EED_0005
BLOCK_NNZ_MAX = 1 << 31
# Tick-kernel DRAM traffic per algorithmic byte, from an ncu capture of
# ell_stream_kernel (f32 weights, spike bitmask through the shared-memory
# summary, LIF epilogue) at 1,048,576 x 1,024: dram__bytes_read.sum +
# dram__bytes_write.sum of one launch (8,599,327,488 + 8,067,072 B) over the
# launch's algorithmic bytes (8,606,973,956 B).
NET_TRAFFIC_RATIO = 8_607_394_560 / 8_606_973_956
NET_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of the same kernel and spike mode at "
                      "1,048,576 x 1,024 (8.6 GB streamed), per algorithmic byte, scaled to this launch")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


# DRAM traffic per algorithmic byte of each workload's dominant kernel, from
# ncu captures (dram__bytes_read.sum + dram__bytes_write.sum of one launch
# over the launch's algorithmic bytes), keyed by workload.
TRAFFIC_RATIO = {
    "ragged_spmv": ((457_363_456 + 1_466_112) / 408_395_452,
                    "ncu capture of the same launch (bench.py --workload ragged), 1,000,000 rows: the ordered "
                    "copy's tiles are padded to their longest row, and x is gathered from DRAM once"),
    "ragged_tick": ((457_627_904 + 3_647_616) / 408_645_452,
                    "ncu capture of the tick kernel's launches (bench.py --workload ragged): the ordered fold with "
                    "the spike bitmask in shared memory; packing and compaction not counted"),
    "spmv": (39_812_352 / 52_800_004, "ncu capture of the same launch (bench.py --workload spmv): the panel "
                                      "layout's 16-bit panel-relative columns read less than the CSR bytes"),
    "spmv_f16": (27_011_584 / 40_000_004, "ncu capture of the same launch (bench.py --workload spmv), f16 weights"),
    "spmv_t": ((51_352_832 + 18_432) / 52_800_004, "ncu capture of the same launch (bench.py --workload spmv): "
                                                   "the transpose's slices pad each column to its slice's longest"),
    "spmm_f32": (6.2e9 / 1_164_395_452, "ncu capture of the same launch (bench.py --workload spmm): DRAM "
                                        "throughput x duration, about 6.2 GB, mostly X-row gathers"),
    "lif_integrate": ((805_336_832 + 553_707_008) / 1_409_286_144,
                      "ncu capture of the cell-by-cell form of the kernel at the same size"),
}


def roofline(algo_bytes, ms, kernel, key=None):
    """The roofline block of a workload line: algorithmic bytes per launch over
    the launch's event-timed duration, against the measured HBM copy peak."""
    pk_, how = peaks()
    peak = float(pk_.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    achieved = algo_bytes / (ms * 1e-3) / 1e9
    ratio = TRAFFIC_RATIO.get(key)
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": algo_bytes * ratio[0] if ratio else None,
            "traffic_source": ratio[1] if ratio else None, "kernel": kernel, "peak_source": how}


# --------------------------------------------------------------------------
# process plumbing
# --------------------------------------------------------------------------
class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", str(self.rank)))
        self.pg = None
        if self.world > 1:
            import torch.distributed as td

            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            td.init_process_group("gloo", rank=self.rank, world_size=self.world,
                                  timeout=datetime.timedelta(seconds=300))
            self.pg = td

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch

        t = torch.tensor([v], dtype=torch.float64)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def bcast_bytes(self, b: bytes | None) -> bytes:
        if not self.pg:
            return b
        obj = [b]
        self.pg.broadcast_object_list(obj, src=0)
        return obj[0]

    def gather(self, obj):
        if not self.pg:
            return [obj]
        out = [None] * self.world
        self.pg.all_gather_object(out, obj)
        return out

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Clocks:
    """nvidia-smi sampling during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# --------------------------------------------------------------------------
# helpers over the C ABI
# --------------------------------------------------------------------------
def lib():
    from sparsl_b200 import _lib

    return _lib.load()


def check(rc, what):
    if rc != 0:
        from sparsl_b200 import _lib

        raise RuntimeError(f"{what} failed: {_lib.last_error()}")


class DevArray:
    def __init__(self, dev, nbytes):
        self.nbytes = int(nbytes)
        self.ptr = lib().sparsl_device_alloc(dev.handle, self.nbytes)
        if not self.ptr:
            raise MemoryError(f"device allocation of {nbytes} bytes failed")

    def to_host(self, dtype, count):
        out = np.empty(count, dtype)
        if count:
            check(lib().sparsl_memcpy(out.ctypes.data, self.ptr, out.nbytes), "memcpy D2H")
        return out

    def span(self, count):
        """The first `count` 4-byte elements, as the array argument of
        Device.prepare_device."""
        return _Span(self.ptr, int(count))

    def free(self):
        if self.ptr:
            lib().sparsl_device_free(self.ptr)
            self.ptr = None


class _Span:
    def __init__(self, ptr, count):
        self._ptr, self._count = ptr, count

    def data_ptr(self):
        return self._ptr

    def numel(self):
        return self._count

    def element_size(self):
        return 4


class Pinned:
    def __init__(self, dtype, count):
        self.count = int(count)
        nbytes = max(np.dtype(dtype).itemsize * self.count, 16)
        self.ptr = lib().sparsl_host_alloc(nbytes)
        buf = (ctypes.c_char * nbytes).from_address(self.ptr)
        self.a = np.frombuffer(buf, dtype=dtype, count=self.count)

    def free(self):
        lib().sparsl_host_free(self.ptr)


def torch_stream(ptr, device_index):
    import torch

    return torch.cuda.ExternalStream(ptr, device=torch.device("cuda", device_index))


def events_ms(stream_ptr, device_index, fn):
    """Device time of whatever fn enqueues on the stream, by CUDA events."""
    import torch

    s = torch_stream(stream_ptr, device_index)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(s)
    fn()
    b.record(s)
    b.synchronize()
    return a.elapsed_time(b)


# --------------------------------------------------------------------------
# LIF network (headline)
# --------------------------------------------------------------------------
def net_blocks(local_rows, fan_in):
    rows_per = BLOCK_NNZ_MAX // fan_in
    out, r = [], 0
    while r < local_rows:
        n = min(rows_per, local_rows - r)
        out.append((r, n))
        r += n
    return out


def build_lif_net(S, dev, dist, n_total, fan_in, keep_host=False):
    """This rank's row blocks, drawn and prepared on the GPU.  With keep_host
    each block's CSR is also copied to host memory (the arrays the GPU
    operators were prepared from) for the CPU check."""
    world, rank = dist.world, dist.rank
    local = n_total // world
    row0 = rank * local
    import torch

    ops, host = [], []
    t0 = time.time()
    for (off, nrows) in net_blocks(local, fan_in):
        # The synapses are drawn on the GPU and the operator is prepared from
        # them there (validated and copied in HBM; no host round trip).
        nnz = nrows * fan_in
        drp = DevArray(dev, (nrows + 1) * 4)
        dcol = DevArray(dev, nnz * 4)
        dw = DevArray(dev, nnz * 4)
        check(lib().sparsl_workload_uniform_row_ptr(nrows, fan_in, drp.ptr, None), "row_ptr")
        check(lib().sparsl_workload_fixed_fanin(NET_SEED, row0 + off, nrows, n_total, fan_in, NET_SIGMA, dcol.ptr,
                                                dw.ptr, None), "workload")
        torch.cuda.synchronize()
        ops.append(dev.prepare_device(drp.span(nrows + 1), dcol.span(nnz), n_total, dw.span(nnz)))
        if keep_host:
            host.append((drp.to_host(np.uint32, nrows + 1), dcol.to_host(np.uint32, nnz),
                         dw.to_host(np.float32, nnz), row0 + off))
        for a in (drp, dcol, dw):
            a.free()
    # initial state for every cell (the spike vector is global)
    dv = DevArray(dev, n_total * 4)
    dth = DevArray(dev, n_total * 4)
    dpk = DevArray(dev, (n_total // 32) * 4)
    check(lib().sparsl_workload_lif_state(NET_SEED ^ 0x57A7E, 0, n_total, 0.0, 1.0, NET_THETA0, NET_DENSITY, dv.ptr,
                                          dth.ptr, dpk.ptr, None), "state")
    v = dv.to_host(np.float32, n_total)
    th = dth.to_host(np.float32, n_total)
    pk = dpk.to_host(np.uint32, n_total // 32)
    for a in (dv, dth, dpk):
        a.free()
    setup_s = time.time() - t0
    return ops, (row0, local), (v, th, pk), host, setup_s


def make_net(S, dev, dist, ops, row0, n_total):
    L = lib()
    nid = None
    if dist.world > 1:
        buf = (ctypes.c_uint8 * 128)()
        if dist.rank == 0:
            check(L.sparsl_nccl_unique_id(buf), "nccl id")
        nid_bytes = dist.bcast_bytes(bytes(buf) if dist.rank == 0 else None)
        nid = (ctypes.c_uint8 * 128).from_buffer_copy(nid_bytes)
    arr = (ctypes.c_void_p * len(ops))(*[op.handle.value for op in ops])
    h = ctypes.c_void_p()
    check(L.sparsl_net_create(dev.handle, arr, len(ops), row0, n_total, dist.rank, dist.world, nid,
                              ctypes.byref(h)), "net_create")
    return h


def net_bytes_per_tick_per_gpu(n_total, fan_in, world):
    # Algorithmic bytes (per GPU per tick): col + weight per synapse, row
    # offsets, v read+write, theta read, packed spikes in and out.
    local = n_total // world
    return local * fan_in * 8 + (local + 1) * 4 + local * 8 + local * 4 + 2 * (n_total // 8) // world


def _popcount(words):
    return int(np.unpackbits(np.ascontiguousarray(words).view(np.uint8)).sum())


def cpu_net_ticks(O, dist, host, n_total, v, th, pk, ticks):
    """The oracle's CpuParallel fused tick (cpu_fused_spikes_*, mod.rs:2572-2614,
    as recurrent_steps, mod.rs:1889-1932) over this rank's row blocks, `ticks`
    ticks from (v, th, pk).  Ranks exchange their packed spike words after each
    tick over the host process group (gloo), so every rank folds against the
    global spike vector; rows never depend on the split.  Returns the global
    per-tick spike counts, the final local (v, theta), the final global spike
    words and the seconds the ticks took (exchange included)."""
    import torch

    local = v.size
    sp = np.zeros(local, np.uint8)
    csrs = [(O.Csr(rp, col, n_total), w) for (rp, col, w, _) in host]
    trace = []
    t0 = time.perf_counter()
    for _ in range(ticks):
        off = 0
        for csr, w in csrs:
            k = csr.nrows
            O.fused_spikes_lif(csr, w, pk, v[off:off + k], th[off:off + k], sp[off:off + k], NET_DECAY, NET_VRESET,
                               NET_DTHETA, par=True)
            off += k
        words = O.pack_spikes(sp)
        if dist.world > 1:
            mine = torch.from_numpy(words.view(np.int32).copy())
            parts = [torch.empty_like(mine) for _ in range(dist.world)]
            dist.pg.all_gather(parts, mine)
            pk = np.concatenate([t_.numpy().view(np.uint32) for t_ in parts])
        else:
            pk = words
        trace.append(_popcount(pk))
    return np.array(trace, np.uint32), v, th, pk, time.perf_counter() - t0


def bench_lif_net(args, dist):
    import torch
    import sparsl_b200 as S

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    torch.cuda.set_device(dist.local)
    dev = S.Device.try_new(S.Backend.Cuda, dist.local)
    n_total, fan_in = NET_N, NET_FANIN
    check_ticks = 0 if args.no_check else min(args.check_ticks, args.warmup + args.steps)
    ops, (row0, local), (v, th, pk), host, setup_s = build_lif_net(S, dev, dist, n_total, fan_in,
                                                                   keep_host=check_ticks > 0)
    net = make_net(S, dev, dist, ops, row0, n_total)
    L = lib()
    check(L.sparsl_net_set_exchange(net, 1 if args.net_exchange == "nccl" else 0), "exchange mode")
    stream = L.sparsl_net_stream(net)
    p = (NET_DECAY, NET_VRESET, NET_DTHETA)
    v_l, th_l = v[row0:row0 + local].copy(), th[row0:row0 + local].copy()

    # Bit-exact check against the CPU: the first check_ticks ticks from the
    # initial state on the GPU, and the same ticks of the oracle over the same
    # arrays (the ones the operators were prepared from) on the host.  The
    # check covers every tick the timed run below executes (warm-up ticks
    # included) unless --check-ticks caps it.
    chk = None
    if check_ticks:
        O.set_threads(max(1, (os.cpu_count() or 1) // dist.world))
        # The device generator against its host definition, on the first and
        # last 64 rows of every block of this rank.
        gen_ok = True
        for (rp, col, w, r0) in host:
            k = rp.size - 1
            for a in (0, max(0, k - 64)):
                m = min(64, k - a)
                hc, hw = O.wl_fixed_fanin(NET_SEED, r0 + a, m, n_total, fan_in, NET_SIGMA)
                gen_ok &= bool(np.array_equal(col[a * fan_in:(a + m) * fan_in], hc)
                               and np.array_equal(w[a * fan_in:(a + m) * fan_in].view(np.uint32), hw.view(np.uint32)))
        hv, hth, hs = O.wl_lif_state(NET_SEED ^ 0x57A7E, 0, n_total, 0.0, 1.0, NET_THETA0, NET_DENSITY)
        gen_ok &= bool(np.array_equal(hv.view(np.uint32), v.view(np.uint32)) and np.array_equal(O.pack_spikes(hs), pk))
        check(L.sparsl_net_write_state(net, pk.ctypes.data, pk.size, v_l.ctypes.data, th_l.ctypes.data, local),
              "write_state")
        check(L.sparsl_net_steps(net, *p, check_ticks), "check ticks")
        gtrace = np.zeros(check_ticks, np.uint32)
        nn = ctypes.c_uint64()
        check(L.sparsl_net_trace(net, gtrace.ctypes.data, gtrace.size, ctypes.byref(nn)), "trace")
        gpk, gv, gth = np.zeros_like(pk), np.zeros(local, np.float32), np.zeros(local, np.float32)
        check(L.sparsl_net_read_state(net, gpk.ctypes.data, gpk.size, gv.ctypes.data, gth.ctypes.data, local),
              "read_state")
        ctrace, cv, cth, cpk, cpu_s = cpu_net_ticks(O, dist, host, n_total, v_l.copy(), th_l.copy(), pk.copy(),
                                                    check_ticks)
        ok = bool(np.array_equal(gtrace, ctrace) and np.array_equal(gv.view(np.uint32), cv.view(np.uint32))
                  and np.array_equal(gth.view(np.uint32), cth.view(np.uint32)) and np.array_equal(gpk, cpk))
        oks = dist.gather((ok, gen_ok))
        chk = {"ticks": check_ticks, "cpu_s": dist.max(cpu_s), "trace": gtrace,
               "bit_exact_vs_cpu": all(o for o, _ in oks), "generator_matches_host": all(g for _, g in oks)}
        del host
    check(L.sparsl_net_write_state(net, pk.ctypes.data, pk.size, v_l.ctypes.data, th_l.ctypes.data, local),
          "write_state")
    # warm-up (untimed)
    check(L.sparsl_net_steps(net, *p, args.warmup), "warmup")
    wtrace = np.zeros(args.warmup, np.uint32)
    nn = ctypes.c_uint64()
    check(L.sparsl_net_trace(net, wtrace.ctypes.data, wtrace.size, ctypes.byref(nn)), "warm-up trace")
    dist.barrier()
    clocks = Clocks(dist.local)
    if dist.rank == 0:
        clocks.start()
    check(L.sparsl_net_set_timing(net, args.steps), "timing")
    dist.barrier()
    ms = events_ms(stream, dist.local, lambda: check(L.sparsl_net_steps_async(net, *p, args.steps), "steps"))
    check(L.sparsl_net_wait(net), "wait")
    dist.barrier()
    ck = clocks.stop() if dist.rank == 0 else None
    ms_max = dist.max(ms)
    kms = ctypes.c_double()
    kt = ctypes.c_uint64()
    check(L.sparsl_net_kernel_ms(net, ctypes.byref(kms), ctypes.byref(kt)), "kernel ms")
    kernel_ms_tick = kms.value / max(kt.value, 1)
    tick_ms = np.zeros(args.steps, np.float32)
    check(L.sparsl_net_tick_ms(net, tick_ms.ctypes.data, tick_ms.size, ctypes.byref(kt)), "tick ms")
    trace = np.zeros(args.steps, np.uint32)
    n = ctypes.c_uint64()
    check(L.sparsl_net_trace(net, trace.ctypes.data, trace.size, ctypes.byref(n)), "trace")
    traces = dist.gather(trace.tolist())
    consistent = all(t == traces[0] for t in traces)
    full_trace = np.concatenate([wtrace, trace])

    # End to end through the C ABI with pinned host buffers: every step takes
    # the spike vector and this rank's membrane state from the host, runs one
    # tick, and returns them (sparsl_net_steps_host: each block's copies
    # overlap the other block's tick kernel).
    check(L.sparsl_net_set_timing(net, 0), "timing off")
    e2e_steps = max(1, min(args.steps, 20))
    hp = Pinned(np.uint32, pk.size)
    hv = Pinned(np.float32, local)
    ht = Pinned(np.float32, local)
    hp.a[:] = pk
    hv.a[:] = v_l
    ht.a[:] = th_l
    dist.barrier()

    def e2e():
        for _ in range(e2e_steps):
            check(L.sparsl_net_steps_host(net, hp.ptr, hp.count, hv.ptr, ht.ptr, local, *p, 1), "e2e step")

    e2e_ms = dist.max(events_ms(stream, dist.local, e2e))
    h2d = pk.nbytes + 2 * local * 4
    d2h = h2d

    cpu = None
    if chk and dist.world == 1:
        cpu = {"value": chk["ticks"] / chk["cpu_s"], "unit": "ticks/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{chk['ticks']} full ticks of the same {n_total * fan_in:.3g}-synapse network (the "
                         "parity check below), C restatement of the reference's CpuParallel fused tick"}
    # fused tick kernel per block + the exchange step (N>1, peer) or the
    # global spike count (N=1, or after the NCCL all-gather)
    kernels_per_tick = len(ops) + 1
    pk_, how = peaks()
    peak = float(pk_.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    algo = net_bytes_per_tick_per_gpu(n_total, fan_in, dist.world)
    achieved = algo / (kernel_ms_tick * 1e-3) / 1e9
    # DRAM traffic of the tick kernel: dram__bytes_read.sum + dram__bytes_write.sum
    # of one ncu capture of this kernel in this spike mode at 1,048,576 x 1,024
    # (8.6 GB of synapses), per launch, scaled to this launch by its algorithmic
    # bytes (traffic grows with the synapses streamed).
    traffic = algo * NET_TRAFFIC_RATIO
    value = args.steps / (ms_max * 1e-3)
    ts = np.sort(tick_ms)
    line = {
        "metric": "LIF net ticks/sec", "value": value, "unit": "ticks/s", "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded ChaCha12 per row, drawn on the GPU; identical to the host definition)",
        "config": {"workload": f"lif_net: {n_total:,} neurons x fan-in {fan_in} ({n_total * fan_in:.3g} synapses), "
                               "f32 weights N(0,0.03^2), decay 0.95, theta 1.0, reset 0, Bernoulli(0.01) initial spikes",
                   "parallelism": f"row-block shards x{dist.world}" + (
                       "" if dist.world == 1 else
                       (", packed spike words stored by the tick kernel into every peer GPU's copy over NVLink, "
                        "one flag/count kernel per tick" if args.net_exchange == "peer" else
                        ", in-place NCCL all-gather of the packed spike words per tick")),
                   "blocks_per_gpu": len(ops), "l2": "inputs per GPU >> 126 MB L2 (no flush needed)",
                   "setup_s": round(setup_s, 1)},
        "clocks": ck,
        "e2e": {"value": e2e_steps / (e2e_ms * 1e-3), "unit": "ticks/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h),
                "path": "sparsl_net_steps_host(1): state in, one tick, state out, pinned host; each "
                        "block's copies overlap the other block's tick kernel"},
        "gpu_launches": kernels_per_tick * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "traffic_source": NET_TRAFFIC_SOURCE,
                     "kernel": "ell_stream_kernel<f32, spike bitmask via shared-memory summary, LIF> "
                               "(TMA-streamed fused spike SpMV + LIF + ballot pack)",
                     "algorithmic_bytes_per_tick_per_gpu": algo, "kernel_ms_per_tick": kernel_ms_tick,
                     "kernel_ms_per_tick_min_median_max": [float(ts[0]), float(ts[len(ts) // 2]), float(ts[-1])],
                     "kernel_ms_first_ticks": [round(float(x), 4) for x in tick_ms[:4]],
                     "peak_source": how},
        "cpu_baseline": cpu,
        "check": {"spike_trace_sum": int(trace.sum()), "trace_identical_on_all_ranks": consistent,
                  "trace_sha1": __import__("hashlib").sha1(trace.tobytes()).hexdigest()[:16],
                  "trace_head": trace[:8].tolist(),
                  f"trace_sha1_first_{full_trace.size}_ticks": __import__("hashlib").sha1(
                      full_trace.tobytes()).hexdigest()[:16]},
    }
    if chk:
        k = chk["ticks"]
        line["check"].update({
            "cpu_check_ticks": k, "bit_exact_vs_cpu": chk["bit_exact_vs_cpu"],
            "cpu_check_scope": "global spike trace, every rank's final v and theta, final global spike words, "
                               "after the first ticks from the initial state (warm-up and timed ticks)",
            "timed_trace_equals_checked_ticks": bool(np.array_equal(full_trace[:k], chk["trace"][:full_trace.size])),
            "device_generator_matches_host_definition": chk["generator_matches_host"],
            "cpu_check_s": round(chk["cpu_s"], 1)})
    for h in (hp, hv, ht):
        h.free()
    L.sparsl_net_destroy(net)
    del ops
    return line


# --------------------------------------------------------------------------
# single-kernel workloads (configs 1-3)
# --------------------------------------------------------------------------
SPMV_N, SPMV_DEG, SPMV_SEED = 100_000, 64, 0x5B11
SCAN_N, SCAN_SEED = 1 << 26, 0x5CA2
LIF_N, LIF_FANIN, LIF_SIGMA, LIF_DENSITY, LIF_SEED = 262_144, 512, 0.05, 0.02, 0x11F3


def gen_distinct_rows(rng, nrows, ncols, deg):
    """deg distinct sorted columns per row (rejection of repeats)."""
    out = np.empty((nrows, deg), np.uint32)
    todo = np.arange(nrows)
    while todo.size:
        cand = np.sort(rng.integers(0, ncols, size=(todo.size, deg + 16), dtype=np.uint32), axis=1)
        dup = np.zeros_like(cand, dtype=bool)
        dup[:, 1:] = cand[:, 1:] == cand[:, :-1]
        key = np.where(dup, np.uint32(0xFFFFFFFF), cand)
        key.sort(axis=1)
        good = key[:, deg - 1] != 0xFFFFFFFF
        out[todo[good]] = key[good, :deg]
        todo = todo[~good]
    return out.reshape(-1)


def flush_l2(buf):
    """Evict the operands from L2: write a buffer 8x the L2, then read it back,
    so the L2 holds clean lines of that buffer.  (A write alone leaves the L2
    full of dirty lines whose write-back to DRAM would then be charged to the
    timed kernel.)  Neither step is timed."""
    buf.zero_()
    buf.sum()


def time_launches(stream, fn, k, flush=None):
    """Per-launch device time (ms) of fn on `stream`, optionally flushing L2 before each."""
    import torch

    ts = []
    for _ in range(k):
        if flush is not None:
            with torch.cuda.stream(stream):
                flush()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn()
        b.record(stream)
        b.synchronize()
        ts.append(a.elapsed_time(b))
    return ts


def bench_spmv(args, dev, want_cpu):
    import torch
    import sparsl_b200 as S

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    r = np.random.default_rng(SPMV_SEED)
    col = gen_distinct_rows(r, SPMV_N, SPMV_N, SPMV_DEG)
    rp = (np.arange(SPMV_N + 1, dtype=np.uint64) * SPMV_DEG).astype(np.uint32)
    w = r.uniform(-1.0, 1.0, col.size).astype(np.float32)
    x = r.uniform(0.0, 1.0, SPMV_N).astype(np.float32)
    op = dev.prepare(S.Csr(rp, col, SPMV_N), SPMV_N, w)
    L = lib()
    s = torch.cuda.Stream()  # a real stream: a NULL handle would mean the operator's own stream
    torch.cuda.set_stream(s)
    dx = torch.from_numpy(x).cuda()
    dy = torch.zeros(SPMV_N, dtype=torch.float32, device="cuda")
    flush = torch.empty(64 << 22, dtype=torch.float32, device="cuda")  # 1 GiB > L2
    run = lambda: check(L.sparsl_op_spmv_device(op.handle, dx.data_ptr(), dy.data_ptr(), s.cuda_stream), "spmv")
    for _ in range(args.warmup):
        run()
    dy.zero_()
    ts = time_launches(s, run, args.kernel_iters, flush=lambda: flush_l2(flush))
    ms = statistics.median(ts)
    algo = col.size * 8 + (SPMV_N + 1) * 4 + SPMV_N * 4 + 2 * SPMV_N * 4
    # bit-exact at full size: y accumulated kernel_iters times from zero vs the oracle doing the same
    import oracle as O

    got = dy.cpu().numpy()
    want = np.zeros(SPMV_N, np.float32)
    csr = O.Csr(rp, col, SPMV_N)
    for _ in range(args.kernel_iters):
        O.spmv(csr, w, x, want, par=True)
    exact = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
    # end to end: the C-ABI slice call with pinned host x and y
    hx, hy = Pinned(np.float32, SPMV_N), Pinned(np.float32, SPMV_N)
    hx.a[:] = x
    hy.a[:] = 0
    ops_stream = L.sparsl_op_stream(op.handle)
    ets = [events_ms(ops_stream, torch.cuda.current_device(),
                     lambda: check(L.sparsl_op_spmv(op.handle, hx.ptr, SPMV_N, hy.ptr, SPMV_N), "spmv e2e"))
           for _ in range(max(3, args.kernel_iters // 2))]
    e2e_ms = statistics.median(ets)
    hx.free()
    hy.free()
    cpu = None
    if want_cpu:
        t0, k = time.perf_counter(), 0
        yy = np.zeros(SPMV_N, np.float32)
        while time.perf_counter() - t0 < args.cpu_seconds / 2:
            O.spmv(csr, w, x, yy, par=True)
            k += 1
        dt = time.perf_counter() - t0
        cpu = {"value": k * algo / dt / 1e9, "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{k} full SpMVs of the same matrix, CpuParallel restatement"}
    # The same matrix with binary16 weights (the half.rs narrow path), and the
    # transpose product over the operator's reverse index; each checked against
    # the oracle after kernel_iters accumulations from zero.
    def measure(op_, fn, xin, ylen, algo_, want_fn):
        dyy = torch.zeros(ylen, dtype=torch.float32, device="cuda")
        run_ = lambda: check(fn(op_.handle, xin.data_ptr(), dyy.data_ptr(), s.cuda_stream), "spmv variant")
        for _ in range(args.warmup):
            run_()
        dyy.zero_()
        ts_ = time_launches(s, run_, args.kernel_iters, flush=lambda: flush_l2(flush))
        ms_ = statistics.median(ts_)
        ref = np.zeros(ylen, np.float32)
        for _ in range(args.kernel_iters):
            want_fn(ref)
        ok_ = bool(np.array_equal(dyy.cpu().numpy().view(np.uint32), ref.view(np.uint32)))
        return {"value": algo_ / (ms_ * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms_, "algorithmic_bytes": algo_,
                "bit_exact_vs_oracle": ok_}, ms_

    op16 = dev.prepare_with(S.Csr(rp, col, SPMV_N), SPMV_N, w, S.WeightPrecision.F16)
    w16 = O.quantise(int(S.WeightPrecision.F16), w)
    algo16 = col.size * 6 + (SPMV_N + 1) * 4 + SPMV_N * 4 + 2 * SPMV_N * 4
    f16, ms16 = measure(op16, L.sparsl_op_spmv_device, dx, SPMV_N, algo16,
                        lambda ref: O.spmv(csr, w16, x, ref, par=True))
    f16["roofline"] = roofline(algo16, ms16, "panel_spmv_kernel<f16 weights, x in shared-memory panels>", "spmv_f16")
    del op16
    opt = dev.prepare_with_transpose(S.Csr(rp, col, SPMV_N), SPMV_N, w)
    xt = r.uniform(0.0, 1.0, SPMV_N).astype(np.float32)
    dxt = torch.from_numpy(xt).cuda()
    csc = O.csc_from_csr(csr, SPMV_N)
    # CSC walk: row index + weight (kept in reverse-index order) per entry, x
    # gathered by row; col_ptr, x and y once.
    algot = col.size * 8 + (SPMV_N + 1) * 4 + SPMV_N * 4 + 2 * SPMV_N * 4
    tr, mst = measure(opt, L.sparsl_op_spmv_t_device, dxt, SPMV_N, algot,
                      lambda ref: O.spmv_t(csc, w, xt, ref, par=True))
    tr["roofline"] = roofline(algot, mst, "panel_spmv_kernel<f32> (transpose: x panels over the sliced-ELL "
                                          "reverse index)", "spmv_t")
    del opt
    # The reverse index itself, built on the GPU from device arrays (gate
    # included; wall clock of the blocking C-ABI call) against the oracle's
    # host counting sort.
    drp, dcol = torch.from_numpy(rp.view(np.int32)).cuda(), torch.from_numpy(col.view(np.int32)).cuda()
    dcp = torch.empty(SPMV_N + 1, dtype=torch.int32, device="cuda")
    drow = torch.empty(col.size, dtype=torch.int32, device="cuda")
    deidx = torch.empty(col.size, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    cts = []
    for _ in range(args.warmup + 5):
        t0 = time.perf_counter()
        dev.csc_from_csr_device(drp, dcol, SPMV_N, dcp, drow, deidx)
        cts.append((time.perf_counter() - t0) * 1e3)
    csc_ms = statistics.median(cts[args.warmup:])
    csc_ok = all(np.array_equal(g.cpu().numpy().view(np.uint32), w_) for g, w_ in zip((dcp, drow, deidx), csc))
    t0 = time.perf_counter()
    O.csc_from_csr(csr, SPMV_N)
    csc_cpu_ms = (time.perf_counter() - t0) * 1e3
    rev = {"ms": csc_ms, "edges_per_s": col.size / (csc_ms * 1e-3), "identical_to_oracle": csc_ok,
           "cpu_ms": csc_cpu_ms, "cpu": "oracle counting sort (sparse.rs:361-427 restated), 1 thread",
           "path": "sparsl_csc_from_csr_device: device gate + 3 radix passes + col_ptr/row"}
    del drp, dcol, dcp, drow, deidx
    return {"metric": "SpMV effective HBM GB/s", "value": algo / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms, "kernel_ms_samples": len(ts), "algorithmic_bytes": algo,
            "config": "100,000 x 100,000, 64 distinct sorted cols/row, w U[-1,1], x U[0,1], f32; L2 flushed "
                      "(1 GiB written, then read back) before every launch",
            "e2e": {"value": algo / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 2 * SPMV_N * 4,
                    "d2h_bytes_per_step": SPMV_N * 4, "path": "sparsl_op_spmv, pinned host x/y"},
            "bit_exact_vs_oracle": exact, "cpu_baseline": cpu,
            "roofline": roofline(algo, ms, "panel_spmv_kernel<f32, x in shared-memory panels>", "spmv"),
            "f16_weights": f16, "transpose": tr, "reverse_index": rev}


def bench_rowshard(args, dev, dist, kind):
    """SpMV (config 1 shape) or SpMM (config 4 shape) sharded by rows with x
    replicated: rank r owns a row block drawn from seed + r (weak scaling, N
    row blocks in all), every rank holds the same x, no exchange.  Each
    rank's kernel is timed by CUDA events with L2 flushed before every
    launch; the step time is the max over ranks of the per-rank median."""
    import torch
    import sparsl_b200 as S

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    L = lib()
    if kind == "spmv":
        n, nv, seed = SPMV_N, 1, SPMV_SEED
        r = np.random.default_rng(seed + dist.rank)
        col = gen_distinct_rows(r, n, n, SPMV_DEG)
        rp = (np.arange(n + 1, dtype=np.uint64) * SPMV_DEG).astype(np.uint32)
        w = r.uniform(-1.0, 1.0, col.size).astype(np.float32)
        x = np.random.default_rng(seed ^ 0x5EED).uniform(0.0, 1.0, n).astype(np.float32)
    else:
        n, nv, seed = SPMM_N, SPMM_NVEC, SPMM_SEED
        rp, col, r = gen_zipf_csr(n, n, SPMM_KMAX, SPMM_ALPHA, seed + dist.rank)
        w = r.uniform(-1.0, 1.0, col.size).astype(np.float32)
        x = np.random.default_rng(seed ^ 0x5EED).uniform(-1.0, 1.0, n * nv).astype(np.float32)
    nnz = col.size
    op = dev.prepare(S.Csr(rp, col, n), n, w)
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    dx = torch.from_numpy(x).cuda()
    dy = torch.zeros(n * nv, dtype=torch.float32, device="cuda")
    flush = torch.empty(64 << 22, dtype=torch.float32, device="cuda")  # 1 GiB > L2
    if kind == "spmv":
        run = lambda: check(L.sparsl_op_spmv_device(op.handle, dx.data_ptr(), dy.data_ptr(), s.cuda_stream), "spmv")
        algo = nnz * 8 + (n + 1) * 4 + n * 4 + 2 * n * 4
    else:
        run = lambda: check(L.sparsl_op_spmm_device(op.handle, dx.data_ptr(), nv, dy.data_ptr(), s.cuda_stream),
                            "spmm")
        algo = nnz * 8 + (n + 1) * 4 + n * nv * 4 + 2 * n * nv * 4
    # parity: one product from y = 0 against the oracle over the whole output
    O.set_threads(max(1, (os.cpu_count() or 1) // dist.world))
    run()
    s.synchronize()
    got = dy.cpu().numpy()
    if kind == "spmv":
        want = O.spmv(O.Csr(rp, col, n), w, x, np.zeros(n, np.float32), par=True)
    else:
        want = O.spmm(O.Csr(rp, col, n), w, x, nv, np.zeros(n * nv, np.float32), par=True)
    exact = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
    del got, want
    for _ in range(args.warmup):
        run()
    dist.barrier()
    clocks = Clocks(dist.local)
    if dist.rank == 0:
        clocks.start()
    dist.barrier()
    ts = time_launches(s, run, args.kernel_iters, flush=lambda: flush_l2(flush))
    dist.barrier()
    ck = clocks.stop() if dist.rank == 0 else None
    ms = dist.max(statistics.median(ts))
    oks = dist.gather(exact)
    if dist.rank != 0:
        return None
    shape = (f"{n:,} x {n:,} per GPU, 64 distinct sorted cols/row" if kind == "spmv" else
             f"{n:,} x {n:,} per GPU, Zipf(1.5) rows in [1,4096], X {n:,} x {nv} row-major")
    return {"metric": f"{'SpMV' if kind == 'spmv' else 'SpMM'} effective HBM GB/s",
            "value": dist.world * algo / (ms * 1e-3) / 1e9, "unit": "GB/s", "n_gpus": dist.world,
            "steps": args.kernel_iters, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, row block per rank)",
            "config": {"workload": f"{kind}: {dist.world} row blocks of {shape}; x replicated",
                       "parallelism": "row blocks, x replicated, no exchange",
                       "l2": "L2 flushed (1 GiB written, then read back) before every launch"},
            "algorithmic_bytes_per_gpu": algo, "clocks": ck, "bit_exact_vs_oracle": all(oks)}


def bench_scan_sharded(args, dev, dist):
    """The exact scan of a sequence split into one run of SCAN_N maps per rank
    (weak scaling: N x SCAN_N maps in all): halo and table all-gather, entry
    guess, local scan, boundary-state check and rejoin rounds
    (sparsl_b200/dist_scan.py; by default the device pipeline: NCCL gathers,
    one host sync).  Each step is timed by CUDA events on the device's
    stream around the whole procedure, host work included;
    the step time is the max over ranks.  Rank r's run is drawn from seed
    SCAN_SEED + r (rank 0's run is exactly the 1-GPU workload)."""
    import torch

    from sparsl_b200 import dist_scan

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    r = np.random.default_rng(SCAN_SEED + dist.rank)
    xs = np.empty((SCAN_N, 2), np.float32)
    xs[:, 0] = r.uniform(0.9, 1.0, SCAN_N).astype(np.float32)
    xs[:, 1] = r.standard_normal(SCAN_N).astype(np.float32)
    din = torch.from_numpy(xs).cuda()
    dout = torch.empty_like(din)
    torch.cuda.synchronize()
    if args.scan_pipeline == "device":
        group = dist.pg.new_group(backend="nccl")
        gather_dev = dist_scan.nccl_all_gather_dev(group, dist.world)
    elif args.scan_exchange == "nccl":
        group = dist.pg.new_group(backend="nccl")
        gather = dist_scan.nccl_all_gather(group, dist.world, torch.device("cuda", dist.local))
    else:
        gather = dist_scan.process_group_all_gather(dist.pg, dist.world)
    run = dist_scan.DeviceRun(dev, din, dout, SCAN_N)
    stream = lib().sparsl_dev_stream(dev.handle)
    st = None

    def step():
        nonlocal st
        if args.scan_pipeline == "device":
            st = dist_scan.sharded_scan_device(dev, din, dout, SCAN_N, dist.rank, dist.world, gather_dev)
        else:
            st = dist_scan.sharded_scan(run, dist.rank, dist.world, gather)

    for _ in range(args.warmup):
        step()
    dist.barrier()
    clocks = Clocks(dist.local)
    if dist.rank == 0:
        clocks.start()
    ts = []
    for _ in range(args.steps):
        dist.barrier()
        ts.append(events_ms(stream, dist.local, step))
    dist.barrier()
    ck = clocks.stop() if dist.rank == 0 else None
    ms = dist.max(statistics.median(ts))
    # Bit-exact, checked in parallel: each rank folds its own run on the CPU
    # from the entry state the GPU run used and compares every output; then
    # each entry must equal the previous rank's CPU-computed exit state.  By
    # induction from rank 0 (no entry), the whole output is the sequential
    # fold of the concatenated sequence.
    got = dout.cpu().numpy()
    per = dist.gather({"last": got[-1].tobytes(), "rounds": st.rounds, "rewritten": st.rewritten,
                       "entry_exact": st.entry_exact, "phases": st.phases_ms})
    x2 = xs.copy()
    if dist.rank > 0:
        x2[0] = _comb_f32(np.frombuffer(per[dist.rank - 1]["last"], np.float32), xs[0])
    want = O.scan_sequential(x2)
    oks = dist.gather(bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))))
    algo = 16 * SCAN_N * dist.world
    if dist.rank != 0:
        return None
    return {"metric": "affine scan effective HBM GB/s", "value": algo / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded numpy per rank: a U[0.9,1], b N(0,1))",
            "config": {"workload": f"scan: {dist.world} x {SCAN_N:,} maps, one consecutive run per GPU",
                       "pipeline": args.scan_pipeline,
                       "exchange": "nccl" if args.scan_pipeline == "device" else args.scan_exchange,
                       "parallelism": "contiguous runs; one all-gather of halos (2,048 maps) and multiplier "
                                      "tables, entry guess, local exact scan, boundary-state all-gather "
                                      "(rejoin rounds only on a mismatch)",
                       "l2": "1 GiB in+out per GPU > L2"},
            "algorithmic_bytes": algo, "clocks": ck,
            "bit_exact_vs_oracle": all(oks),
            "boundary": {"rounds": per[0]["rounds"], "rewritten": sum(p["rewritten"] for p in per),
                         "entry_guess_exact": sum(1 for p in per if p["entry_exact"]), "ranks": dist.world,
                         "phases_ms_last_step": {f"rank{i}": {k: round(v, 3) for k, v in p["phases"].items()}
                                                 for i, p in enumerate(per)}}}


def _comb_f32(p, q):
    """(q.a * p.a, q.a * p.b + q.b) in f32 with two roundings (scan.rs:127-132)."""
    a = np.float32(q[0]) * np.float32(p[0])
    b = np.float32(q[0]) * np.float32(p[1]) + np.float32(q[1])
    return np.array([a, b], np.float32)


def bench_scan(args, dev, want_cpu):
    import torch

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    r = np.random.default_rng(SCAN_SEED)
    xs = np.empty((SCAN_N, 2), np.float32)
    xs[:, 0] = r.uniform(0.9, 1.0, SCAN_N).astype(np.float32)
    xs[:, 1] = r.standard_normal(SCAN_N).astype(np.float32)
    L = lib()
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    din = torch.from_numpy(xs).cuda()
    dout = torch.empty_like(din)
    run = lambda: check(L.sparsl_dev_assoc_scan_device(dev.handle, din.data_ptr(), SCAN_N, dout.data_ptr(),
                                                       s.cuda_stream), "scan")
    for _ in range(args.warmup):
        run()
    ts = time_launches(s, run, args.kernel_iters)
    ms = statistics.median(ts)
    rep, seg = dev.scan_stats()
    got = dout.cpu().numpy()
    want = O.scan_sequential(xs)
    exact = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
    algo = 16 * SCAN_N
    hin, hout = Pinned(np.float32, 2 * SCAN_N), Pinned(np.float32, 2 * SCAN_N)
    hin.a[:] = xs.reshape(-1)
    ets = [events_ms(L.sparsl_dev_stream(dev.handle), torch.cuda.current_device(),
                     lambda: check(L.sparsl_dev_assoc_scan(dev.handle, hin.ptr, SCAN_N, hout.ptr), "scan e2e"))
           for _ in range(3)]
    e2e_ms = statistics.median(ets)
    hin.free()
    hout.free()
    cpu = None
    if want_cpu:
        t0 = time.perf_counter()
        O.scan_chunked(xs, 256)
        dt_par = time.perf_counter() - t0
        t0 = time.perf_counter()
        O.scan_sequential(xs)
        dt_seq = time.perf_counter() - t0
        cpu = {"value": algo / dt_par / 1e9, "unit": "GB/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"one full 2^26 scan: chunked (CpuParallel arm) {dt_par:.2f} s, sequential {dt_seq:.2f} s"}
    return {"metric": "affine scan effective HBM GB/s", "value": algo / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms, "algorithmic_bytes": algo,
            "config": "2^26 maps, a U[0.9,1.0], b N(0,1), f32; 1 GiB in+out > L2",
            "repair": {"elements_replayed": rep, "segments": seg},
            "e2e": {"value": algo / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 8 * SCAN_N,
                    "d2h_bytes_per_step": 8 * SCAN_N, "path": "sparsl_dev_assoc_scan, pinned host"},
            "roofline": roofline(algo, ms, "scan_main + scan_check (+ scan_repair)", "scan"),
            "bit_exact_vs_oracle": exact, "cpu_baseline": cpu}


SPMM_N, SPMM_NVEC, SPMM_KMAX, SPMM_ALPHA, SPMM_SEED = 1_000_000, 64, 4096, 1.5, 0x5B33


def gen_zipf_csr(n, ncols, kmax, alpha, seed):
    """Row lengths from Zipf(alpha) restricted to [1, kmax] (inverse CDF), then
    that many distinct sorted uniform columns per row (repeats are redrawn)."""
    import torch

    r = np.random.default_rng(seed)
    k = np.arange(1, kmax + 1, dtype=np.float64)
    cdf = np.cumsum(k ** -alpha)
    cdf /= cdf[-1]
    lens = np.minimum(np.searchsorted(cdf, r.random(n), side="right") + 1, kmax).astype(np.int64)
    rp = np.zeros(n + 1, np.int64)
    np.cumsum(lens, out=rp[1:])
    nnz = int(rp[-1])
    rows = torch.from_numpy(np.repeat(np.arange(n, dtype=np.int64), lens)).cuda()
    cols = torch.from_numpy(r.integers(0, ncols, nnz, dtype=np.int64)).cuda()
    while True:
        key, _ = torch.sort(rows * ncols + cols)
        cols = key % ncols
        dup = torch.nonzero(key[1:] == key[:-1]).flatten() + 1
        if dup.numel() == 0:
            break
        cols[dup] = torch.from_numpy(r.integers(0, ncols, dup.numel(), dtype=np.int64)).cuda()
    col = cols.to(torch.int32).cpu().numpy().view(np.uint32)
    del rows, cols, key
    return rp.astype(np.uint32), col, r


def bench_spmm(args, dev, want_cpu):
    """SpMM with power-law rows: Y += A X, X 1M x 64 row-major, f32 and f16 weights."""
    import torch
    import sparsl_b200 as S

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    n, nv = SPMM_N, SPMM_NVEC
    t0 = time.perf_counter()
    rp, col, r = gen_zipf_csr(n, n, SPMM_KMAX, SPMM_ALPHA, SPMM_SEED)
    nnz = col.size
    w = r.uniform(-1.0, 1.0, nnz).astype(np.float32)
    x = r.uniform(-1.0, 1.0, (n, nv)).astype(np.float32)
    setup_s = time.perf_counter() - t0
    L = lib()
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    dx = torch.from_numpy(x).cuda()
    dy = torch.zeros((n, nv), dtype=torch.float32, device="cuda")
    flush = torch.empty(64 << 22, dtype=torch.float32, device="cuda")  # 1 GiB > L2
    csr = O.Csr(rp, col, n)
    out = {}
    cpu_s = None
    for prec, tag in ((S.WeightPrecision.F32, "f32"), (S.WeightPrecision.F16, "f16")):
        op = dev.prepare_with(S.Csr(rp, col, n), n, w, prec)
        wb = 4 if tag == "f32" else 2
        run = lambda: check(L.sparsl_op_spmm_device(op.handle, dx.data_ptr(), nv, dy.data_ptr(), s.cuda_stream),
                            "spmm")
        # parity over the whole Y: one product from Y = 0 against the oracle
        dy.zero_()
        run()
        s.synchronize()
        got = dy.cpu().numpy()
        t1 = time.perf_counter()
        want = O.spmm(csr, O.quantise(int(prec), w), x.reshape(-1), nv, np.zeros(n * nv, np.float32),
                      par=True).reshape(n, nv)
        if tag == "f32":
            cpu_s = time.perf_counter() - t1
        exact = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
        del got, want
        for _ in range(args.warmup):
            run()
        ts = time_launches(s, run, max(3, args.kernel_iters // 2), flush=lambda: flush_l2(flush))
        ms = statistics.median(ts)
        algo = nnz * (4 + wb) + (n + 1) * 4 + n * nv * 4 + 2 * n * nv * 4
        out[tag] = {"value": algo / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms, "algorithmic_bytes": algo,
                    "bit_exact_vs_oracle": exact,
                    "roofline": roofline(algo, ms, f"SpMM kernels ({tag} weights; compulsory bytes)", "spmm_" + tag)}
        if tag == "f32":
            hx, hy = Pinned(np.float32, n * nv), Pinned(np.float32, n * nv)
            hx.a[:] = x.reshape(-1)
            hy.a[:] = 0
            ets = [events_ms(L.sparsl_op_stream(op.handle), torch.cuda.current_device(),
                             lambda: check(L.sparsl_op_spmm(op.handle, hx.ptr, n * nv, nv, hy.ptr, n * nv), "spmm e2e"))
                   for _ in range(3)]
            e2e_ms = statistics.median(ets)
            hx.free()
            hy.free()
            out[tag]["e2e"] = {"value": algo / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                               "h2d_bytes_per_step": 2 * n * nv * 4, "d2h_bytes_per_step": n * nv * 4,
                               "path": "sparsl_op_spmm, pinned host X/Y"}
        if tag == "f32":
            ragged, rtick = bench_ragged(args, op, csr, w, s, flush)
        del op
    cpu = None
    if want_cpu:
        cpu = {"value": out["f32"]["algorithmic_bytes"] / cpu_s / 1e9, "unit": "GB/s", "cores": O.num_threads(),
               "kind": "port", "sample": f"one full f32 SpMM of the same matrix ({cpu_s:.2f} s, the parity check), "
                                         "CpuParallel restatement"}
    f32 = out["f32"]
    return {"metric": "SpMM effective HBM GB/s", "value": f32["value"], "unit": "GB/s",
            "ms_per_step": f32["ms_per_step"], "algorithmic_bytes": f32["algorithmic_bytes"],
            "config": f"{n:,} x {n:,}, row lengths Zipf({SPMM_ALPHA}) restricted to [1,{SPMM_KMAX}] "
                      f"(realised nnz {nnz:,}, mean {nnz / n:.1f}), distinct sorted uniform cols, w U[-1,1], "
                      f"X {n:,} x {nv} row-major U[-1,1]; L2 flushed (1 GiB written, then read back) before every launch",
            "setup_s": round(setup_s, 1), "e2e": f32.get("e2e"),
            "bit_exact_vs_oracle": f32["bit_exact_vs_oracle"], "roofline": f32["roofline"], "f16": out["f16"],
            "cpu_baseline": cpu, "ragged_spmv": ragged, "ragged_lif_tick": rtick}


def bench_ragged(args, op, csr, w, s, flush):
    """SpMV and the recurrent fused spike-LIF tick over the config-4 power-law
    matrix (n_vec = 1): the row fold in descending-length order.  Bit-exact
    against the oracle; the tick's CPU arm is timed on the same ticks."""
    import torch

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    L = lib()
    n, nnz = csr.nrows, csr.nnz
    r = np.random.default_rng(SPMM_SEED ^ 0x5A)
    x = r.uniform(0.0, 1.0, n).astype(np.float32)
    dx = torch.from_numpy(x).cuda()
    dy = torch.zeros(n, dtype=torch.float32, device="cuda")
    run = lambda: check(L.sparsl_op_spmv_device(op.handle, dx.data_ptr(), dy.data_ptr(), s.cuda_stream), "spmv")
    for _ in range(args.warmup):
        run()
    dy.zero_()
    ts = time_launches(s, run, args.kernel_iters, flush=lambda: flush_l2(flush))
    ms = statistics.median(ts)
    want = np.zeros(n, np.float32)
    for _ in range(args.kernel_iters):
        O.spmv(csr, w, x, want, par=True)
    exact = bool(np.array_equal(dy.cpu().numpy().view(np.uint32), want.view(np.uint32)))
    algo = nnz * 8 + (n + 1) * 4 + n * 4 + 2 * n * 4
    spmv = {"metric": "ragged SpMV effective HBM GB/s", "value": algo / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms, "algorithmic_bytes": algo, "bit_exact_vs_oracle": exact,
            "config": f"the SpMM matrix ({n:,} rows, {nnz:,} nnz, Zipf(1.5) lengths) times a dense x U[0,1]; "
                      "L2 flushed before every launch",
            "roofline": roofline(algo, ms, "ordered_fold_kernel<f32, dense x> (rows of 1,024+ entries a warp "
                                           "each, the rest from the tile-interleaved ordered copy)", "ragged_spmv")}
    # Recurrent ticks (fused spike SpMV + LIF + packing + index list), timed
    # from the initial state; the timed ticks are checked against the CPU.
    ticks = 20
    v0 = r.uniform(0.0, 1.0, n).astype(np.float32)
    th0 = np.full(n, 1.0, np.float32)
    pk0 = O.pack_spikes((r.random(n) < 0.02).astype(np.uint8))
    wt = (w * np.float32(0.05)).astype(np.float32)  # a network that neither dies out nor saturates
    # (the caller destroys the operator right after, so its weights stay scaled)
    check(L.sparsl_op_set_weights(op.handle, wt.ctypes.data, wt.size), "set_weights")
    opx = lambda a: a.ctypes.data
    for _ in range(2):
        check(L.sparsl_op_write_x_spikes(op.handle, opx(pk0), pk0.size), "write spikes")
        check(L.sparsl_op_write_lif_state(op.handle, opx(v0), opx(th0), n), "write state")
        st = L.sparsl_op_stream(op.handle)
        tms = events_ms(st, torch.cuda.current_device(),
                        lambda: check(L.sparsl_op_recurrent_steps_async(op.handle, 0.95, 0.0, 0.0, ticks), "ticks"))
        check(L.sparsl_op_wait(op.handle), "wait")
    trace = np.zeros(ticks, np.uint32)
    cnt = ctypes.c_uint64()
    check(L.sparsl_op_spike_trace(op.handle, trace.ctypes.data, ticks, ctypes.byref(cnt)), "trace")
    vg, tg, sg = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.uint8)
    check(L.sparsl_op_sync_lif_state(op.handle, opx(vg), opx(tg), opx(sg), n), "sync state")
    vw, tw, sw, xw = v0.copy(), th0.copy(), np.zeros(n, np.uint8), pk0.copy()
    t0 = time.perf_counter()
    trace_w = O.recurrent_steps(csr, wt, xw, vw, tw, sw, 0.95, 0.0, 0.0, ticks, par=True)
    cpu_s = time.perf_counter() - t0
    ok = bool(np.array_equal(trace, trace_w) and np.array_equal(vg.view(np.uint32), vw.view(np.uint32))
              and np.array_equal(sg, sw))
    per = tms / ticks
    talgo = nnz * 8 + (n + 1) * 4 + 2 * n * 4 + n * 4 + 2 * n // 8
    tick = {"metric": "ragged LIF ticks/sec", "value": 1e3 / per, "unit": "ticks/s", "ms_per_step": per,
            "ticks": ticks, "algorithmic_bytes_per_tick": talgo, "spike_trace": trace.tolist(),
            "bit_exact_vs_oracle": ok,
            "config": f"the SpMM matrix as a recurrent network (weights x 0.05), decay 0.95, theta 1, reset 0, "
                      "Bernoulli(0.02) initial spikes",
            "roofline": roofline(talgo, per, "ordered_fold_kernel<f32, spike bitmask in shared memory, LIF> + "
                                             "pack_kernel + compact_bits_kernel", "ragged_tick"),
            "cpu_baseline": {"value": ticks / cpu_s, "unit": "ticks/s", "cores": O.num_threads(), "kind": "port",
                             "sample": f"the same {ticks} ticks (the parity check), CpuParallel restatement"}}
    return spmv, tick


def bench_ragged_only(args, dev, want_cpu):
    """The config-4 power-law matrix as a plain SpMV and as a recurrent
    network (n_vec = 1), without the SpMM legs."""
    import torch
    import sparsl_b200 as S

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    n = SPMM_N
    rp, col, r = gen_zipf_csr(n, n, SPMM_KMAX, SPMM_ALPHA, SPMM_SEED)
    w = r.uniform(-1.0, 1.0, col.size).astype(np.float32)
    s = torch.cuda.Stream()
    torch.cuda.set_stream(s)
    flush = torch.empty(64 << 22, dtype=torch.float32, device="cuda")  # 1 GiB > L2
    op = dev.prepare(S.Csr(rp, col, n), n, w)
    spmv, tick = bench_ragged(args, op, O.Csr(rp, col, n), w, s, flush)
    del op
    spmv["ragged_lif_tick"] = tick
    return spmv


def bench_lif_integrate(args, dev, n=1 << 26):
    """Device::lif_integrate over dense currents (mod.rs:1202-1229) on 2^26
    cells in device memory: v, theta, currents read, v, theta, spike bytes
    written (21 B per cell; 1.4 GB > L2, no flush needed)."""
    import torch

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    L = lib()
    r = np.random.default_rng(0x11F)
    v0 = r.uniform(0.0, 1.0, n).astype(np.float32)
    t0 = np.full(n, 1.0, np.float32)
    cur = (r.standard_normal(n) * 0.1).astype(np.float32)
    s = torch.cuda.Stream()
    dv, dt, dc = (torch.from_numpy(a.copy()).cuda() for a in (v0, t0, cur))
    ds = torch.zeros(n, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    run = lambda: check(L.sparsl_dev_lif_integrate_device(dev.handle, dv.data_ptr(), dt.data_ptr(), dc.data_ptr(),
                                                          ds.data_ptr(), n, 0.95, 0.0, 0.0, s.cuda_stream), "lif")
    for _ in range(args.warmup):
        run()
    # parity: one more step from a fresh state against the oracle (the
    # warm-up launches must be done before the state is rewritten)
    s.synchronize()
    dv.copy_(torch.from_numpy(v0))
    dt.copy_(torch.from_numpy(t0))
    torch.cuda.synchronize()
    run()
    s.synchronize()
    vw, tw, sw = v0.copy(), t0.copy(), np.zeros(n, np.uint8)
    O.lif_integrate(vw, tw, cur, sw, np.float32(0.95), np.float32(0.0), np.float32(0.0), par=True)
    ok = bool(np.array_equal(dv.cpu().numpy().view(np.uint32), vw.view(np.uint32))
              and np.array_equal(dt.cpu().numpy().view(np.uint32), tw.view(np.uint32))
              and np.array_equal(ds.cpu().numpy(), sw))
    ts = time_launches(s, run, args.kernel_iters)
    ms = statistics.median(ts)
    algo = 21 * n
    del dv, dt, dc, ds
    return {"metric": "lif_integrate effective HBM GB/s", "value": algo / (ms * 1e-3) / 1e9, "unit": "GB/s",
            "ms_per_step": ms, "algorithmic_bytes": algo, "bit_exact_vs_oracle": ok,
            "config": f"{n:,} cells, v U[0,1], theta 1, currents N(0,0.1^2), decay 0.95; 1.4 GB > L2",
            "roofline": roofline(algo, ms, "lif_integrate_kernel", "lif_integrate")}


def bench_lif(args, dev, want_cpu):
    import torch
    import sparsl_b200 as S

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    n, fan = LIF_N, LIF_FANIN
    nnz = n * fan
    dcol, dw = DevArray(dev, nnz * 4), DevArray(dev, nnz * 4)
    check(lib().sparsl_workload_fixed_fanin(LIF_SEED, 0, n, n, fan, LIF_SIGMA, dcol.ptr, dw.ptr, None), "gen")
    col, w = dcol.to_host(np.uint32, nnz), dw.to_host(np.float32, nnz)
    dcol.free()
    dw.free()
    rp = (np.arange(n + 1, dtype=np.uint64) * fan).astype(np.uint32)
    dv, dth, dpk = DevArray(dev, n * 4), DevArray(dev, n * 4), DevArray(dev, n // 8)
    check(lib().sparsl_workload_lif_state(LIF_SEED ^ 0x57A7E, 0, n, 0.0, 1.0, 1.0, LIF_DENSITY, dv.ptr, dth.ptr,
                                          dpk.ptr, None), "state")
    v0, th0, pk0 = dv.to_host(np.float32, n), dth.to_host(np.float32, n), dpk.to_host(np.uint32, n // 32)
    for a in (dv, dth, dpk):
        a.free()
    op = dev.prepare(S.Csr(rp, col, n), n, w)
    L = lib()
    # warm-up from the initial state, then the timed run of `ticks` ticks from
    # the initial state again; the timed ticks are the ones checked below
    op.write_x_spikes(pk0)
    op.write_lif_state(v0, th0)
    check(L.sparsl_op_recurrent_steps(op.handle, 0.95, 0.0, 0.0, args.warmup), "warm")
    op.write_x_spikes(pk0)
    op.write_lif_state(v0, th0)
    ticks = args.lif_ticks
    st = L.sparsl_op_stream(op.handle)
    ms = events_ms(st, torch.cuda.current_device(),
                   lambda: check(L.sparsl_op_recurrent_steps_async(op.handle, 0.95, 0.0, 0.0, ticks), "ticks"))
    check(L.sparsl_op_wait(op.handle), "wait")
    trace = op.spike_trace()
    vg, tg, sg = np.zeros(n, np.float32), np.zeros(n, np.float32), np.zeros(n, np.bool_)
    op.sync_lif_state(vg, tg, sg)
    xg = op.sync_x_spikes()
    # Bit-exact against the oracle's CpuParallel recurrent ticks over the same
    # arrays: every tick's spike count, the final membrane, threshold, spikes
    # and packed spike words.  The CPU run is also the CPU baseline.
    csr = O.Csr(rp, col, n)
    vw, tw, sw, xw = v0.copy(), th0.copy(), np.zeros(n, np.uint8), pk0.copy()
    t0 = time.perf_counter()
    trace_w = O.recurrent_steps(csr, w, xw, vw, tw, sw, 0.95, 0.0, 0.0, ticks, par=True)
    cpu_s = time.perf_counter() - t0
    exact = bool(np.array_equal(trace, trace_w) and np.array_equal(vg.view(np.uint32), vw.view(np.uint32))
                 and np.array_equal(tg.view(np.uint32), tw.view(np.uint32))
                 and np.array_equal(sg.astype(np.uint8), sw) and np.array_equal(xg, xw))
    algo = nnz * 8 + (n + 1) * 4 + 2 * n * 4 + n * 4 + 2 * n // 8
    # end to end: one tick per slice-API call with pinned host buffers
    hs, hv, ht, ho = Pinned(np.uint32, n // 32), Pinned(np.float32, n), Pinned(np.float32, n), Pinned(np.uint8, n)
    hs.a[:] = pk0
    hv.a[:] = v0
    ht.a[:] = th0
    e2e_steps = 20

    def e2e():
        for _ in range(e2e_steps):
            check(L.sparsl_op_fused_spikes_lif(op.handle, hs.ptr, n // 32, hv.ptr, ht.ptr, ho.ptr, n, 0.95, 0.0, 0.0),
                  "e2e tick")
            hs.a[:] = S.pack_spikes(ho.a)  # the host-side pack_spikes_into of the reference API

    e2e_ms = statistics.median(events_ms(st, torch.cuda.current_device(), e2e) for _ in range(3))
    for h in (hs, hv, ht, ho):
        h.free()
    cpu = None
    if want_cpu:
        cpu = {"value": ticks / cpu_s, "unit": "ticks/s", "cores": O.num_threads(), "kind": "port",
               "sample": f"{ticks} full ticks of the same network ({cpu_s:.1f} s, the parity check), "
                         "CpuParallel restatement"}
    per_tick = ms / ticks
    standalone = bench_lif_integrate(args, dev)
    return {"metric": "LIF net ticks/sec (1 GPU)", "value": 1e3 / per_tick, "unit": "ticks/s",
            "ms_per_step": per_tick, "ticks": ticks, "algorithmic_bytes_per_tick": algo,
            "effective_GBs": algo / (per_tick * 1e-3) / 1e9,
            "config": "262,144 neurons x fan-in 512, w N(0,0.05^2), decay 0.95, theta 1, reset 0, Bernoulli(0.02)",
            "spike_trace_sum": int(trace.sum()),
            "e2e": {"value": e2e_steps / (e2e_ms * 1e-3), "unit": "ticks/s",
                    "h2d_bytes_per_step": n // 8 + 8 * n, "d2h_bytes_per_step": 9 * n,
                    "path": "sparsl_op_fused_spikes_lif per tick + host repack, pinned host"},
            "roofline": roofline(algo, per_tick, "ell_stream_kernel<f32, spike bitmask in shared memory, LIF> + "
                                                 "compact_bits_kernel (side stream)", "lif"),
            "bit_exact_vs_oracle": exact, "checked_ticks": ticks, "cpu_baseline": cpu,
            "lif_integrate": standalone}


# --------------------------------------------------------------------------
# reference arm: the oracle's CpuParallel restatement on the host cores
# --------------------------------------------------------------------------
def bench_reference(args, dist):
    """The reference arm: the oracle's CpuParallel restatement of the tick
    (cpu_fused_spikes_*, mod.rs:2572-2614, driven as recurrent_steps,
    mod.rs:1889-1932) on this host's cores, over the whole 4.29e9-synapse
    network drawn on the host from the workload's definition (the arrays the
    GPU arm draws, bit for bit).  Every step is one full tick; nothing is
    sampled or extrapolated.  Rank 0 alone runs it."""
    if dist.rank != 0:
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O

    n_total, fan_in = NET_N, NET_FANIN
    O.set_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    blocks = []
    for (off, nrows) in net_blocks(n_total, fan_in):
        rp = (np.arange(nrows + 1, dtype=np.uint64) * fan_in).astype(np.uint32)
        col, w = O.wl_fixed_fanin(NET_SEED, off, nrows, n_total, fan_in, NET_SIGMA)
        blocks.append((rp, col, w))
    v, th, s0 = O.wl_lif_state(NET_SEED ^ 0x57A7E, 0, n_total, 0.0, 1.0, NET_THETA0, NET_DENSITY)
    pk = O.pack_spikes(s0)
    setup_s = time.perf_counter() - t0
    sp = np.zeros(n_total, np.uint8)
    p = (NET_DECAY, NET_VRESET, NET_DTHETA)
    trace = [O.net_ticks(blocks, n_total, pk, v, th, sp, *p, args.warmup)]
    ts = []
    for _ in range(args.steps):
        t1 = time.perf_counter()
        trace.append(O.net_ticks(blocks, n_total, pk, v, th, sp, *p, 1))
        ts.append(time.perf_counter() - t1)
    full = np.concatenate(trace).astype(np.uint32)
    dt = sum(ts)
    value = args.steps / dt
    desc = (f"{args.steps} full ticks of the {n_total:,} x {fan_in} network ({n_total * fan_in:.3g} synapses) after "
            f"{args.warmup} warm-up ticks, {dt:.1f} s; network drawn on the host in {setup_s:.0f} s")
    return {
        "impl": "reference", "metric": "LIF net ticks/sec", "value": value, "unit": "ticks/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 / value,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded ChaCha12 per row, drawn on the host from the workload definition)",
        "config": {"workload": f"lif_net: {n_total:,} neurons x fan-in {fan_in} ({n_total * fan_in:.3g} synapses), "
                               "f32 weights N(0,0.03^2), decay 0.95, theta 1.0, reset 0, Bernoulli(0.01) initial spikes",
                   "arm": "C restatement of sparsl's CpuParallel arm (Rust toolchain absent here)",
                   "setup_s": round(setup_s, 1)},
        "cpu_baseline": {"value": value, "unit": "ticks/s", "cores": O.num_threads(), "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": "ticks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "check": {"spike_trace_sum": int(full[args.warmup:].sum()), "trace_head": full[args.warmup:][:8].tolist(),
                  f"trace_sha1_first_{full.size}_ticks": __import__("hashlib").sha1(full.tobytes()).hexdigest()[:16],
                  "tick_s_min_median_max": [min(ts), sorted(ts)[len(ts) // 2], max(ts)]},
    }


def main():
    faulthandler.enable()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="sparsl", choices=["sparsl", "reference"])
    ap.add_argument("--workload", default="lif_net", choices=["lif_net", "spmv", "spmm", "scan", "lif", "ragged"])
    ap.add_argument("--no-extras", action="store_true", help="N=1: skip the SpMV / scan / LIF-1GPU figures")
    ap.add_argument("--kernel-iters", type=int, default=20)
    ap.add_argument("--scan-exchange", default="gloo", choices=["gloo", "nccl"],
                    help="N>1 host-driven scan: the process group that carries the boundary exchanges")
    ap.add_argument("--scan-pipeline", default="device", choices=["device", "host"],
                    help="N>1 scan: every step enqueued on the device with NCCL gathers and one host sync "
                         "(device), or the host-driven steps (host)")
    # Smaller instances of the same workloads (profiling captures, quick runs).
    ap.add_argument("--scan-n", type=int, default=None, help="scan length (default 2^26)")
    ap.add_argument("--lif-ticks", type=int, default=1000, help="timed ticks of the 1-GPU LIF network")
    ap.add_argument("--net-n", type=int, default=None, help="neurons of the LIF network (default 4,194,304)")
    ap.add_argument("--net-fanin", type=int, default=None, help="fan-in of the LIF network (default 1024)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--check-ticks", type=int, default=32,
                    help="LIF network: ticks compared bit for bit with the CPU (capped at warm-up + steps)")
    ap.add_argument("--no-check", action="store_true", help="LIF network: skip the CPU comparison")
    ap.add_argument("--net-exchange", default="peer", choices=["peer", "nccl"],
                    help="LIF network, N>1: spike-vector exchange through peer memory or an NCCL all-gather")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    global SCAN_N, NET_N, NET_FANIN
    if args.scan_n:
        SCAN_N = args.scan_n
    if args.net_n:
        NET_N = args.net_n
    if args.net_fanin:
        NET_FANIN = args.net_fanin
    if args.steps is None:
        args.steps = 10 if args.impl == "reference" else 200
    args.warmup = max(args.warmup, 1)
    dist = Dist()
    try:
        if args.impl == "reference":
            line = bench_reference(args, dist)
        elif args.workload != "lif_net":
            import torch
            import sparsl_b200 as S

            torch.cuda.set_device(dist.local)
            dev = S.Device.try_new(S.Backend.Cuda, dist.local)
            if args.workload == "scan" and dist.world > 1:
                line = bench_scan_sharded(args, dev, dist)
            elif args.workload in ("spmv", "spmm") and dist.world > 1:
                line = bench_rowshard(args, dev, dist, args.workload)
            else:
                fn = {"spmv": bench_spmv, "spmm": bench_spmm, "scan": bench_scan, "lif": bench_lif,
                      "ragged": bench_ragged_only}[args.workload]
                line = fn(args, dev, dist.rank == 0 and not args.no_cpu) if dist.rank == 0 else None
        else:
            line = bench_lif_net(args, dist)
            if dist.world == 1 and not args.no_extras:
                import torch
                import sparsl_b200 as S

                torch.cuda.empty_cache()
                dev = S.Device.try_new(S.Backend.Cuda, dist.local)
                extras = {}
                for name, fn in (("spmv", bench_spmv), ("spmm", bench_spmm), ("scan", bench_scan), ("lif", bench_lif)):
                    try:
                        extras[name] = fn(args, dev, not args.no_cpu)
                    except Exception as e:  # report, never hide
                        extras[name] = {"error": repr(e)}
                line["workloads"] = extras
        if dist.rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()


if __name__ == "__main__":
    main()

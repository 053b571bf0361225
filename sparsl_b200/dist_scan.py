"""The exact affine-map scan over maps split into consecutive runs, one run
per rank (one process per GPU).

The reference has one device and a strict left fold (src/scan.rs:298-313);
splitting the sequence keeps the fold's bits by the same speculate/verify
rule the single-device kernel uses between tiles:

1. every rank receives the last ``halo`` maps before its run (one all-gather
   of each rank's tail);
2. it guesses its entry state: the offset chain B by folding the halo from a
   copy of its first map (B contracts for |a| < 1, so the guess usually lands
   on the sequential trajectory exactly); the multiplier chain A exactly, by
   carrying rank 0's exit multiplier through the other runs' transfer tables
   (the f32 chain settles on a value in {0..7} * 2^-149, whose image under a
   run is what the table records) -- gathered with the halos;
3. it scans its run from that entry state;
4. the ranks exchange (entry used, exit state); rank r's run is exact when its
   entry equals rank r-1's exit bit for bit and rank r-1 is exact, rank 0
   being exact by construction.  The first rank that fails the check rewrites
   its run from its predecessor's exit until the output rejoins the stored
   trajectory, and the exchange repeats (at most world - 1 times).

Every rank runs the same collectives in the same order, so no rank waits for
another that left the loop.  The driver is written against a small engine
(tail / table / settle / fold / scan / exit_state / rejoin) so the same logic runs on the GPU
engine and, in the tests, on the CPU oracle.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional

import numpy as np

DEFAULT_HALO = 2048


@dataclass
class ShardedScanStats:
    rounds: int            # boundary exchanges after the first
    rewritten: int         # maps this rank rewrote while rejoining
    entry_exact: bool      # this rank's first guess was already exact
    phases_ms: Dict[str, float] = field(default_factory=dict)  # host wall clock per phase


def _bits(v) -> np.ndarray:
    return np.ascontiguousarray(v, dtype=np.float32).view(np.uint32)


def _nibble(table: int, m: int) -> int:
    return (table >> (4 * m)) & 0xF


def _f2u(x: float) -> int:
    return int(np.array([x], np.float32).view(np.uint32)[0])


def _u2f(u: int) -> np.float32:
    return np.array([u], np.uint32).view(np.float32)[0]


def sharded_scan(engine, rank: int, world: int, all_gather: Callable[[np.ndarray], List[np.ndarray]],
                 halo: int = DEFAULT_HALO) -> ShardedScanStats:
    """Run one rank's part.  ``engine`` works on this rank's run (n >= 1 maps);
    ``all_gather(a)`` returns every rank's float32 array ``a`` (same shape on
    every rank) in rank order."""
    if engine.n < 1:
        raise ValueError("every rank's run needs at least one map")
    ph: Dict[str, float] = {}
    t0 = time.perf_counter()

    def mark(name):
        nonlocal t0
        t1 = time.perf_counter()
        ph[name] = ph.get(name, 0.0) + (t1 - t0) * 1e3
        t0 = t1

    # 1. What every rank tells the others, in one all-gather:
    #    - its last `halo` maps (padded in front with identity maps) and how
    #      many are real: the offset chain B is guessed from them;
    #    - its run's transfer table for the multiplier chain A, and on rank 0
    #      the exact multiplier leaving its run (the chain settles on a value
    #      in {0..7} * 2^-149 and the tables carry it exactly), so every rank
    #      gets its exact entry multiplier when the chain has settled.
    tail = np.ones((halo, 2), np.float32)
    tail[:, 1] = 0.0
    t = engine.tail(halo)
    if len(t):
        tail[halo - len(t):] = t
    table, a_exit0 = 0xFFFFFFFF, 8
    if rank == 0:
        a_s, k = engine.settle()
        if _f2u(a_s) <= 7:
            a_exit0 = _nibble(engine.table(k), _f2u(a_s)) if k < engine.n else _f2u(a_s)
    else:
        table = engine.table(0)
    meta = np.array([min(engine.n, halo), 0, 0], np.uint32)
    meta[1], meta[2] = table, a_exit0
    blob = np.concatenate([tail.ravel(), meta.view(np.float32)])
    mark("local_tables")
    parts = all_gather(blob)
    mark("exchange_halo")
    tails = [p[: 2 * halo].reshape(halo, 2) for p in parts]
    metas = [p[2 * halo:].view(np.uint32) for p in parts]
    entry: Optional[np.ndarray] = None
    if rank > 0:
        # B: fold the maps just before this run, nearest last, at most `halo`.
        chunks, need = [], halo
        for r in range(rank - 1, -1, -1):
            k = int(metas[r][0])
            take = min(k, need)
            chunks.append(tails[r][halo - take:])
            need -= take
            if need == 0:
                break
        entry = np.asarray(engine.fold(np.concatenate(chunks[::-1])), np.float32).copy()
        # A: rank 0's exit multiplier carried through the tables of ranks 1..rank-1.
        m = int(metas[0][2])
        for r in range(1, rank):
            if m > 7:
                break
            m = _nibble(int(metas[r][1]), m)
        if m <= 7:
            entry[0] = _u2f(m)
    mark("entry_guess")
    # 2. the run from the guessed entry state
    engine.scan(entry)
    first_entry = None if entry is None else entry.copy()
    rewritten, rounds = 0, 0
    nan2 = np.array([np.nan, np.nan], np.float32)
    # 3. verify: every entry against its predecessor's exit, bit for bit;
    #    the first rank that fails rewrites its run from that exit.
    while True:
        mine = np.concatenate([nan2 if entry is None else np.asarray(entry, np.float32), engine.exit_state()])
        mark("scan" if rounds == 0 else "rejoin")
        states = all_gather(mine.astype(np.float32))
        mark("exchange_states")
        bad = next((r for r in range(1, world)
                    if not np.array_equal(_bits(states[r][:2]), _bits(states[r - 1][2:]))), None)
        if bad is None:
            break
        rounds += 1
        if rounds >= world:
            raise RuntimeError("sharded scan: boundary states did not settle")
        if rank == bad:
            entry = states[bad - 1][2:].copy()
            rewritten += engine.rejoin(entry)
    exact_first = rank == 0 or (first_entry is not None and np.array_equal(_bits(first_entry), _bits(entry)))
    return ShardedScanStats(rounds=rounds, rewritten=rewritten, entry_exact=bool(exact_first), phases_ms=ph)


class _Offset:
    def __init__(self, base, nbytes: int):
        self._p = base.data_ptr() + nbytes

    def data_ptr(self) -> int:
        return self._p


class DeviceRun:
    """The GPU engine: a run of ``n`` maps in device memory (d_in, d_out:
    objects with ``data_ptr()``, n (a, b) f32 pairs each) on ``device``."""

    def __init__(self, device, d_in, d_out, n: int, host_tail: Optional[np.ndarray] = None):
        # Everything runs on the device's own stream (sparsl_dev_stream).
        self.device, self.d_in, self.d_out, self.n, self.stream = device, d_in, d_out, int(n), None
        self._tail = host_tail
        self._staging = None
        self._exit = None

    def tail(self, h: int) -> np.ndarray:
        if self._tail is not None:
            return self._tail[-h:]
        from . import _lib

        k = min(h, self.n)
        out = np.empty((k, 2), np.float32)
        if k:
            src = self.d_in.data_ptr() + (self.n - k) * 8
            rc = _lib.load().sparsl_memcpy(out.ctypes.data, src, out.nbytes)
            if rc != 0:
                raise RuntimeError(f"tail copy failed: {_lib.last_error()}")
        return out

    def fold(self, prefix: np.ndarray) -> np.ndarray:
        import torch

        if self._staging is None or self._staging.shape[0] < len(prefix):
            self._staging = torch.empty((len(prefix), 2), dtype=torch.float32, device=f"cuda:{torch.cuda.current_device()}")
        self._staging[: len(prefix)].copy_(torch.from_numpy(np.ascontiguousarray(prefix)))
        torch.cuda.synchronize()
        return self.device.scan_fold_device(self._staging, len(prefix), None, self.stream)

    def table(self, k: int) -> int:
        return self.device.scan_table_device(_Offset(self.d_in, 8 * k), self.n - k, self.stream)

    def settle(self):
        return self.device.scan_settle_device(self.d_in, self.n, self.stream)

    def scan(self, entry) -> None:
        self.device.assoc_scan_from_device(self.d_in, self.n, self.d_out, entry, self.stream)
        self._exit = None

    def exit_state(self) -> np.ndarray:
        if self._exit is None:
            from . import _lib

            self.device.wait()
            out = np.empty(2, np.float32)
            rc = _lib.load().sparsl_memcpy(out.ctypes.data, self.d_out.data_ptr() + (self.n - 1) * 8, 8)
            if rc != 0:
                raise RuntimeError(f"exit state copy failed: {_lib.last_error()}")
            self._exit = out
        return self._exit

    def rejoin(self, entry) -> int:
        ex, k = self.device.scan_rejoin_device(self.d_in, self.d_out, self.n, entry, self.stream)
        self._exit = ex
        return int(k)


def process_group_all_gather(pg, world: int) -> Callable[[np.ndarray], List[np.ndarray]]:
    """``all_gather`` over a torch.distributed process group with a CPU
    backend (gloo): the boundary states and halos are host values."""
    import torch

    def gather(a: np.ndarray) -> List[np.ndarray]:
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
        parts = [torch.zeros_like(t) for _ in range(world)]
        pg.all_gather(parts, t)
        return [p.numpy() for p in parts]

    return gather


def nccl_all_gather(group, world: int, device) -> Callable[[np.ndarray], List[np.ndarray]]:
    """``all_gather`` over a torch.distributed NCCL group: the host values go
    through a small device buffer (one all-gather over NVLink, then one copy
    back to the host)."""
    import torch

    def gather(a: np.ndarray) -> List[np.ndarray]:
        t = torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(device)
        out = torch.empty((world,) + tuple(t.shape), dtype=torch.float32, device=device)
        torch.distributed.all_gather_into_tensor(out, t, group=group)
        h = out.cpu().numpy()
        return [h[i] for i in range(world)]

    return gather


def sharded_scan_device(device, d_in, d_out, n: int, rank: int, world: int, all_gather_dev,
                        halo: int = DEFAULT_HALO) -> ShardedScanStats:
    """The same algorithm as ``sharded_scan`` with every step enqueued on the
    device's own stream and one host synchronisation per call.

    ``d_in`` / ``d_out`` are (n, 2) float32 CUDA tensors of this rank's run;
    ``all_gather_dev(t)`` returns a (world, *t.shape) CUDA tensor of every
    rank's ``t`` in rank order, enqueued on the current stream (an NCCL
    all-gather).  The halo and tables travel in one gather, the boundary
    states in a second; only those states come back to the host, and only a
    failed boundary check (rare: the multiplier arrives exactly and the offset
    contracts) falls back to host-driven rejoin rounds.
    """
    import torch

    if n < 1:
        raise ValueError("every rank's run needs at least one map")
    t0 = time.perf_counter()
    dev_t = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.ExternalStream(device.stream_handle(), device=dev_t)
    with torch.cuda.stream(stream):
        blob = torch.empty(2 * halo + 4, dtype=torch.float32, device=dev_t)
        device.scan_publish_device(d_in, n, rank == 0, halo, blob)
        gathered = all_gather_dev(blob)
        st = torch.empty(4, dtype=torch.float32, device=dev_t)
        if rank > 0:
            entry_d = torch.empty(2, dtype=torch.float32, device=dev_t)
            device.scan_entry_device(gathered, world, rank, halo, entry_d)
            device.assoc_scan_after_device(d_in, n, d_out, entry_d)
            st[:2].copy_(entry_d)
        else:
            device.assoc_scan_from_device(d_in, n, d_out, None)
            st[:2].fill_(float("nan"))
        st[2:].copy_(d_out[n - 1])
        states = all_gather_dev(st).cpu().numpy()
    ph = {"device_pipeline": (time.perf_counter() - t0) * 1e3}
    entry = None if rank == 0 else states[rank][:2].copy()
    first_entry = None if entry is None else entry.copy()
    exit_state = states[rank][2:].copy()
    rewritten, rounds = 0, 0

    def host_gather(a: np.ndarray) -> List[np.ndarray]:
        with torch.cuda.stream(stream):
            g = all_gather_dev(torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev_t)).cpu().numpy()
        return [g[i] for i in range(world)]

    while True:
        bad = next((r for r in range(1, world)
                    if not np.array_equal(_bits(states[r][:2]), _bits(states[r - 1][2:]))), None)
        if bad is None:
            break
        rounds += 1
        if rounds >= world:
            raise RuntimeError("sharded scan: boundary states did not settle")
        if rank == bad:
            entry = states[bad - 1][2:].copy()
            ex, k = device.scan_rejoin_device(d_in, d_out, n, entry)
            exit_state = np.asarray(ex, np.float32)
            rewritten += int(k)
        nan2 = np.array([np.nan, np.nan], np.float32)
        states = host_gather(np.concatenate([nan2 if entry is None else np.asarray(entry, np.float32), exit_state]))
    if rounds:
        ph["rejoin_rounds"] = (time.perf_counter() - t0) * 1e3 - ph["device_pipeline"]
    exact_first = rank == 0 or np.array_equal(_bits(first_entry), _bits(entry))
    return ShardedScanStats(rounds=rounds, rewritten=rewritten, entry_exact=bool(exact_first), phases_ms=ph)


def nccl_all_gather_dev(group, world: int):
    """``all_gather_dev`` for ``sharded_scan_device`` over an NCCL group."""
    import torch

    def gather(t):
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        torch.distributed.all_gather_into_tensor(out, t.contiguous(), group=group)
        return out

    return gather

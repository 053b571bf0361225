"""Host-side mirror of sparsl's ``Device`` / ``SparseOp`` API over libsparsl_cuda.

Names, argument meaning, check order and error variants follow
``src/backend/mod.rs`` of bharathvbcr/sparsl 0.3.0, so code written against
the reference reads the same here.  Arrays are numpy; mutable outputs
(``y``, ``v``, ``theta``, ``spikes``) are updated in place, as the Rust
``&mut [T]`` arguments are.

This package is the CUDA substrate only.  ``Device.try_new`` opens a real
B200 or raises :class:`BackendUnavailable` -- it never returns a CPU device
under a GPU label, and no operation here ever runs on the CPU instead.
"""
from __future__ import annotations

import ctypes
import enum
import math
import sys
from dataclasses import dataclass
from typing import Optional

import numpy as np

from . import _lib
from ._lib import Shape

# --------------------------------------------------------------------------
# Backend identity and availability (mod.rs:60-202)
# --------------------------------------------------------------------------


class Backend(enum.Enum):
    CpuSequential = 0
    CpuParallel = 1
    Metal = 2
    Cuda = 3

    def label(self) -> str:
        return {
            Backend.CpuSequential: "CPU sequential",
            Backend.CpuParallel: "CPU parallel (rayon)",
            Backend.Metal: "Metal GPU",
            Backend.Cuda: "CUDA GPU",
        }[self]

    def unavailable_reason(self):
        """Why this backend cannot execute here, or None (mod.rs:106-112)."""
        if self is Backend.Cuda:
            why = ctypes.c_char_p()
            rc = _lib.load().sparsl_cuda_probe(ctypes.byref(why))
            return None if rc == 0 else (why.value.decode() if why.value else _lib.last_error())
        if self is Backend.Metal:
            return "Metal is only available on macOS"
        return "this package provides the CUDA substrate only; the CPU arms are the reference crate's"

    def is_available(self) -> bool:
        return self.unavailable_reason() is None

    def is_gpu(self) -> bool:
        return self in (Backend.Metal, Backend.Cuda)

    def __str__(self) -> str:
        return self.label()


ALL_BACKENDS = (Backend.CpuSequential, Backend.CpuParallel, Backend.Metal, Backend.Cuda)


def available_backends():
    """Backends that can execute right now, in a stable order (mod.rs:193-202)."""
    return [b for b in ALL_BACKENDS if b.is_available()]


class BackendUnavailable(Exception):
    def __init__(self, requested: Backend, reason: str):
        super().__init__(f"backend `{requested.label()}` is unavailable: {reason}")
        self.requested = requested
        self.reason = reason


# --------------------------------------------------------------------------
# Parameters and errors (mod.rs:213-420)
# --------------------------------------------------------------------------


class LifParamsError(ValueError):
    def __init__(self, field: str):
        super().__init__(f"LIF parameter `{field}` must be finite")
        self.field = field


@dataclass(frozen=True)
class LifParams:
    """``v <- v * decay + current``; on ``v >= theta`` spike, reset, raise theta."""

    _decay: float
    _v_reset: float
    _delta_theta: float

    @classmethod
    def new(cls, decay: float, v_reset: float, delta_theta: float) -> "LifParams":
        for field, value in (("decay", decay), ("v_reset", v_reset), ("delta_theta", delta_theta)):
            if not math.isfinite(float(np.float32(value))):
                raise LifParamsError(field)
        return cls(float(np.float32(decay)), float(np.float32(v_reset)), float(np.float32(delta_theta)))

    def decay(self) -> float:
        return self._decay

    def v_reset(self) -> float:
        return self._v_reset

    def delta_theta(self) -> float:
        return self._delta_theta


class WeightPrecision(enum.IntEnum):
    F32 = 0
    F16 = 1
    Bf16 = 2

    def bytes(self) -> int:
        return 4 if self is WeightPrecision.F32 else 2

    def epsilon(self) -> float:
        return {WeightPrecision.F32: float(np.finfo(np.float32).eps), WeightPrecision.F16: 9.765625e-4,
                WeightPrecision.Bf16: 7.8125e-3}[self]


class SparsePlanError(Exception):
    """``SparsePlanError`` (mod.rs:277-305); ``kind`` names the variant."""

    def __init__(self, kind: str, message: str, **fields):
        super().__init__(message)
        self.kind = kind
        self.fields = fields

    def __eq__(self, other):
        return isinstance(other, SparsePlanError) and (self.kind, self.fields) == (other.kind, other.fields)

    def __hash__(self):
        return hash(self.kind)


class OpError(Exception):
    """``OpError`` (mod.rs:357-392); ``kind`` names the variant."""

    def __init__(self, kind: str, message: str, **fields):
        super().__init__(message)
        self.kind = kind
        self.fields = fields


def _require_len(what: str, got: int, expected: int):
    if got != expected:
        raise OpError("Length", f"`{what}` must have length {expected}, got {got}", what=what, expected=expected,
                      got=got)


def _require_min_len(what: str, got: int, minimum: int):
    if got < minimum:
        raise OpError("TooShort", f"`{what}` must have length >= {minimum}, got {got}", what=what, min=minimum,
                      got=got)


def _check(rc: int, operation: str):
    """Map a C-ABI status onto the reference's error variants."""
    if rc == _lib.SPARSL_OK:
        return
    detail = _lib.last_error()
    if rc == _lib.SPARSL_ERR_BACKEND:
        raise OpError("Backend", f"backend refused: {detail}", reason=_lib.last_reason())
    if rc == _lib.SPARSL_ERR_EXECUTION:
        raise OpError("Execution", f"{operation}: device execution failed: {detail}", operation=operation,
                      detail=detail)
    if rc == _lib.SPARSL_ERR_NO_TRANSPOSE:
        raise OpError("TransposeNotPrepared", detail)
    if rc == _lib.SPARSL_ERR_LENGTH:
        raise OpError("Length", detail)
    if rc == _lib.SPARSL_ERR_ALLOCATION:
        raise OpError("Backend", f"device allocation failed: {detail}", reason=_lib.last_reason())
    raise OpError("Backend", detail, reason=_lib.last_reason())


# --------------------------------------------------------------------------
# Shapes
# --------------------------------------------------------------------------


@dataclass(frozen=True)
class SparseShape:
    """Validated dimensions (mod.rs:457-503)."""

    _nrows: int
    _ncols: int
    _nnz: int
    _max_row_nnz: int

    def nrows(self) -> int:
        return self._nrows

    def ncols(self) -> int:
        return self._ncols

    def nnz(self) -> int:
        return self._nnz

    def max_row_nnz(self) -> int:
        return self._max_row_nnz

    def nnz_per_row(self) -> int:
        return 0 if self._nrows == 0 else -(-self._nnz // self._nrows)


_PLAN_MESSAGES = {
    1: ("EmptyRowPtr", lambda s: "CSR row_ptr must be non-empty", lambda s: {}),
    2: ("NonZeroStart", lambda s: f"CSR row_ptr must start at 0, got {s.a}", lambda s: {"start": s.a}),
    3: ("NotMonotonic", lambda s: f"CSR row_ptr not monotonic at index {s.a}", lambda s: {"index": s.a}),
    4: ("NnzMismatch", lambda s: f"CSR row_ptr end ({s.a}) != col.len() ({s.b})",
        lambda s: {"row_ptr_end": s.a, "col_len": s.b}),
    5: ("NcolsMismatch", lambda s: f"CSR ncols {s.a} does not match prepare ncols {s.b}",
        lambda s: {"stored": s.a, "declared": s.b}),
    6: ("ColumnOutOfRange", lambda s: f"CSR column index {s.b} at edge {s.a} is out of range (ncols = {s.c})",
        lambda s: {"edge": s.a, "col": s.b, "ncols": s.c}),
    7: ("RowUnsorted", lambda s: f"CSR row {s.a} is unsorted at edge {s.b} (columns must be non-decreasing)",
        lambda s: {"row": s.a, "edge": s.b}),
    8: ("TooLarge", lambda s: f"{('nrows', 'ncols', 'nnz')[s.a]} = {s.b} exceeds the u32 index range of the GPU kernels",
        lambda s: {"what": ("nrows", "ncols", "nnz")[s.a], "value": s.b}),
    9: ("WeightsLen", lambda s: f"weights must have one entry per non-zero: expected {s.a}, got {s.b}",
        lambda s: {"expected": s.a, "got": s.b}),
}


def _plan_error(s: Shape) -> SparsePlanError:
    kind, msg, fields = _PLAN_MESSAGES[s.code]
    return SparsePlanError(kind, msg(s), **fields(s))


# --------------------------------------------------------------------------
# CSR (src/sparse.rs)
# --------------------------------------------------------------------------


class CsrError(ValueError):
    def __init__(self, kind: str, message: str):
        super().__init__(message)
        self.kind = kind


class Csr:
    """CSR connectivity with its declared column count (sparse.rs:80-84)."""

    def __init__(self, row_ptr, col, ncols: int):
        self._row_ptr = np.ascontiguousarray(row_ptr, dtype=np.uint32)
        self._col = np.ascontiguousarray(col, dtype=np.uint32)
        self._ncols = int(ncols)

    @classmethod
    def from_parts(cls, row_ptr, col, ncols: int) -> "Csr":
        """Validated construction (sparse.rs:99-106); raises CsrError."""
        rp = np.ascontiguousarray(row_ptr, dtype=np.uint32)
        c = np.ascontiguousarray(col, dtype=np.uint32)
        sh = Shape()
        _lib.load().sparsl_validate_csr(rp.ctypes.data, rp.size, c.ctypes.data, c.size, int(ncols), int(ncols),
                                        ctypes.byref(sh))
        if sh.code not in (0, 8):
            e = _plan_error(sh)
            raise CsrError(e.kind, str(e))
        return cls(rp, c, ncols)

    @classmethod
    def from_parts_unchecked(cls, row_ptr, col, ncols: int) -> "Csr":
        return cls(row_ptr, col, ncols)

    @classmethod
    def from_adjacency(cls, rows) -> "Csr":
        """sparse.rs:135-172: stable sort per row; ncols = max(nrows, max col + 1)."""
        row_ptr = np.zeros(len(rows) + 1, np.uint64)
        parts = []
        max_col = -1
        for i, r in enumerate(rows):
            a = np.sort(np.asarray(r, dtype=np.uint32), kind="stable")
            parts.append(a)
            if a.size:
                max_col = max(max_col, int(a[-1]))
            row_ptr[i + 1] = row_ptr[i] + a.size
        if row_ptr[-1] > 0xFFFFFFFF:
            raise OverflowError("CSR adjacency has more non-zeros than u32 offsets can represent")
        col = np.concatenate(parts) if parts else np.zeros(0, np.uint32)
        nrows = len(rows)
        ncols = nrows if max_col < 0 else max(nrows, max_col + 1)
        return cls(row_ptr.astype(np.uint32), col, ncols)

    @classmethod
    def empty(cls, nrows: int, ncols: int) -> "Csr":
        return cls(np.zeros(nrows + 1, np.uint32), np.zeros(0, np.uint32), ncols)

    def row_ptr(self):
        return self._row_ptr

    def col(self):
        return self._col

    def nrows(self) -> int:
        return max(self._row_ptr.size - 1, 0)

    def nnz(self) -> int:
        return self._col.size

    def ncols(self) -> int:
        return self._ncols


# --------------------------------------------------------------------------
# Helpers
# --------------------------------------------------------------------------


def _ptr(a) -> int:
    return a.ctypes.data if a is not None and a.size else 0


def _in(a, dtype, name: str):
    arr = np.ascontiguousarray(a, dtype=dtype)
    return arr


def _out(a, dtype, name: str):
    if not isinstance(a, np.ndarray) or a.dtype != dtype or not a.flags.c_contiguous or not a.flags.writeable:
        raise TypeError(f"`{name}` must be a writable C-contiguous numpy array of {np.dtype(dtype).name}")
    return a


def packed_len(n: int) -> int:
    """spikes.rs packed_len: 32 spikes per u32 word."""
    return (int(n) + 31) // 32


def pack_spikes(spikes) -> np.ndarray:
    """LSB-first packing, tail bits zero (src/spikes.rs:207-235): spike i is
    bit i % 32 of word i // 32.  Little-endian bit order within each byte,
    read as little-endian words, is exactly that layout."""
    s = np.asarray(spikes, dtype=bool).reshape(-1)
    n = s.size
    pad = packed_len(n) * 32 - n
    if pad:
        s = np.concatenate([s, np.zeros(pad, dtype=bool)])
    return np.packbits(s, bitorder="little").view("<u4").astype(np.uint32, copy=False)


def unpack_spikes(words, n: int) -> np.ndarray:
    w = np.asarray(words, dtype=np.uint32)
    if w.size < packed_len(n):
        raise ValueError(f"sparsl: {w.size} words cannot hold {n} spikes")
    b = np.ascontiguousarray(w[: packed_len(n)]).astype("<u4", copy=False).view(np.uint8)
    return np.unpackbits(b, bitorder="little")[:n].astype(bool)


def spikes_to_f32(words, n: int) -> np.ndarray:
    return unpack_spikes(words, n).astype(np.float32)


# --------------------------------------------------------------------------
# Device
# --------------------------------------------------------------------------


class Device:
    """A handle to a CUDA device that was available when it was opened."""

    def __init__(self, backend: Backend, handle, ordinal: int):
        self._backend = backend
        self._h = handle
        self._ordinal = ordinal

    @classmethod
    def try_new(cls, backend: Backend, ordinal: int = 0) -> "Device":
        """Open ``backend`` or explain why not; never falls back (mod.rs:882-917)."""
        reason = backend.unavailable_reason()
        if reason is not None:
            raise BackendUnavailable(backend, reason)
        if backend is not Backend.Cuda:
            # Unreachable: only CUDA reports available in this package.  Kept
            # as a hard stop rather than a CPU device under another label.
            raise BackendUnavailable(backend, "backend opened a different substrate than requested")
        h = ctypes.c_void_p()
        rc = _lib.load().sparsl_device_open(int(ordinal), ctypes.byref(h))
        if rc != 0:
            raise BackendUnavailable(backend, _lib.last_error())
        return cls(backend, h, ordinal)

    def __del__(self):
        # Device handles are shared by operators; the process keeps them.
        pass

    def backend(self) -> Backend:
        return self._backend

    def label(self) -> str:
        return self._backend.label()

    def device_name(self):
        buf = ctypes.create_string_buffer(256)
        _check(_lib.load().sparsl_device_name(self._h, buf, 256), "device_name")
        return buf.value.decode()

    @property
    def handle(self):
        return self._h

    @staticmethod
    def reset_cuda() -> None:
        """Clear the quarantine once no call is admitted (mod.rs:825-843)."""
        rc = _lib.load().sparsl_device_reset()
        if rc != 0:
            raise OpError("Backend", _lib.last_error(), reason=_lib.last_reason())

    # ---- prepare family (mod.rs:966-1121) ----
    def prepare(self, csr: Csr, ncols: int, weights) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, False, WeightPrecision.F32)

    def prepare_f16(self, csr: Csr, ncols: int, weights) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, False, WeightPrecision.F16)

    def prepare_bf16(self, csr: Csr, ncols: int, weights) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, False, WeightPrecision.Bf16)

    def prepare_with(self, csr: Csr, ncols: int, weights, precision: WeightPrecision) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, False, precision)

    def prepare_with_transpose(self, csr: Csr, ncols: int, weights) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, True, WeightPrecision.F32)

    def prepare_with_transpose_precision(self, csr: Csr, ncols: int, weights,
                                         precision: WeightPrecision) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, True, precision)

    def prepare_f16_with_transpose(self, csr: Csr, ncols: int, weights) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, True, WeightPrecision.F16)

    def prepare_bf16_with_transpose(self, csr: Csr, ncols: int, weights) -> "SparseOp":
        return SparseOp._prepare(self, csr, ncols, weights, True, WeightPrecision.Bf16)

    def csc_from_csr_device(self, row_ptr, col, ncols: int, col_ptr, row, edge_idx) -> None:
        """``Csc::from_csr_slices`` (sparse.rs:361-427) on the GPU.

        Inputs and outputs are 32-bit device arrays of this GPU (torch tensors
        or objects with ``data_ptr()`` / ``numel()``): ``col_ptr`` holds
        ``ncols + 1`` entries, ``row`` and ``edge_idx`` one per edge.  The CSR
        passes the same gate as ``prepare`` first (SparsePlanError)."""
        torch = sys.modules.get("torch")
        if torch is not None and isinstance(col, torch.Tensor) and col.is_cuda:
            torch.cuda.synchronize(col.device)
        sh = Shape()
        rc = _lib.load().sparsl_csc_from_csr_device(self._h, row_ptr.data_ptr(), row_ptr.numel(), col.data_ptr(),
                                                    col.numel(), int(ncols), col_ptr.data_ptr(), row.data_ptr(),
                                                    edge_idx.data_ptr(), ctypes.byref(sh))
        if rc == _lib.SPARSL_ERR_INVALID and sh.code != 0:
            raise _plan_error(sh)
        if rc != 0:
            raise SparsePlanError("Backend", f"backend refused: {_lib.last_error()}", reason=_lib.last_reason())

    def prepare_device(self, row_ptr, col, ncols: int, weights, precision: WeightPrecision = WeightPrecision.F32,
                       transpose: bool = False, csr_ncols: Optional[int] = None) -> "SparseOp":
        """``prepare_with`` / ``prepare_with_transpose_precision`` for a CSR whose
        arrays already live on this GPU; the same gate, errors and operator.
        ``csr_ncols`` is the CSR's own column count (defaults to ``ncols``)."""
        return SparseOp._prepare_device(self, row_ptr, col, ncols if csr_ncols is None else csr_ncols, ncols,
                                        weights, transpose, precision)

    def prepare_device_borrowed(self, row_ptr, col, ncols: int, weights, transpose: bool = False,
                                csr_ncols: Optional[int] = None) -> "SparseOp":
        """``prepare_device`` in f32 where the operator uses the caller's
        arrays in place instead of copying them (extension: for operators too
        large to hold twice).  Each tensor must start on a 256-byte boundary
        and be followed by 256 bytes of its allocation; the operator keeps
        references to the tensors, and ``set_weights`` writes into
        ``weights``.  Keep ``row_ptr`` and ``col`` unchanged."""
        return SparseOp._prepare_device(self, row_ptr, col, ncols if csr_ncols is None else csr_ncols, ncols,
                                        weights, transpose, WeightPrecision.F32, borrow=True)

    # ---- device-level ops ----
    def assoc_scan(self, xs) -> np.ndarray:
        """Inclusive scan of (a, b) maps, bit-identical to assoc_scan_sequential.

        ``xs`` is an (n, 2) float32 array of ``State`` pairs (scan.rs:78-96).
        """
        a = np.ascontiguousarray(xs, dtype=np.float32).reshape(-1, 2)
        out = np.empty_like(a)
        if a.shape[0] == 0:
            return out
        _check(_lib.load().sparsl_dev_assoc_scan(self._h, a.ctypes.data, a.shape[0], out.ctypes.data),
               "assoc_scan")
        return out

    def wait(self) -> None:
        """Bounded wait for the device's own stream, then its error word."""
        _check(_lib.load().sparsl_dev_wait(self._h), "device wait")

    def stream_handle(self) -> int:
        """The device's own stream (cudaStream_t) as an integer."""
        return _lib.load().sparsl_dev_stream(self._h) or 0

    # ---- a scan split into runs across devices (extension) ----
    def assoc_scan_from_device(self, d_in, n: int, d_out, entry=None, stream=None) -> None:
        """Exact scan of n device-resident maps that continue a sequence whose
        state before ``d_in[0]`` is ``entry`` ((a, b), or None: the run starts
        the sequence).  Enqueued on ``stream`` (a cudaStream_t, None = the
        device's own)."""
        e = None if entry is None else np.asarray(entry, np.float32)
        _check(_lib.load().sparsl_dev_assoc_scan_from_device(self._h, _dptr(d_in), int(n), _dptr(d_out),
                                                             None if e is None else e.ctypes.data, stream),
               "assoc_scan")

    def scan_fold_device(self, d_in, n: int, entry=None, stream=None) -> np.ndarray:
        """The (a, b) state after folding n device maps (serial, synchronous)."""
        e = None if entry is None else np.asarray(entry, np.float32)
        out = np.zeros(2, np.float32)
        _check(_lib.load().sparsl_dev_scan_fold_device(self._h, _dptr(d_in), int(n),
                                                       None if e is None else e.ctypes.data, out.ctypes.data,
                                                       stream), "scan_fold")
        return out

    def scan_rejoin_device(self, d_in, d_out, n: int, entry, stream=None):
        """Rewrite a run's output from its exact entry state until it rejoins
        the stored trajectory; returns (exit state, rewritten maps)."""
        e = np.asarray(entry, np.float32)
        out = np.zeros(2, np.float32)
        cnt = ctypes.c_uint64()
        _check(_lib.load().sparsl_dev_scan_rejoin_device(self._h, _dptr(d_in), _dptr(d_out), int(n), e.ctypes.data,
                                                         out.ctypes.data, ctypes.byref(cnt), stream), "scan_rejoin")
        return out, cnt.value

    def scan_table_device(self, d_in, n: int, stream=None) -> int:
        """Transfer table (8 nibbles) of n device maps for the multiplier chain."""
        t = ctypes.c_uint32()
        _check(_lib.load().sparsl_dev_scan_table_device(self._h, _dptr(d_in), int(n), ctypes.byref(t), stream),
               "scan_table")
        return t.value

    def scan_settle_device(self, d_in, n: int, stream=None):
        """(multiplier, maps folded): the multiplier chain from a copy of the
        first map until it settles in {0..7} * 2^-149 or the run ends."""
        a = ctypes.c_float()
        k = ctypes.c_uint64()
        _check(_lib.load().sparsl_dev_scan_settle_device(self._h, _dptr(d_in), int(n), ctypes.byref(a),
                                                         ctypes.byref(k), stream), "scan_settle")
        return np.float32(a.value), int(k.value)

    def scan_publish_device(self, d_in, n: int, first: bool, halo: int, d_blob, stream=None) -> None:
        """Enqueue a run's published blob (halo, multiplier table, first run's
        exit multiplier) into ``d_blob`` (2*halo + 4 floats)."""
        _check(_lib.load().sparsl_dev_scan_publish_device(self._h, _dptr(d_in), int(n), int(bool(first)), int(halo),
                                                          _dptr(d_blob), stream), "scan_publish")

    def scan_entry_device(self, d_gathered, world: int, rank: int, halo: int, d_entry, stream=None) -> None:
        """Enqueue run ``rank``'s guessed entry state (2 floats) from the
        gathered blobs of every run."""
        _check(_lib.load().sparsl_dev_scan_entry_device(self._h, _dptr(d_gathered), int(world), int(rank), int(halo),
                                                        _dptr(d_entry), stream), "scan_entry")

    def assoc_scan_after_device(self, d_in, n: int, d_out, d_entry, stream=None) -> None:
        """Enqueue the scan of a run whose entry state is in device memory."""
        _check(_lib.load().sparsl_dev_assoc_scan_after_device(self._h, _dptr(d_in), int(n), _dptr(d_out),
                                                              _dptr(d_entry), stream), "assoc_scan")

    def scan_stats(self):
        rep, seg = ctypes.c_uint64(), ctypes.c_uint64()
        _check(_lib.load().sparsl_dev_scan_stats(self._h, ctypes.byref(rep), ctypes.byref(seg)), "scan_stats")
        return rep.value, seg.value

    def lif_integrate(self, v, theta, currents, spikes, params: LifParams) -> None:
        """Standalone LIF over dense currents (mod.rs:1202-1229)."""
        n = len(v)
        _require_len("theta", len(theta), n)
        _require_len("currents", len(currents), n)
        _require_len("spikes", len(spikes), n)
        if n == 0:
            return
        v = _out(v, np.float32, "v")
        theta = _out(theta, np.float32, "theta")
        cur = _in(currents, np.float32, "currents")
        sp = _spike_view(spikes)
        _check(_lib.load().sparsl_dev_lif_integrate(self._h, v.ctypes.data, theta.ctypes.data, cur.ctypes.data,
                                                    sp.ctypes.data, n, params.decay(), params.v_reset(),
                                                    params.delta_theta()), "lif_integrate")


def _spike_view(spikes):
    """A bool/uint8 numpy array viewed as uint8 (Rust bool is one byte 0/1)."""
    if not isinstance(spikes, np.ndarray) or spikes.dtype not in (np.bool_, np.uint8) or \
            not spikes.flags.c_contiguous or not spikes.flags.writeable:
        raise TypeError("`spikes` must be a writable C-contiguous numpy array of bool or uint8")
    return spikes.view(np.uint8)


def _dptr(buffer):
    return None if buffer is None else buffer.data_ptr()


def _event_handle(event):
    if event is None:
        return None
    if isinstance(event, int):
        return event
    return getattr(event, "cuda_event")  # torch.cuda.Event


class DeviceBuffer:
    """Device memory returned by ``SparseOp.alloc_cuda_f32`` (freed on ``free``
    or garbage collection)."""

    def __init__(self, ptr: int, n: int):
        self._ptr, self._n = ptr, n

    def data_ptr(self) -> int:
        return self._ptr

    def numel(self) -> int:
        return self._n

    def element_size(self) -> int:
        return 4

    def to_numpy(self) -> np.ndarray:
        out = np.empty(self._n, np.float32)
        if self._n:
            _check(_lib.load().sparsl_memcpy(out.ctypes.data, self._ptr, out.nbytes), "memcpy")
        return out

    def free(self) -> None:
        if self._ptr:
            _lib.load().sparsl_device_free(self._ptr)
            self._ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class _PinnedBlock:
    """Owns one sparsl_host_alloc block; freed when the last reference goes."""

    def __init__(self, ptr: int):
        self.ptr = ptr

    def release(self) -> None:
        if self.ptr:
            _lib.load().sparsl_host_free(self.ptr)
            self.ptr = 0

    def __del__(self):
        try:
            self.release()
        except Exception:
            pass


class HostBuffer:
    """Page-locked host memory that the GPU can address (``sparsl_host_alloc``),
    as a numpy array (``.array``).  Passed as ``y`` of ``spmv`` /
    ``spmv_spikes``, or as ``v``, ``theta`` and the spike bytes of the fused
    LIF calls (all three), it is read and written in place by the kernels over
    PCIe instead of being staged through device copies; the results are the
    same bit for bit.  The memory lives while the buffer or any view of it
    does."""

    def __init__(self, n: int, dtype=np.float32):
        dt = np.dtype(dtype)
        n = int(n)
        nbytes = max(n * dt.itemsize, 16)
        ptr = _lib.load().sparsl_host_alloc(nbytes)
        if not ptr:
            raise OpError("Backend", "page-locked host allocation failed (is a CUDA device present?)",
                          reason="host allocation failed")
        buf = (ctypes.c_char * nbytes).from_address(ptr)
        buf._block = _PinnedBlock(ptr)  # every view of buf keeps the block alive
        self._buf = buf
        self.array = np.frombuffer(buf, dtype=dt, count=n)

    def data_ptr(self) -> int:
        return ctypes.addressof(self._buf)


# --------------------------------------------------------------------------
# SparseOp (mod.rs:1281-2108)
# --------------------------------------------------------------------------


class SparseOp:
    """A CSR operator validated against ``ncols`` and resident on the GPU."""

    def __init__(self, device: Device, handle, shape: SparseShape, precision: WeightPrecision):
        self._device = device
        self._h = handle
        self._shape = shape
        self._precision = precision

    @classmethod
    def _prepare(cls, device: Device, csr: Csr, ncols: int, weights, transpose: bool,
                 precision: WeightPrecision) -> "SparseOp":
        rp = csr.row_ptr()
        col = csr.col()
        w = np.ascontiguousarray(weights, dtype=np.float32)
        sh = Shape()
        h = ctypes.c_void_p()
        rc = _lib.load().sparsl_op_prepare(device.handle, _ptr(rp), rp.size, _ptr(col), col.size, csr.ncols(),
                                           int(ncols), _ptr(w), w.size, int(precision), int(transpose),
                                           ctypes.byref(sh), ctypes.byref(h))
        return cls._finish(device, rc, sh, h, precision)

    @classmethod
    def _prepare_device(cls, device: Device, row_ptr, col, csr_ncols: int, ncols: int, weights, transpose: bool,
                        precision: WeightPrecision, borrow: bool = False) -> "SparseOp":
        """``prepare`` from arrays already on the GPU (sparsl_op_prepare_device).

        ``row_ptr`` and ``col`` are 32-bit integer tensors and ``weights`` a
        float32 tensor, contiguous, on this device (torch tensors or any object
        with ``data_ptr()``, ``numel()`` and ``element_size()``).  Torch work
        that writes them is synchronised first.
        """
        for name, t, size in (("row_ptr", row_ptr, 4), ("col", col, 4), ("weights", weights, 4)):
            if t.element_size() != size:
                raise SparsePlanError("Backend", f"{name} must have {size}-byte elements", reason=name)
            if hasattr(t, "is_contiguous") and not t.is_contiguous():
                raise SparsePlanError("Backend", f"{name} must be contiguous", reason=name)
        torch = sys.modules.get("torch")
        if torch is not None and isinstance(weights, torch.Tensor) and weights.is_cuda:
            torch.cuda.synchronize(weights.device)
        sh = Shape()
        h = ctypes.c_void_p()
        if borrow:
            rc = _lib.load().sparsl_op_prepare_device_borrowed(
                device.handle, row_ptr.data_ptr(), row_ptr.numel(), col.data_ptr(), col.numel(), int(csr_ncols),
                int(ncols), weights.data_ptr(), weights.numel(), int(transpose), ctypes.byref(sh), ctypes.byref(h))
            op = cls._finish(device, rc, sh, h, precision)
            op._borrowed = (row_ptr, col, weights)  # alive as long as the operator
            return op
        rc = _lib.load().sparsl_op_prepare_device(device.handle, row_ptr.data_ptr(), row_ptr.numel(), col.data_ptr(),
                                                  col.numel(), int(csr_ncols), int(ncols), weights.data_ptr(),
                                                  weights.numel(), int(precision), int(transpose), ctypes.byref(sh),
                                                  ctypes.byref(h))
        return cls._finish(device, rc, sh, h, precision)

    @classmethod
    def _finish(cls, device: Device, rc: int, sh, h, precision: WeightPrecision) -> "SparseOp":
        if rc == _lib.SPARSL_ERR_INVALID and sh.code != 0:
            raise _plan_error(sh)
        if rc == _lib.SPARSL_ERR_ALLOCATION:
            raise SparsePlanError("Allocation", f"device allocation failed for {_lib.last_reason()}",
                                  what=_lib.last_reason())
        if rc != 0:
            raise SparsePlanError("Backend", f"backend refused: {_lib.last_error()}", reason=_lib.last_reason())
        return cls(device, h, SparseShape(sh.nrows, sh.ncols, sh.nnz, sh.max_row_nnz), precision)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            try:
                _lib.load().sparsl_op_destroy(h)
            except Exception:
                pass
            self._h = None

    @property
    def handle(self):
        return self._h

    def backend(self) -> Backend:
        return self._device.backend()

    def label(self) -> str:
        return self._device.label()

    def shape(self) -> SparseShape:
        return self._shape

    def weight_precision(self) -> WeightPrecision:
        return WeightPrecision(_lib.load().sparsl_op_weight_precision(self._h))

    def layouts(self) -> int:
        """SPARSL_LAYOUT_* bits: the device layouts this operator holds."""
        return int(_lib.load().sparsl_op_layouts(self._h))

    def force_plain_row_fold(self) -> None:
        """Route later forward products through the generic row-fold engine
        (a test hook that compares both engines on one operator)."""
        _check(_lib.load().sparsl_op_force_plain_row_fold(self._h), "force_plain_row_fold")

    def has_transpose(self) -> bool:
        return bool(_lib.load().sparsl_op_has_transpose(self._h))

    def set_weights(self, weights) -> None:
        w = np.ascontiguousarray(weights, dtype=np.float32)
        _require_len("weights", w.size, self._shape.nnz())
        _check(_lib.load().sparsl_op_set_weights(self._h, _ptr(w), w.size), "set_weights")

    # ---- slice API ----
    def spmv(self, x, y) -> None:
        """``y += A x`` (mod.rs:1411-1429)."""
        s = self._shape
        _require_min_len("x", len(x), s.ncols())
        _require_len("y", len(y), s.nrows())
        if s.nrows() == 0:
            return
        x = _in(x, np.float32, "x")
        y = _out(y, np.float32, "y")
        _check(_lib.load().sparsl_op_spmv(self._h, _ptr(x), x.size, y.ctypes.data, y.size), "spmv")

    def spmv_spikes(self, spikes, y) -> None:
        """``y += A s`` for a bit-packed spike vector (mod.rs:1449-1468)."""
        s = self._shape
        _require_min_len("spikes", len(spikes), packed_len(s.ncols()))
        _require_len("y", len(y), s.nrows())
        if s.nrows() == 0:
            return
        sp = _in(spikes, np.uint32, "spikes")
        y = _out(y, np.float32, "y")
        _check(_lib.load().sparsl_op_spmv_spikes(self._h, _ptr(sp), sp.size, y.ctypes.data, y.size),
               "spmv_spikes")

    def spmv_t(self, x, y) -> None:
        """``y += A^T x`` (mod.rs:1486-1505)."""
        s = self._shape
        _require_min_len("x", len(x), s.nrows())
        _require_len("y", len(y), s.ncols())
        if s.ncols() == 0:
            return
        if not self.has_transpose():
            raise OpError("TransposeNotPrepared",
                          "this operator has no reverse index; build it with `Device::prepare_with_transpose` "
                          "to use `spmv_t`")
        x = _in(x, np.float32, "x")
        y = _out(y, np.float32, "y")
        _check(_lib.load().sparsl_op_spmv_t(self._h, _ptr(x), x.size, y.ctypes.data, y.size), "spmv_t")

    def spmm(self, x, n_vec: int, y) -> None:
        """``Y += A X``, batch-minor (mod.rs:1528-1571)."""
        s = self._shape
        if n_vec == 0:
            raise OpError("Length", "`n_vec` must have length 1, got 0", what="n_vec", expected=1, got=0)
        limit = (1 << 64) - 1
        if s.ncols() and n_vec > limit // s.ncols():
            raise OpError("SizeOverflow", "SpMM input element count overflowed usize",
                          what="SpMM input element count", lhs=s.ncols(), rhs=n_vec)
        if s.nrows() and n_vec > limit // s.nrows():
            raise OpError("SizeOverflow", "SpMM output element count overflowed usize",
                          what="SpMM output element count", lhs=s.nrows(), rhs=n_vec)
        _require_min_len("x", len(x), s.ncols() * n_vec)
        _require_len("y", len(y), s.nrows() * n_vec)
        if s.nrows() == 0:
            return
        x = _in(x, np.float32, "x")
        y = _out(y, np.float32, "y")
        _check(_lib.load().sparsl_op_spmm(self._h, _ptr(x), x.size, int(n_vec), y.ctypes.data, y.size), "spmm")

    def fused_spmv_lif(self, x, v, theta, spikes, params: LifParams) -> None:
        """``current = A x`` then the LIF step, fused (mod.rs:1609-1636)."""
        s = self._shape
        _require_min_len("x", len(x), s.ncols())
        _require_len("v", len(v), s.nrows())
        _require_len("theta", len(theta), s.nrows())
        _require_len("spikes", len(spikes), s.nrows())
        if s.nrows() == 0:
            return
        x = _in(x, np.float32, "x")
        v = _out(v, np.float32, "v")
        theta = _out(theta, np.float32, "theta")
        sp = _spike_view(spikes)
        _check(_lib.load().sparsl_op_fused_lif(self._h, _ptr(x), x.size, v.ctypes.data, theta.ctypes.data,
                                               sp.ctypes.data, v.size, params.decay(), params.v_reset(),
                                               params.delta_theta()), "fused_spmv_lif")

    def fused_spmv_spikes_lif(self, spikes_in, v, theta, spikes_out, params: LifParams) -> None:
        """Spike-vector variant (mod.rs:1644-1678)."""
        s = self._shape
        _require_min_len("spikes_in", len(spikes_in), packed_len(s.ncols()))
        _require_len("v", len(v), s.nrows())
        _require_len("theta", len(theta), s.nrows())
        _require_len("spikes_out", len(spikes_out), s.nrows())
        if s.nrows() == 0:
            return
        si = _in(spikes_in, np.uint32, "spikes_in")
        v = _out(v, np.float32, "v")
        theta = _out(theta, np.float32, "theta")
        so = _spike_view(spikes_out)
        _check(_lib.load().sparsl_op_fused_spikes_lif(self._h, _ptr(si), si.size, v.ctypes.data, theta.ctypes.data,
                                                      so.ctypes.data, v.size, params.decay(), params.v_reset(),
                                                      params.delta_theta()), "fused_spmv_spikes_lif")

    # ---- resident API (mod.rs:1680-1973) ----
    def write_x(self, x) -> None:
        _require_min_len("x", len(x), self._shape.ncols())
        x = _in(x, np.float32, "x")
        _check(_lib.load().sparsl_op_write_x(self._h, _ptr(x), x.size), "write_x")

    def write_x_spikes(self, spikes) -> None:
        _require_min_len("spikes", len(spikes), packed_len(self._shape.ncols()))
        s = _in(spikes, np.uint32, "spikes")
        _check(_lib.load().sparsl_op_write_x_spikes(self._h, _ptr(s), s.size), "write_x_spikes")

    def write_y(self, y) -> None:
        _require_len("y", len(y), self._shape.nrows())
        y = _in(y, np.float32, "y")
        _check(_lib.load().sparsl_op_write_y(self._h, _ptr(y), y.size), "write_y")

    def write_lif_state(self, v, theta) -> None:
        _require_len("v", len(v), self._shape.nrows())
        _require_len("theta", len(theta), self._shape.nrows())
        v = _in(v, np.float32, "v")
        th = _in(theta, np.float32, "theta")
        _check(_lib.load().sparsl_op_write_lif_state(self._h, _ptr(v), _ptr(th), v.size), "write_lif_state")

    def spmv_resident(self) -> None:
        if self._shape.nrows() == 0:
            return
        _check(_lib.load().sparsl_op_spmv_resident(self._h), "spmv_resident")

    def fused_spmv_lif_resident(self, params: LifParams) -> None:
        if self._shape.nrows() == 0:
            return
        _check(_lib.load().sparsl_op_fused_lif_resident(self._h, params.decay(), params.v_reset(),
                                                        params.delta_theta()), "fused_spmv_lif_resident")

    def fused_spmv_spikes_lif_resident(self, params: LifParams) -> None:
        if self._shape.nrows() == 0:
            return
        _check(_lib.load().sparsl_op_fused_spikes_lif_resident(self._h, params.decay(), params.v_reset(),
                                                               params.delta_theta()),
               "fused_spmv_spikes_lif_resident")

    def pack_resident_spikes_to_x_spikes(self) -> None:
        _require_len("recurrent nrows", self._shape.nrows(), self._shape.ncols())
        if self._shape.nrows() == 0:
            return
        _check(_lib.load().sparsl_op_pack_resident_spikes(self._h), "pack_resident_spikes_to_x_spikes")

    def fused_spmv_spikes_lif_recurrent_steps(self, params: LifParams, steps: int) -> None:
        _require_len("recurrent nrows", self._shape.nrows(), self._shape.ncols())
        if steps == 0 or self._shape.nrows() == 0:
            return
        _check(_lib.load().sparsl_op_recurrent_steps(self._h, params.decay(), params.v_reset(),
                                                     params.delta_theta(), int(steps)),
               "fused_spmv_spikes_lif_recurrent_steps")

    def sync_y(self, y) -> None:
        _require_len("y", len(y), self._shape.nrows())
        y = _out(y, np.float32, "y")
        _check(_lib.load().sparsl_op_sync_y(self._h, _ptr(y), y.size), "sync_y")

    def sync_lif_state(self, v, theta, spikes) -> None:
        n = self._shape.nrows()
        _require_len("v", len(v), n)
        _require_len("theta", len(theta), n)
        _require_len("spikes", len(spikes), n)
        v = _out(v, np.float32, "v")
        theta = _out(theta, np.float32, "theta")
        sp = _spike_view(spikes)
        _check(_lib.load().sparsl_op_sync_lif_state(self._h, _ptr(v), _ptr(theta), _ptr(sp), n),
               "sync_lif_state")

    # ---- zero-copy interop (mod.rs:1975-2098) ----
    def bind_cuda_x(self, buffer) -> None:
        """``bind_mtl_x``: a caller device buffer (torch tensor, DeviceBuffer or
        anything with ``data_ptr()``) of at least ncols f32 becomes this
        operator's x.  The caller keeps it alive while bound."""
        _check(_lib.load().sparsl_op_bind_x(self._h, _dptr(buffer)), "bind_x")

    def bind_cuda_y(self, buffer) -> None:
        """``bind_mtl_y``: a caller device buffer of at least nrows f32 becomes y."""
        _check(_lib.load().sparsl_op_bind_y(self._h, _dptr(buffer)), "bind_y")

    def unbind_cuda_x(self) -> None:
        _check(_lib.load().sparsl_op_unbind_x(self._h), "unbind_x")

    def unbind_cuda_y(self) -> None:
        _check(_lib.load().sparsl_op_unbind_y(self._h), "unbind_y")

    def cuda_x_gpu_address(self) -> int:
        out = ctypes.c_uint64()
        _check(_lib.load().sparsl_op_x_address(self._h, ctypes.byref(out)), "x_address")
        return out.value

    def cuda_y_gpu_address(self) -> int:
        out = ctypes.c_uint64()
        _check(_lib.load().sparsl_op_y_address(self._h, ctypes.byref(out)), "y_address")
        return out.value

    def alloc_cuda_f32(self, data) -> "DeviceBuffer":
        """``alloc_mtl_f32``: an f32 device buffer on this operator's GPU holding ``data``."""
        a = np.ascontiguousarray(data, dtype=np.float32)
        out = ctypes.c_void_p()
        _check(_lib.load().sparsl_op_alloc_f32(self._h, _ptr(a) if a.size else None, a.size, ctypes.byref(out)),
               "alloc_f32")
        return DeviceBuffer(out.value, a.size)

    def wait_cuda_event(self, event, timeout_ms: int) -> None:
        """``wait_shared_event`` for a CUDA event (torch.cuda.Event or a raw
        cudaEvent_t): device-side ordering plus a bounded host wait."""
        _check(_lib.load().sparsl_op_wait_event(self._h, _event_handle(event), int(timeout_ms)), "wait_event")

    def signal_cuda_event(self, event) -> None:
        """``signal_shared_event``: records the (already created) CUDA event on
        this operator's stream, after all of its enqueued work."""
        _check(_lib.load().sparsl_op_signal_event(self._h, _event_handle(event)), "signal_event")

    # ---- extensions: tick trace ----
    def sync_x_spikes(self) -> np.ndarray:
        out = np.zeros(max(packed_len(self._shape.ncols()), 1), np.uint32)
        _check(_lib.load().sparsl_op_sync_x_spikes(self._h, out.ctypes.data, out.size), "sync_x_spikes")
        return out[: packed_len(self._shape.ncols())]

    def spike_trace(self) -> np.ndarray:
        n = ctypes.c_uint64()
        _check(_lib.load().sparsl_op_spike_trace(self._h, 0, 0, ctypes.byref(n)), "spike_trace")
        out = np.zeros(max(n.value, 1), np.uint32)
        _check(_lib.load().sparsl_op_spike_trace(self._h, out.ctypes.data, out.size, ctypes.byref(n)),
               "spike_trace")
        return out[: n.value]

    def spike_indices(self) -> np.ndarray:
        out = np.zeros(max(self._shape.nrows(), 1), np.uint32)
        cnt = ctypes.c_uint64()
        _check(_lib.load().sparsl_op_spike_indices(self._h, out.ctypes.data, out.size, ctypes.byref(cnt)),
               "spike_indices")
        return out[: cnt.value]


# --------------------------------------------------------------------------
# Tolerances (mod.rs:533-769; scan.rs:160-188)
# --------------------------------------------------------------------------

_EPS = np.float32(np.finfo(np.float32).eps)
_MINPOS = np.float32(np.finfo(np.float32).tiny)


def _fmax(a, b):
    a = np.float32(a)
    return b if not (a >= b) else a


def tolerance_for_elementwise(max_abs_operand: float) -> float:
    mag = _fmax(abs(np.float32(max_abs_operand)), _MINPOS)
    return float(np.float32(2.0) * _EPS * mag)


def tolerance_for_spmv(max_row_nnz: int, max_abs_term: float, max_abs_result: float) -> float:
    n = np.float32(max(int(max_row_nnz), 1))
    term = _fmax(abs(np.float32(max_abs_term)), _MINPOS)
    result = _fmax(abs(np.float32(max_abs_result)), _MINPOS)
    fused = np.float32(np.float64(n) * np.float64(term) + np.float64(result))  # mul_add rounds once
    return float(np.float32(8.0) * _EPS * fused)


def tolerance_for_spmv_narrow(precision: WeightPrecision, max_row_nnz: int, max_abs_term: float,
                              max_abs_result: float) -> float:
    n = np.float32(max(int(max_row_nnz), 1))
    term = _fmax(abs(np.float32(max_abs_term)), _MINPOS)
    acc = np.float32(tolerance_for_spmv(max_row_nnz, max_abs_term, max_abs_result))
    if precision is WeightPrecision.F32:
        return float(acc)
    return float(np.float32(8.0) * n * np.float32(precision.epsilon()) * term + acc)


def tolerance_for_spmv_f16(max_row_nnz, max_abs_term, max_abs_result):
    return tolerance_for_spmv_narrow(WeightPrecision.F16, max_row_nnz, max_abs_term, max_abs_result)


def tolerance_for_spmv_bf16(max_row_nnz, max_abs_term, max_abs_result):
    return tolerance_for_spmv_narrow(WeightPrecision.Bf16, max_row_nnz, max_abs_term, max_abs_result)


def tolerance_for_scan(prefix_len: int, magnitude_envelope: float) -> float:
    env = np.float32(magnitude_envelope)
    if not np.isfinite(env):
        return float(abs(env))
    n = np.float32(max(int(prefix_len), 1))
    mag = _fmax(abs(env), np.float32(1.0))
    return float(np.float32(8.0) * _EPS * n * mag)


def scan_magnitude_envelope(xs) -> float:
    a = np.asarray(xs, dtype=np.float32).reshape(-1, 2)
    suffix_a, prefix_b, env = 1.0, 0.0, 1.0
    for ai, bi in a.astype(np.float64):
        ai, bi = abs(ai), abs(bi)
        if not (math.isfinite(ai) and math.isfinite(bi)):
            return float("inf")
        suffix_a = ai * max(suffix_a, 1.0)
        prefix_b = ai * prefix_b + bi
        if not (math.isfinite(suffix_a) and math.isfinite(prefix_b)):
            return float("inf")
        env = max(env, suffix_a, prefix_b)
    r = np.float32(env)
    if not np.isfinite(r) or float(r) >= env:
        return float(r)
    return float(np.nextafter(r, np.float32(np.inf)))


# --------------------------------------------------------------------------
# Narrow codecs (half.rs), native
# --------------------------------------------------------------------------


def f32_to_f16_bits(values) -> np.ndarray:
    a = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(a.size, np.uint16)
    if a.size:
        _lib.load().sparsl_f32_to_f16_bits(a.ctypes.data, out.ctypes.data, a.size)
    return out


def f32_to_bf16_bits(values) -> np.ndarray:
    a = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty(a.size, np.uint16)
    if a.size:
        _lib.load().sparsl_f32_to_bf16_bits(a.ctypes.data, out.ctypes.data, a.size)
    return out


def quantise(precision: WeightPrecision, values) -> np.ndarray:
    a = np.ascontiguousarray(values, dtype=np.float32)
    out = np.empty_like(a)
    if a.size:
        _lib.load().sparsl_quantise(int(precision), a.ctypes.data, out.ctypes.data, a.size)
    return out

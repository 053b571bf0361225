"""ctypes view of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle is a plain-C restatement of the reference crate's CPU sequential
and CPU parallel arms (bharathvbcr/sparsl 0.3.0, ``src/backend/mod.rs``,
``src/scan.rs``, ``src/spikes.rs``, ``src/half.rs``, ``src/rng.rs``).  It is
the checker for the CUDA library and the timed CPU baseline.  Only ``tests/``,
``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this file;
the product package never does.

Parity of the restatement itself is pinned by the reference's golden vectors
(``src/rng.rs:104-117`` and ``tests/golden.rs:77``), checked in
``tests/test_oracle.py``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
sz = ctypes.c_size_t
c_f = ctypes.c_float


def build() -> str:
    """Compile liboracle.so from the C sources beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is not None:
        return _lib
    src = os.path.join(_HERE, "sparsl_oracle.c")
    if not os.path.exists(_LIB_PATH) or (
        os.path.exists(src) and os.path.getmtime(src) > os.path.getmtime(_LIB_PATH)
    ):
        build()
    L = ctypes.CDLL(_LIB_PATH)
    L.or_rng_size.restype = sz
    L.or_rng_init.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    for name, rt in [("or_rng_next_u32", ctypes.c_uint32), ("or_rng_next_u64", ctypes.c_uint64),
                     ("or_rng_next_f32", ctypes.c_float), ("or_rng_next_f64", ctypes.c_double)]:
        getattr(L, name).restype = rt
        getattr(L, name).argtypes = [ctypes.c_void_p]
    L.or_rng_gen_index.restype = ctypes.c_uint64
    L.or_rng_gen_index.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
    L.or_f16_bits_to_f32.restype = ctypes.c_float
    L.or_f16_bits_to_f32.argtypes = [ctypes.c_uint16]
    L.or_bf16_bits_to_f32.restype = ctypes.c_float
    L.or_bf16_bits_to_f32.argtypes = [ctypes.c_uint16]
    L.or_f32_to_f16_bits.restype = ctypes.c_uint16
    L.or_f32_to_f16_bits.argtypes = [ctypes.c_float]
    L.or_f32_to_bf16_bits.restype = ctypes.c_uint16
    L.or_f32_to_bf16_bits.argtypes = [ctypes.c_float]
    L.or_quantise.argtypes = [ctypes.c_int, f32p, f32p, sz]
    L.or_narrow_bits.argtypes = [ctypes.c_int, f32p, u16p, sz]
    L.or_validate_csr.restype = ctypes.c_int
    L.or_validate_csr.argtypes = [u32p, sz, u32p, sz, sz, sz, ctypes.c_void_p]
    L.or_csc_from_csr.restype = ctypes.c_int
    L.or_csc_from_csr.argtypes = [u32p, sz, u32p, sz, sz, u32p, u32p, u32p]
    L.or_random_csr.restype = sz
    L.or_random_csr.argtypes = [ctypes.c_void_p, sz, sz, sz, u32p, u32p]
    L.or_random_vec.argtypes = [ctypes.c_void_p, f32p, sz, c_f]
    L.or_nnz_balanced_partitions.restype = sz
    L.or_nnz_balanced_partitions.argtypes = [u32p, sz, sz, u64p]
    L.or_num_threads.restype = ctypes.c_int
    L.or_set_num_threads.argtypes = [ctypes.c_int]
    L.or_spmv.argtypes = [ctypes.c_int, u32p, u32p, f32p, sz, f32p, f32p]
    L.or_spmv_spikes.argtypes = [ctypes.c_int, u32p, u32p, f32p, sz, u32p, f32p]
    L.or_spmv_t.argtypes = [ctypes.c_int, u32p, u32p, u32p, f32p, sz, f32p, f32p]
    L.or_spmm.argtypes = [ctypes.c_int, u32p, u32p, f32p, sz, f32p, sz, f32p]
    L.or_lif_integrate.argtypes = [ctypes.c_int, f32p, f32p, f32p, u8p, sz, c_f, c_f, c_f]
    L.or_fused_lif.argtypes = [ctypes.c_int, u32p, u32p, f32p, sz, f32p, f32p, f32p, u8p, c_f, c_f, c_f]
    L.or_fused_spikes_lif.argtypes = [ctypes.c_int, u32p, u32p, f32p, sz, u32p, f32p, f32p, u8p,
                                      c_f, c_f, c_f]
    L.or_recurrent_steps.argtypes = [ctypes.c_int, u32p, u32p, f32p, sz, u32p, f32p, f32p, u8p,
                                     c_f, c_f, c_f, sz, ctypes.c_void_p]
    L.or_packed_len.restype = sz
    L.or_packed_len.argtypes = [sz]
    L.or_pack_spikes_into.argtypes = [u8p, sz, u32p, sz]
    L.or_unpack_spikes.argtypes = [u32p, sz, u8p]
    L.or_scan_sequential.argtypes = [f32p, sz, f32p]
    L.or_scan_chunked.argtypes = [f32p, sz, sz, f32p]
    L.or_scan_magnitude_envelope.restype = c_f
    L.or_scan_magnitude_envelope.argtypes = [f32p, sz]
    L.or_tolerance_for_elementwise.restype = c_f
    L.or_tolerance_for_elementwise.argtypes = [c_f]
    L.or_tolerance_for_spmv.restype = c_f
    L.or_tolerance_for_spmv.argtypes = [ctypes.c_uint64, c_f, c_f]
    L.or_tolerance_for_spmv_narrow.restype = c_f
    L.or_tolerance_for_spmv_narrow.argtypes = [ctypes.c_int, ctypes.c_uint64, c_f, c_f]
    L.or_tolerance_for_scan.restype = c_f
    L.or_tolerance_for_scan.argtypes = [ctypes.c_uint64, c_f]
    L.or_golden_fingerprint.restype = ctypes.c_uint64
    L.or_wl_log.restype = ctypes.c_double
    L.or_wl_log.argtypes = [ctypes.c_double]
    L.or_wl_cos2pi.restype = ctypes.c_double
    L.or_wl_cos2pi.argtypes = [ctypes.c_double]
    L.or_wl_fixed_fanin.argtypes = [ctypes.c_uint64, ctypes.c_uint64, sz, ctypes.c_uint64, ctypes.c_uint32, c_f,
                                    u32p, f32p]
    L.or_wl_lif_state.argtypes = [ctypes.c_uint64, ctypes.c_uint64, sz, c_f, c_f, c_f, c_f, f32p, f32p, u8p]
    L.or_net_ticks.argtypes = [sz, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, sz, u32p,
                               f32p, f32p, u8p, c_f, c_f, c_f, sz, ctypes.c_void_p]
    _lib = L
    return L


# --------------------------------------------------------------------------
# Rng (src/rng.rs)
# --------------------------------------------------------------------------
class Rng:
    """The reference's ChaCha12 stream (``src/rng.rs:21-71``)."""

    def __init__(self, seed: int):
        L = lib()
        self._buf = ctypes.create_string_buffer(L.or_rng_size())
        L.or_rng_init(self._buf, ctypes.c_uint64(seed & 0xFFFFFFFFFFFFFFFF))

    def next_u32(self) -> int:
        return lib().or_rng_next_u32(self._buf)

    def next_u64(self) -> int:
        return lib().or_rng_next_u64(self._buf)

    def next_f32(self) -> float:
        return lib().or_rng_next_f32(self._buf)

    def next_f64(self) -> float:
        return lib().or_rng_next_f64(self._buf)

    def gen_index(self, max_: int) -> int:
        assert max_ > 0
        return lib().or_rng_gen_index(self._buf, max_)


class Csr:
    """Minimal CSR triple (``src/sparse.rs:80-84``)."""

    def __init__(self, row_ptr, col, ncols):
        self.row_ptr = np.ascontiguousarray(row_ptr, dtype=np.uint32)
        self.col = np.ascontiguousarray(col, dtype=np.uint32)
        self.ncols = int(ncols)

    @property
    def nrows(self) -> int:
        return max(len(self.row_ptr) - 1, 0)

    @property
    def nnz(self) -> int:
        return len(self.col)

    @classmethod
    def from_adjacency(cls, rows):
        """``sparse.rs:135-172``: stable sort per row, ncols = max(nrows, max col + 1)."""
        row_ptr = [0]
        col = []
        max_col = None
        for r in rows:
            s = sorted(int(c) for c in r)
            col.extend(s)
            if s:
                max_col = s[-1] if max_col is None else max(max_col, s[-1])
            row_ptr.append(len(col))
        nrows = len(rows)
        ncols = nrows if max_col is None else max(nrows, max_col + 1)
        return cls(np.array(row_ptr, np.uint32), np.array(col, np.uint32), ncols)


def random_csr(nrows: int, ncols: int, max_deg: int, rng: Rng) -> Csr:
    """``tests/common/mod.rs:11-30``."""
    rp = np.zeros(nrows + 1, np.uint32)
    col = np.zeros(max(nrows * max_deg, 1), np.uint32)
    nnz = lib().or_random_csr(rng._buf, nrows, ncols, max_deg, rp, col)
    return Csr(rp, col[:nnz].copy(), ncols)


def random_vec(n: int, scale: float, rng: Rng) -> np.ndarray:
    """``tests/common/mod.rs:33-37``: uniform in ``[-scale, scale)``."""
    out = np.zeros(max(n, 1), np.float32)
    lib().or_random_vec(rng._buf, out, n, scale)
    return out[:n].copy()


# --------------------------------------------------------------------------
# half.rs
# --------------------------------------------------------------------------
def f32_to_f16_bits(a) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.zeros(max(a.size, 1), np.uint16)
    lib().or_narrow_bits(1, a, out, a.size)
    return out[: a.size]


def f32_to_bf16_bits(a) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    out = np.zeros(max(a.size, 1), np.uint16)
    lib().or_narrow_bits(2, a, out, a.size)
    return out[: a.size]


def f16_bits_to_f32(bits) -> np.ndarray:
    L = lib()
    return np.array([L.or_f16_bits_to_f32(int(b)) for b in np.asarray(bits).ravel()], np.float32)


def bf16_bits_to_f32(bits) -> np.ndarray:
    return (np.asarray(bits, np.uint32) << 16).view(np.float32)


def quantise(precision: int, w) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros(max(w.size, 1), np.float32)
    lib().or_quantise(precision, w, out, w.size)
    return out[: w.size]


# --------------------------------------------------------------------------
# CSR validation / CSC
# --------------------------------------------------------------------------
class OrShape(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("a", "b", "c", "nrows", "ncols", "nnz", "max_row_nnz")]


VALIDATE_CODES = {0: "Ok", 1: "EmptyRowPtr", 2: "NonZeroStart", 3: "NotMonotonic", 4: "NnzMismatch",
                  5: "NcolsMismatch", 6: "ColumnOutOfRange", 7: "RowUnsorted", 8: "TooLarge"}


def validate_csr(row_ptr, col, csr_ncols, ncols):
    """``mod.rs:2116-2182``; returns (code name, shape struct)."""
    rp = np.ascontiguousarray(row_ptr, np.uint32)
    c = np.ascontiguousarray(col, np.uint32)
    sh = OrShape()
    code = lib().or_validate_csr(rp if rp.size else np.zeros(1, np.uint32), rp.size,
                                 c if c.size else np.zeros(1, np.uint32), c.size, csr_ncols, ncols,
                                 ctypes.byref(sh))
    return VALIDATE_CODES[code], sh


def csc_from_csr(csr: Csr, ncols: int):
    """``sparse.rs:361-427`` stable reverse index (col_ptr, row, edge_idx)."""
    cp = np.zeros(ncols + 1, np.uint32)
    row = np.zeros(max(csr.nnz, 1), np.uint32)
    eidx = np.zeros(max(csr.nnz, 1), np.uint32)
    rc = lib().or_csc_from_csr(csr.row_ptr, csr.nrows, csr.col if csr.nnz else np.zeros(1, np.uint32),
                               csr.nnz, ncols, cp, row, eidx)
    if rc != 0:
        raise ValueError(f"csc build failed: {rc}")
    return cp, row[: csr.nnz].copy(), eidx[: csr.nnz].copy()


# --------------------------------------------------------------------------
# Kernels
# --------------------------------------------------------------------------
def _nz(a, dtype):
    a = np.ascontiguousarray(a, dtype)
    return a if a.size else np.zeros(1, dtype)


def spmv(csr: Csr, w, x, y, par: bool = False):
    """In-place ``y += A x`` (``mod.rs:2442-2459``)."""
    if csr.nrows == 0:
        return y
    lib().or_spmv(int(par), csr.row_ptr, _nz(csr.col, np.uint32), _nz(w, np.float32), csr.nrows,
                  _nz(x, np.float32), y)
    return y


def spmv_spikes(csr: Csr, w, spikes, y, par: bool = False):
    if csr.nrows == 0:
        return y
    lib().or_spmv_spikes(int(par), csr.row_ptr, _nz(csr.col, np.uint32), _nz(w, np.float32),
                         csr.nrows, _nz(spikes, np.uint32), y)
    return y


def spmv_t(csc, w, x, y, par: bool = False):
    cp, row, eidx = csc
    ncols = len(cp) - 1
    if ncols == 0:
        return y
    lib().or_spmv_t(int(par), _nz(cp, np.uint32), _nz(row, np.uint32), _nz(eidx, np.uint32),
                    _nz(w, np.float32), ncols, _nz(x, np.float32), y)
    return y


def spmm(csr: Csr, w, x, n_vec: int, y, par: bool = False):
    if csr.nrows == 0:
        return y
    lib().or_spmm(int(par), csr.row_ptr, _nz(csr.col, np.uint32), _nz(w, np.float32), csr.nrows,
                  _nz(x, np.float32), n_vec, y)
    return y


def lif_integrate(v, theta, cur, spikes, decay, v_reset, dtheta, par: bool = False):
    if v.size == 0:
        return
    lib().or_lif_integrate(int(par), v, theta, np.ascontiguousarray(cur, np.float32), spikes, v.size,
                           decay, v_reset, dtheta)


def fused_lif(csr: Csr, w, x, v, theta, spikes, decay, v_reset, dtheta, par: bool = False):
    if csr.nrows == 0:
        return
    lib().or_fused_lif(int(par), csr.row_ptr, _nz(csr.col, np.uint32), _nz(w, np.float32), csr.nrows,
                       _nz(x, np.float32), v, theta, spikes, decay, v_reset, dtheta)


def fused_spikes_lif(csr: Csr, w, s, v, theta, spikes, decay, v_reset, dtheta, par: bool = False):
    if csr.nrows == 0:
        return
    lib().or_fused_spikes_lif(int(par), csr.row_ptr, _nz(csr.col, np.uint32), _nz(w, np.float32),
                              csr.nrows, _nz(s, np.uint32), v, theta, spikes, decay, v_reset, dtheta)


def recurrent_steps(csr: Csr, w, x_spikes, v, theta, spikes, decay, v_reset, dtheta, steps: int,
                    par: bool = False):
    """Ticks of ``mod.rs:1889-1932``; returns the per-tick spike-count trace."""
    trace = np.zeros(max(steps, 1), np.uint32)
    lib().or_recurrent_steps(int(par), csr.row_ptr, _nz(csr.col, np.uint32), _nz(w, np.float32),
                             csr.nrows, x_spikes, v, theta, spikes, decay, v_reset, dtheta, steps,
                             trace.ctypes.data)
    return trace[:steps]


def packed_len(n: int) -> int:
    return (n + 31) // 32


def pack_spikes(spikes) -> np.ndarray:
    s = np.ascontiguousarray(spikes, np.uint8)
    out = np.zeros(max(packed_len(s.size), 1), np.uint32)
    lib().or_pack_spikes_into(_nz(s, np.uint8), s.size, out, packed_len(s.size))
    return out[: packed_len(s.size)]


def unpack_spikes(words, n: int) -> np.ndarray:
    out = np.zeros(max(n, 1), np.uint8)
    lib().or_unpack_spikes(_nz(words, np.uint32), n, out)
    return out[:n]


def scan_sequential(xs) -> np.ndarray:
    """``scan.rs:298-313`` over ``[a0, b0, a1, b1, ...]`` pairs (shape (n, 2))."""
    xs = np.ascontiguousarray(xs, np.float32).reshape(-1, 2)
    out = np.zeros_like(xs) if xs.size else np.zeros((0, 2), np.float32)
    if xs.shape[0]:
        lib().or_scan_sequential(xs.ravel(), xs.shape[0], out.reshape(-1))
    return out


def scan_chunked(xs, chunk: int = 256) -> np.ndarray:
    """``scan.rs:218-295``: the CPU-parallel arm, bit-identical to sequential."""
    xs = np.ascontiguousarray(xs, np.float32).reshape(-1, 2)
    out = np.zeros_like(xs)
    if xs.shape[0]:
        lib().or_scan_chunked(xs.ravel(), xs.shape[0], chunk, out.reshape(-1))
    return out


def scan_magnitude_envelope(xs) -> float:
    xs = np.ascontiguousarray(xs, np.float32).reshape(-1)
    return lib().or_scan_magnitude_envelope(_nz(xs, np.float32), xs.size // 2)


def tolerance_for_elementwise(m):
    return lib().or_tolerance_for_elementwise(m)


def tolerance_for_spmv(n, term, result):
    return lib().or_tolerance_for_spmv(n, term, result)


def tolerance_for_spmv_narrow(precision, n, term, result):
    return lib().or_tolerance_for_spmv_narrow(precision, n, term, result)


def tolerance_for_scan(n, env):
    return lib().or_tolerance_for_scan(n, env)


def golden_fingerprint() -> int:
    return lib().or_golden_fingerprint()


def set_threads(n: int) -> None:
    lib().or_set_num_threads(n)


def num_threads() -> int:
    return lib().or_num_threads()


# --------------------------------------------------------------------------
# Benchmark workloads (no reference counterpart): the definition the GPU
# generator follows, drawn on the host.
# --------------------------------------------------------------------------
def wl_log(x: float) -> float:
    return lib().or_wl_log(float(x))


def wl_cos2pi(u: float) -> float:
    return lib().or_wl_cos2pi(float(u))


def wl_fixed_fanin(seed: int, row0: int, nrows: int, ncols: int, fan_in: int, sigma: float, col=None, w=None):
    """Rows [row0, row0 + nrows) of the fixed fan-in network: (col u32, w f32),
    nrows * fan_in each (row-major); drawn on all host threads."""
    n = nrows * fan_in
    col = np.empty(max(n, 1), np.uint32) if col is None else col
    w = np.empty(max(n, 1), np.float32) if w is None else w
    lib().or_wl_fixed_fanin(seed & (2 ** 64 - 1), row0, nrows, ncols, fan_in, sigma, col, w)
    return col[:n], w[:n]


def wl_lif_state(seed: int, cell0: int, n: int, v_lo: float, v_hi: float, theta0: float, density: float):
    """(v, theta, spikes u8) of cells [cell0, cell0 + n)."""
    v = np.empty(max(n, 1), np.float32)
    th = np.empty(max(n, 1), np.float32)
    sp = np.empty(max(n, 1), np.uint8)
    lib().or_wl_lif_state(seed & (2 ** 64 - 1), cell0, n, v_lo, v_hi, theta0, density, v, th, sp)
    return v[:n], th[:n], sp[:n]


def net_ticks(blocks, n_total: int, x_spikes, v, theta, spikes, decay, v_reset, dtheta, steps: int):
    """Recurrent ticks of a network split into row blocks [(row_ptr, col, w), ...]
    (CpuParallel arm); returns the per-tick spike counts.  Updates x_spikes,
    v, theta, spikes in place."""
    nb = len(blocks)
    rps = (ctypes.c_void_p * nb)(*[b[0].ctypes.data for b in blocks])
    cols = (ctypes.c_void_p * nb)(*[b[1].ctypes.data for b in blocks])
    ws = (ctypes.c_void_p * nb)(*[b[2].ctypes.data for b in blocks])
    rows = (ctypes.c_size_t * nb)(*[b[0].size - 1 for b in blocks])
    trace = np.zeros(max(steps, 1), np.uint32)
    lib().or_net_ticks(nb, rps, cols, ws, rows, n_total, x_spikes, v, theta, spikes, decay, v_reset, dtheta,
                       steps, trace.ctypes.data)
    return trace[:steps]

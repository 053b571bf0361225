"""The C-ABI library on a machine without a GPU: it loads, exports every symbol
the header declares, and its host-side logic (the CSR gate, the half.rs
encoders, the tolerances, the availability gate) matches the oracle."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT

import sparsl_b200 as S
from sparsl_b200 import _lib


def _declared_symbols():
    names = set()
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if h.endswith(".h"):
            src = open(os.path.join(ROOT, "include", h)).read()
            src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
            names |= set(re.findall(r"\b(sparsl_[a-z0-9_]+)\s*\(", src))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    declared = _declared_symbols()
    assert len(declared) > 60
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, missing
    # The ctypes table covers the header exactly.
    assert set(declared) == set(_lib.SIGNATURES)


def test_library_is_the_in_tree_build():
    L = _lib.load()
    assert os.path.dirname(L._name) == os.path.join(ROOT, "sparsl_b200")
    assert b"sm_100a" in L.sparsl_version()


def test_f16_encoder_matches_oracle_exhaustively_on_half_values(O):
    allbits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    wide = O.f16_bits_to_f32(allbits)
    assert np.array_equal(S.f32_to_f16_bits(wide), O.f32_to_f16_bits(wide))


@pytest.mark.parametrize("seed", [1, 2, 3])
def test_narrow_encoders_match_oracle_on_random_bit_patterns(O, seed):
    r = np.random.default_rng(seed)
    pats = r.integers(0, 2 ** 32, size=400_000, dtype=np.uint64).astype(np.uint32)
    # Dense coverage of the subnormal and overflow edges too.
    edges = np.concatenate([np.arange(0x33000000, 0x33800000, 997, dtype=np.uint32),
                            np.arange(0x38700000, 0x38900000, 131, dtype=np.uint32),
                            np.arange(0x477fe000, 0x47800100, 7, dtype=np.uint32)])
    vals = np.concatenate([pats, edges, edges | 0x80000000]).view(np.float32)
    assert np.array_equal(S.f32_to_f16_bits(vals), O.f32_to_f16_bits(vals))
    assert np.array_equal(S.f32_to_bf16_bits(vals), O.f32_to_bf16_bits(vals))
    for p in (S.WeightPrecision.F16, S.WeightPrecision.Bf16):
        a = S.quantise(p, vals)
        b = O.quantise(int(p), vals)
        assert np.array_equal(a.view(np.uint32)[~np.isnan(a)], b.view(np.uint32)[~np.isnan(b)])


def test_validate_csr_matches_oracle_variants_and_payloads(O):
    cases = [
        ([], [], 0, 0), ([1, 1], [0], 1, 1), ([0, 2, 1], [0, 0], 1, 1), ([0, 2], [0], 1, 1),
        ([0, 1], [0], 2, 1), ([0, 2], [0, 5], 2, 2), ([0, 2], [1, 0], 2, 2), ([0, 2, 3], [0, 1, 1], 2, 2),
        ([0, 0, 3, 5], [0, 2, 1, 3, 3], 4, 4), ([0, 3, 5], [4, 2, 9, 1, 1], 4, 4),
    ]
    for rp, col, csr_ncols, ncols in cases:
        code, osh = O.validate_csr(rp, col, csr_ncols, ncols)
        sh = _lib.Shape()
        rpa = np.array(rp, np.uint32)
        ca = np.array(col, np.uint32)
        _lib.load().sparsl_validate_csr(rpa.ctypes.data if rpa.size else None, rpa.size,
                                        ca.ctypes.data if ca.size else None, ca.size, csr_ncols, ncols,
                                        ctypes.byref(sh))
        names = {0: "Ok", 1: "EmptyRowPtr", 2: "NonZeroStart", 3: "NotMonotonic", 4: "NnzMismatch",
                 5: "NcolsMismatch", 6: "ColumnOutOfRange", 7: "RowUnsorted", 8: "TooLarge"}
        assert names[sh.code] == code, (rp, col)
        if code != "Ok":
            assert (sh.a, sh.b) == (osh.a, osh.b), (rp, col, code)
        else:
            assert (sh.nrows, sh.ncols, sh.nnz, sh.max_row_nnz) == (osh.nrows, osh.ncols, osh.nnz, osh.max_row_nnz)


def test_validate_large_random_csr_is_ok(O):
    rng = O.Rng(7)
    csr = O.random_csr(5000, 3000, 40, rng)
    sh = _lib.Shape()
    rc = _lib.load().sparsl_validate_csr(csr.row_ptr.ctypes.data, csr.row_ptr.size, csr.col.ctypes.data,
                                         csr.col.size, 3000, 3000, ctypes.byref(sh))
    assert rc == 0 and sh.nnz == csr.nnz


def test_tolerances_match_oracle(O):
    for n, t, r in [(0, 0.0, 0.0), (1, 1.0, 1.0), (1000, 0.25, 0.25), (64, 3.5, 100.0), (2 ** 40, 1.0, 1.0)]:
        assert np.float32(S.tolerance_for_spmv(n, t, r)) == np.float32(O.tolerance_for_spmv(n, t, r))
        for p in (0, 1, 2):
            assert np.float32(S.tolerance_for_spmv_narrow(S.WeightPrecision(p), n, t, r)) == \
                np.float32(O.tolerance_for_spmv_narrow(p, n, t, r))
    for m in (0.0, -1.0, 1.0, 1e-30, 3e38):
        assert np.float32(S.tolerance_for_elementwise(m)) == np.float32(O.tolerance_for_elementwise(m))
    for n, e in [(1, 1.0), (100, 24.0), (2000, 0.5), (5, float("inf"))]:
        assert np.float32(S.tolerance_for_scan(n, e)) == np.float32(O.tolerance_for_scan(n, e))
    xs = np.array([[2.0, 3.0], [-4.0, 12.0]], np.float32)
    assert S.scan_magnitude_envelope(xs) == 24.0 == O.scan_magnitude_envelope(xs)
    # The reference's bounds pin (mod.rs:2725-2744).
    t = S.tolerance_for_spmv(1000, 0.25, 0.25)
    assert 3.3e-6 < t < 1e-3


def test_spike_helpers_match_oracle(O):
    r = np.random.default_rng(3)
    for n in (0, 1, 31, 32, 33, 63, 64, 65, 1000, 262_145):
        s = r.random(n) < 0.37
        assert np.array_equal(S.pack_spikes(s), O.pack_spikes(s.astype(np.uint8)))
        assert np.array_equal(S.unpack_spikes(S.pack_spikes(s), n), s)
        # any nonzero byte is a spike; bits past n in the last word are ignored
        b = s.astype(np.uint8) * r.integers(1, 256, n, dtype=np.uint8)
        assert np.array_equal(S.pack_spikes(b), O.pack_spikes(s.astype(np.uint8)))
        w = S.pack_spikes(s)
        if n % 32:
            w[-1] |= np.uint32(0xFFFFFFFF) << np.uint32(n % 32)
        assert np.array_equal(S.unpack_spikes(w, n), s)


@pytest.mark.skipif(_lib.load().sparsl_device_count() > 0, reason="a GPU is visible")
def test_cuda_fails_closed_without_a_device():
    """Backend::Cuda is unavailable with a reason and unconstructible (honesty.rs:38-60)."""
    reason = S.Backend.Cuda.unavailable_reason()
    assert reason and "device" in reason
    with pytest.raises(S.BackendUnavailable) as ei:
        S.Device.try_new(S.Backend.Cuda)
    assert ei.value.requested is S.Backend.Cuda
    assert S.Backend.Cuda not in S.available_backends()


def test_no_cpu_device_under_any_label():
    for b in (S.Backend.CpuSequential, S.Backend.CpuParallel, S.Backend.Metal):
        with pytest.raises(S.BackendUnavailable):
            S.Device.try_new(b)
    assert S.Backend.Cuda.label() == "CUDA GPU" and S.Backend.Cuda.is_gpu()


def test_lif_params_reject_non_finite():
    for args, field in [((float("nan"), 0, 0), "decay"), ((0.9, float("inf"), 0), "v_reset"),
                        ((0.9, 0, float("-inf")), "delta_theta")]:
        with pytest.raises(S.LifParamsError) as ei:
            S.LifParams.new(*args)
        assert ei.value.field == field
    assert S.LifParams.new(0.0, 0.0, 0.0).decay() == 0.0


def test_csr_from_adjacency_and_parts():
    csr = S.Csr.from_adjacency([[2, 1], [0], [0, 1]])
    assert list(csr.row_ptr()) == [0, 2, 3, 5] and list(csr.col()) == [1, 2, 0, 0, 1] and csr.ncols() == 3
    with pytest.raises(S.CsrError):
        S.Csr.from_parts([0, 2], [1, 0], 2)
    assert S.Csr.from_parts([0, 2], [0, 1], 2).nnz() == 2


def test_host_buffer_is_pinned_or_refused():
    """HostBuffer: page-locked host memory as a numpy array where a CUDA device
    exists, the Backend error where none does.  A view of the array keeps the
    memory alive after the buffer object is gone."""
    import gc

    import torch

    if not torch.cuda.is_available():
        with pytest.raises(S.OpError) as e:
            S.HostBuffer(100)
        assert e.value.kind == "Backend"
        return
    h = S.HostBuffer(100, np.float32)
    assert h.array.dtype == np.float32 and h.array.size == 100 and h.array.flags.writeable
    assert h.data_ptr() == h.array.ctypes.data
    view = h.array[10:20]
    del h
    gc.collect()
    view[:] = 3.0
    assert float(view.sum()) == 30.0

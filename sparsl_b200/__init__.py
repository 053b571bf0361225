"""sparsl_b200 -- the B200 (sm_100a) CUDA substrate for sparsl.

The hot path is native: ``libsparsl_cuda.so`` (C ABI in
``include/sparsl_cuda.h``) holds hand-written sm_100a kernels and the
runtime around them.  This package is the host-side mirror of the reference
crate's ``Device`` / ``SparseOp`` API (bharathvbcr/sparsl,
``src/backend/mod.rs``) over that ABI, plus the multi-GPU network tick.
"""
from .backend import (  # noqa: F401
    ALL_BACKENDS,
    Backend,
    BackendUnavailable,
    Csr,
    CsrError,
    DeviceBuffer,
    Device,
    HostBuffer,
    LifParams,
    LifParamsError,
    OpError,
    SparseOp,
    SparsePlanError,
    SparseShape,
    WeightPrecision,
    available_backends,
    f32_to_bf16_bits,
    f32_to_f16_bits,
    pack_spikes,
    packed_len,
    quantise,
    scan_magnitude_envelope,
    spikes_to_f32,
    tolerance_for_elementwise,
    tolerance_for_scan,
    tolerance_for_spmv,
    tolerance_for_spmv_bf16,
    tolerance_for_spmv_f16,
    tolerance_for_spmv_narrow,
    unpack_spikes,
)

DEFAULT_CHUNK_SIZE = 256  # scan.rs:64; the CUDA scan's output does not depend on it

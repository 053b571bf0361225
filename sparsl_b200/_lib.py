"""ctypes binding of libsparsl_cuda.so (the C ABI in include/sparsl_cuda.h).

The library is loaded from this package directory only.  If it is missing
the import of any GPU entry point raises: there is no CPU fallback anywhere
in this package.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsparsl_cuda.so")

_lock = threading.Lock()
_lib = None

vp = ctypes.c_void_p
u64 = ctypes.c_uint64
i32 = ctypes.c_int
f32 = ctypes.c_float

SPARSL_OK = 0
SPARSL_ERR_BACKEND = 1
SPARSL_ERR_EXECUTION = 2
SPARSL_ERR_ALLOCATION = 3
SPARSL_ERR_INVALID = 4
SPARSL_ERR_LENGTH = 5
SPARSL_ERR_NO_TRANSPOSE = 6


class Shape(ctypes.Structure):
    """``sparsl_shape``."""

    _fields_ = [("code", ctypes.c_int32), ("a", u64), ("b", u64), ("c", u64), ("nrows", u64), ("ncols", u64),
                ("nnz", u64), ("max_row_nnz", u64)]


# name -> (restype, argtypes); every symbol include/*.h declares.
SIGNATURES = {
    "sparsl_last_error": (ctypes.c_char_p, []),
    "sparsl_last_reason": (ctypes.c_char_p, []),
    "sparsl_version": (ctypes.c_char_p, []),
    "sparsl_set_timeout_ms": (None, [u64]),
    "sparsl_cuda_probe": (i32, [ctypes.POINTER(ctypes.c_char_p)]),
    "sparsl_device_count": (i32, []),
    "sparsl_device_open": (i32, [i32, ctypes.POINTER(vp)]),
    "sparsl_device_close": (None, [vp]),
    "sparsl_device_name": (i32, [vp, ctypes.c_char_p, ctypes.c_size_t]),
    "sparsl_device_reset": (i32, []),
    "sparsl_quarantined": (i32, []),
    "sparsl_dev_assoc_scan": (i32, [vp, vp, u64, vp]),
    "sparsl_dev_lif_integrate": (i32, [vp, vp, vp, vp, vp, u64, f32, f32, f32]),
    "sparsl_dev_lif_integrate_device": (i32, [vp, vp, vp, vp, vp, u64, f32, f32, f32, vp]),
    "sparsl_validate_csr": (i32, [vp, u64, vp, u64, u64, u64, ctypes.POINTER(Shape)]),
    "sparsl_f32_to_f16_bits": (None, [vp, vp, u64]),
    "sparsl_f32_to_bf16_bits": (None, [vp, vp, u64]),
    "sparsl_quantise": (None, [i32, vp, vp, u64]),
    "sparsl_op_prepare": (i32, [vp, vp, u64, vp, u64, u64, u64, vp, u64, i32, i32, ctypes.POINTER(Shape),
                                ctypes.POINTER(vp)]),
    "sparsl_op_prepare_device": (i32, [vp, vp, u64, vp, u64, u64, u64, vp, u64, i32, i32,
                                       ctypes.POINTER(Shape), ctypes.POINTER(vp)]),
    "sparsl_op_prepare_device_borrowed": (i32, [vp, vp, u64, vp, u64, u64, u64, vp, u64, i32,
                                                ctypes.POINTER(Shape), ctypes.POINTER(vp)]),
    "sparsl_csc_from_csr_device": (i32, [vp, vp, u64, vp, u64, u64, vp, vp, vp, ctypes.POINTER(Shape)]),
    "sparsl_op_bind_x": (i32, [vp, vp]),
    "sparsl_op_bind_y": (i32, [vp, vp]),
    "sparsl_op_unbind_x": (i32, [vp]),
    "sparsl_op_unbind_y": (i32, [vp]),
    "sparsl_op_x_address": (i32, [vp, ctypes.POINTER(u64)]),
    "sparsl_op_y_address": (i32, [vp, ctypes.POINTER(u64)]),
    "sparsl_op_alloc_f32": (i32, [vp, vp, u64, ctypes.POINTER(vp)]),
    "sparsl_op_wait_event": (i32, [vp, vp, u64]),
    "sparsl_op_signal_event": (i32, [vp, vp]),
    "sparsl_dev_assoc_scan_from_device": (i32, [vp, vp, u64, vp, vp, vp]),
    "sparsl_dev_scan_fold_device": (i32, [vp, vp, u64, vp, vp, vp]),
    "sparsl_dev_scan_rejoin_device": (i32, [vp, vp, vp, u64, vp, vp, ctypes.POINTER(u64), vp]),
    "sparsl_dev_scan_table_device": (i32, [vp, vp, u64, ctypes.POINTER(ctypes.c_uint32), vp]),
    "sparsl_dev_scan_settle_device": (i32, [vp, vp, u64, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(u64), vp]),
    "sparsl_op_layouts": (i32, [vp]),
    "sparsl_op_force_plain_row_fold": (i32, [vp]),
    "sparsl_dev_test_expired_wait": (i32, [vp]),
    "sparsl_op_test_mark_canary": (i32, [vp]),
    "sparsl_dev_scan_publish_device": (i32, [vp, vp, u64, i32, ctypes.c_uint32, vp, vp]),
    "sparsl_dev_scan_entry_device": (i32, [vp, vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, vp, vp]),
    "sparsl_dev_assoc_scan_after_device": (i32, [vp, vp, u64, vp, vp, vp]),
    "sparsl_op_destroy": (None, [vp]),
    "sparsl_op_shape": (i32, [vp, ctypes.POINTER(Shape)]),
    "sparsl_op_weight_precision": (i32, [vp]),
    "sparsl_op_has_transpose": (i32, [vp]),
    "sparsl_op_set_weights": (i32, [vp, vp, u64]),
    "sparsl_op_spmv": (i32, [vp, vp, u64, vp, u64]),
    "sparsl_op_spmv_spikes": (i32, [vp, vp, u64, vp, u64]),
    "sparsl_op_spmv_t": (i32, [vp, vp, u64, vp, u64]),
    "sparsl_op_spmm": (i32, [vp, vp, u64, u64, vp, u64]),
    "sparsl_op_fused_lif": (i32, [vp, vp, u64, vp, vp, vp, u64, f32, f32, f32]),
    "sparsl_op_fused_spikes_lif": (i32, [vp, vp, u64, vp, vp, vp, u64, f32, f32, f32]),
    "sparsl_op_write_x": (i32, [vp, vp, u64]),
    "sparsl_op_write_x_spikes": (i32, [vp, vp, u64]),
    "sparsl_op_write_y": (i32, [vp, vp, u64]),
    "sparsl_op_write_lif_state": (i32, [vp, vp, vp, u64]),
    "sparsl_op_spmv_resident": (i32, [vp]),
    "sparsl_op_fused_lif_resident": (i32, [vp, f32, f32, f32]),
    "sparsl_op_fused_spikes_lif_resident": (i32, [vp, f32, f32, f32]),
    "sparsl_op_pack_resident_spikes": (i32, [vp]),
    "sparsl_op_recurrent_steps": (i32, [vp, f32, f32, f32, u64]),
    "sparsl_op_sync_y": (i32, [vp, vp, u64]),
    "sparsl_op_sync_lif_state": (i32, [vp, vp, vp, vp, u64]),
    "sparsl_op_sync_x_spikes": (i32, [vp, vp, u64]),
    "sparsl_op_spike_trace": (i32, [vp, vp, u64, ctypes.POINTER(u64)]),
    "sparsl_op_spike_indices": (i32, [vp, vp, u64, ctypes.POINTER(u64)]),
    "sparsl_op_spmv_device": (i32, [vp, vp, vp, vp]),
    "sparsl_op_spmv_spikes_device": (i32, [vp, vp, vp, vp]),
    "sparsl_op_spmv_t_device": (i32, [vp, vp, vp, vp]),
    "sparsl_op_spmm_device": (i32, [vp, vp, u64, vp, vp]),
    "sparsl_dev_assoc_scan_device": (i32, [vp, vp, u64, vp, vp]),
    "sparsl_op_recurrent_steps_async": (i32, [vp, f32, f32, f32, u64]),
    "sparsl_op_stream": (vp, [vp]),
    "sparsl_dev_stream": (vp, [vp]),
    "sparsl_op_wait": (i32, [vp]),
    "sparsl_dev_wait": (i32, [vp]),
    "sparsl_dev_scan_stats": (i32, [vp, ctypes.POINTER(u64), ctypes.POINTER(u64)]),
    "sparsl_dev_assoc_scan_noalloc": (i32, [i32, vp, u64, vp, vp, u64]),
    "sparsl_host_alloc": (vp, [u64]),
    "sparsl_host_free": (None, [vp]),
    "sparsl_device_alloc": (vp, [vp, u64]),
    "sparsl_device_free": (None, [vp]),
    "sparsl_memcpy": (i32, [vp, vp, u64]),
    "sparsl_nccl_unique_id": (i32, [vp]),
    "sparsl_net_create": (i32, [vp, vp, ctypes.c_uint32, u64, u64, i32, i32, vp, ctypes.POINTER(vp)]),
    "sparsl_net_destroy": (None, [vp]),
    "sparsl_net_write_state": (i32, [vp, vp, u64, vp, vp, u64]),
    "sparsl_net_steps": (i32, [vp, f32, f32, f32, u64]),
    "sparsl_net_steps_async": (i32, [vp, f32, f32, f32, u64]),
    "sparsl_net_wait": (i32, [vp]),
    "sparsl_net_stream": (vp, [vp]),
    "sparsl_net_read_state": (i32, [vp, vp, u64, vp, vp, u64]),
    "sparsl_net_steps_host": (i32, [vp, vp, u64, vp, vp, u64, f32, f32, f32, u64]),
    "sparsl_net_trace": (i32, [vp, vp, u64, ctypes.POINTER(u64)]),
    "sparsl_net_set_timing": (i32, [vp, u64]),
    "sparsl_net_kernel_ms": (i32, [vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(u64)]),
    "sparsl_net_tick_ms": (i32, [vp, vp, u64, ctypes.POINTER(u64)]),
    "sparsl_net_set_exchange": (i32, [vp, i32]),
    # include/sparsl_workload.h
    "sparsl_workload_fixed_fanin": (i32, [u64, u64, u64, u64, ctypes.c_uint32, f32, vp, vp, vp]),
    "sparsl_workload_uniform_row_ptr": (i32, [u64, ctypes.c_uint32, vp, vp]),
    "sparsl_workload_lif_state": (i32, [u64, u64, u64, f32, f32, f32, f32, vp, vp, vp, vp]),
}


def load():
    """Load the library (once).  Raises if it is absent -- never falls back."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libsparsl_cuda.so is not built ({LIB_PATH}); run `python -m sparsl_b200.build`. "
                "There is no CPU fallback.")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
        return L


def last_error() -> str:
    v = load().sparsl_last_error()
    return v.decode() if v else ""


def last_reason() -> str:
    v = load().sparsl_last_reason()
    return v.decode() if v else ""

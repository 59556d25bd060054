"""ctypes binding of libbarracuda_fhe.so (the C ABI in include/barracuda_fhe.h).

The library is built in-tree (``python -m barracuda_b200.build``).  There is no
fallback: if the shared library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "lib", "libbarracuda_fhe.so")

BC_OK = 0
BC_ERR_DEVICE = 1
BC_ERR_INVALID_INPUT = 2
BC_ERR_OUT_OF_MEMORY = 3
BC_ERR_DEVICE_LOST = 4
BC_ERR_GPU = 5
BC_ERR_UNSUPPORTED = 6
BC_ERR_DEVICE_NOT_AVAILABLE = 7
BC_ERR_EXECUTION = 8
BC_ERR_INTERNAL = 9

BC_NTT_CYCLIC = 0
BC_NTT_NEGACYCLIC = 1

# Rust Display prefixes of the BarracudaError variants (crates/barracuda/src/error.rs)
_DISPLAY = {
    BC_ERR_DEVICE: "Device error: ",
    BC_ERR_INVALID_INPUT: "Invalid input: ",
    BC_ERR_OUT_OF_MEMORY: "Out of memory: ",
    BC_ERR_DEVICE_LOST: "GPU device lost: ",
    BC_ERR_GPU: "GPU error: ",
    BC_ERR_UNSUPPORTED: "Operation not supported on device: ",
    BC_ERR_DEVICE_NOT_AVAILABLE: "Device not available: ",
    BC_ERR_EXECUTION: "Execution error: ",
    BC_ERR_INTERNAL: "Internal error: ",
}

KIND_NAMES = {
    BC_ERR_DEVICE: "Device", BC_ERR_INVALID_INPUT: "InvalidInput",
    BC_ERR_OUT_OF_MEMORY: "OutOfMemory", BC_ERR_DEVICE_LOST: "DeviceLost", BC_ERR_GPU: "Gpu",
    BC_ERR_UNSUPPORTED: "UnsupportedOperation", BC_ERR_DEVICE_NOT_AVAILABLE: "DeviceNotAvailable",
    BC_ERR_EXECUTION: "ExecutionError", BC_ERR_INTERNAL: "Internal",
}


class BarracudaError(RuntimeError):
    """Mirror of BarracudaError: ``kind`` is the variant name, ``message`` its payload."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.kind = KIND_NAMES.get(status, f"status{status}")
        self.message = message
        super().__init__(_DISPLAY.get(status, "") + message)


class NativeLibraryMissing(RuntimeError):
    pass


class bc_layout(ctypes.Structure):
    _fields_ = [("limb_stride", ctypes.c_int64), ("poly_stride", ctypes.c_int64)]


class bc_plan_info(ctypes.Structure):
    _fields_ = [("degree", ctypes.c_uint32), ("n_limbs", ctypes.c_uint32), ("mode", ctypes.c_int32),
                ("word_bits", ctypes.c_int32), ("kernel_kind", ctypes.c_int32),
                ("cluster_size", ctypes.c_int32), ("table_bytes", ctypes.c_uint64)]


_vp = ctypes.c_void_p
_u32, _u64, _i32, _sz = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_size_t
_u64p = ctypes.POINTER(ctypes.c_uint64)
_lay = ctypes.POINTER(bc_layout)

# name -> (restype, argtypes); the list mirrors include/barracuda_fhe.h
SIGNATURES = {
    "bc_last_error": (ctypes.c_char_p, []),
    "bc_abi_version": (_i32, []),
    "bc_device_count": (_i32, [ctypes.POINTER(ctypes.c_int)]),
    "bc_ctx_create": (_i32, [_i32, ctypes.POINTER(_vp)]),
    "bc_ctx_destroy": (_i32, [_vp]),
    "bc_ctx_device": (_i32, [_vp, ctypes.POINTER(ctypes.c_int)]),
    "bc_ctx_stream": (_i32, [_vp, ctypes.POINTER(_vp)]),
    "bc_ctx_sync": (_i32, [_vp]),
    "bc_buf_alloc": (_i32, [_vp, _sz, ctypes.POINTER(_vp)]),
    "bc_buf_free": (_i32, [_vp, _vp]),
    "bc_buf_h2d": (_i32, [_vp, _vp, _vp, _sz]),
    "bc_buf_d2h": (_i32, [_vp, _vp, _vp, _sz]),
    "bc_buf_h2d_async": (_i32, [_vp, _vp, _vp, _sz, _vp]),
    "bc_buf_d2h_async": (_i32, [_vp, _vp, _vp, _sz, _vp]),
    "bc_host_alloc": (_i32, [_sz, ctypes.POINTER(_vp)]),
    "bc_host_free": (_i32, [_vp]),
    "bc_compute_primitive_root": (_u64, [_u32, _u64]),
    "bc_compute_inverse_root": (_u64, [_u32, _u64, _u64]),
    "bc_fhe_ntt_check": (_i32, [_sz, _u32, _u64, _u64]),
    "bc_fhe_ntt": (_i32, [_vp, _vp, _sz, _u32, _u64, _u64, _vp]),
    "bc_fhe_intt_check": (_i32, [_sz, _u32, _u64, _u64]),
    "bc_fhe_intt": (_i32, [_vp, _vp, _sz, _u32, _u64, _u64, _vp]),
    "bc_fhe_pointwise_mul_check": (_i32, [_sz, _sz, _u32, _u64]),
    "bc_fhe_pointwise_mul": (_i32, [_vp, _vp, _sz, _vp, _sz, _u32, _u64, _vp]),
    "bc_fhe_fast_poly_mul_check": (_i32, [_sz, _sz, _u32, _u64, _u64]),
    "bc_fhe_poly_add_check": (_i32, [_sz, _sz, _u32, _u64]),
    "bc_fhe_poly_add": (_i32, [_vp, _vp, _sz, _vp, _sz, _u32, _u64, _vp]),
    "bc_fhe_poly_sub_check": (_i32, [_sz, _sz, _u32, _u64]),
    "bc_fhe_poly_sub": (_i32, [_vp, _vp, _sz, _vp, _sz, _u32, _u64, _vp]),
    "bc_fhe_poly_mul_check": (_i32, [_sz, _sz, _u32, _u64]),
    "bc_fhe_poly_mul": (_i32, [_vp, _vp, _sz, _vp, _sz, _u32, _u64, _vp]),
    "bc_fhe_fast_poly_mul": (_i32, [_vp, _vp, _sz, _vp, _sz, _u32, _u64, _u64, _vp]),
    "bc_fhe_rotate_check": (_i32, [_sz, _u32, _i32, _u64]),
    "bc_fhe_rotate": (_i32, [_vp, _vp, _sz, _u32, _i32, _u64, _vp]),
    "bc_rotation_galois": (_u32, [_u32, _i32]),
    "bc_fhe_modulus_switch_check": (_i32, [_sz, _u32, _u64, _u64]),
    "bc_fhe_modulus_switch": (_i32, [_vp, _vp, _sz, _u32, _u64, _u64, _vp]),
    "bc_fhe_key_switch_check": (_i32, [_sz, _u32, _u64, _u32, _u32]),
    "bc_fhe_key_switch": (_i32, [_vp, _vp, _sz, _u32, _u64, _u32, _u32, _vp]),
    "bc_plan_create": (_i32, [_vp, _u32, _u32, _u64p, _u64p, _u64p, _i32, ctypes.POINTER(_vp)]),
    "bc_plan_destroy": (_i32, [_vp]),
    "bc_plan_info_get": (_i32, [_vp, ctypes.POINTER(bc_plan_info)]),
    "bc_ntt_forward": (_i32, [_vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_inverse": (_i32, [_vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_poly_add": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_poly_sub": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_poly_mul": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_pointwise_mul": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_forward_mul": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_inverse_mul": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_forward_add": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_forward_sub": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_inverse_add": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_ntt_inverse_sub": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_polymul": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_polymul_static_scratch": (_i32, [_vp, _vp, _vp, _vp, _u32, _lay, _vp]),
    "bc_automorphism": (_i32, [_vp, _vp, _vp, _u32, _lay, _u32, _vp]),
    "bc_modulus_switch": (_i32, [_vp, _vp, _vp, _sz, _u64, _u64, _vp]),
    "bc_decompose": (_i32, [_vp, _vp, _vp, _sz, _u32, _u32, _vp]),
    "bc_fill_uniform": (_i32, [_vp, _vp, _u32, _lay, _u64, _u64, _u64, _vp]),
    "bc_digest": (_i32, [_vp, _vp, _sz, _u64, _vp, _vp]),
    "bc_calibrate_butterflies": (_i32, [_vp, _i32, ctypes.POINTER(ctypes.c_double)]),
    "bc_partition": (_i32, [_u64, _u32, _u32, _u64p, _u64p]),
    "bc_ntt_prime": (_u64, [_u32, _u32, _u32]),
    "bc_negacyclic_root": (_u64, [_u64, _u32]),
    "bc_debug_twiddle": (_i32, [_u32, _u64, _u64, _u64, _i32, _i32, _u32, _u64p, _u64p]),
}

_lib = None


def lib():
    """The loaded library; raises NativeLibraryMissing if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise NativeLibraryMissing(
                f"{LIB_PATH} is missing: build it with `python -m barracuda_b200.build` "
                "(there is no CPU fallback for this path)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    m = lib().bc_last_error()
    return m.decode("utf-8", "replace") if m else ""


def check(status: int) -> None:
    """Raise BarracudaError for a non-zero status."""
    if status != BC_OK:
        raise BarracudaError(status, last_error())

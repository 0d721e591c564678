"""ctypes binding of the C ABI declared in include/mxfp4_b200.h.

The shared library is built in-tree (``python -m mxfp4_b200.build``) next to this file.
There is no fallback: if it is missing, importing the operator module fails loudly.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
# MXFP4_B200_LIB may point at another build of the same library (e.g. a profiling build)
LIB_PATH = os.environ.get("MXFP4_B200_LIB") or os.path.join(_HERE, "libmxfp4_b200.so")

LAYOUT_REF, LAYOUT_NK, LAYOUT_G, LAYOUT_PREPACKED = 0, 1, 2, 3
DTYPE_F32, DTYPE_BF16 = 0, 1
PATH_AUTO, PATH_TC, PATH_TC_SMEM, PATH_GEMV = 0, 1, 2, 3
RULE_REF, RULE_OCP = 0, 1
MX_Q8, MX_SPLIT2 = 0, 1
MX_MODES = {"q8": MX_Q8, "split2": MX_SPLIT2}

PATH_NAMES = {"auto": PATH_AUTO, "tc": PATH_TC, "tc_smem": PATH_TC_SMEM, "gemv": PATH_GEMV}

# every symbol include/mxfp4_b200.h declares
EXPORTED = (
    "mxfp4_abi_version",
    "mxfp4_device_info_get",
    "mxfp4_device_error",
    "mxfp4_error_string",
    "mxfp4_test_hooks",
    "mxfp4_quantize",
    "mxfp4_dequantize",
    "mxfp4_prepacked_bytes",
    "mxfp4_prepack",
    "mxfp4_dequantize_prepacked",
    "mxfp4_select_path",
    "mxfp4_shape_supported",
    "mxfp4_gemm_workspace_bytes",
    "mxfp4_gemm",
    "mxfp4_gemm_noalloc",
    "mxfp4_gemm_allgather",
    "mxfp4_ipc_handle_bytes",
    "mxfp4_ipc_export",
    "mxfp4_ipc_open",
    "mxfp4_ipc_close",
    "mxfp4_copy_columns",
    "mxfp4_mx_weight_bytes",
    "mxfp4_prepack_mx",
    "mxfp4_mx_workspace_bytes",
    "mxfp4_quantize_act_mx8",
    "mxfp4_gemm_mx",
)


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("name", ctypes.c_char * 256),
        ("major", ctypes.c_int),
        ("minor", ctypes.c_int),
        ("multi_processor_count", ctypes.c_int),
        ("warp_size", ctypes.c_int),
        ("total_global_mem", ctypes.c_longlong),
        ("shared_mem_per_block", ctypes.c_longlong),
        ("shared_mem_per_block_optin", ctypes.c_longlong),
        ("l2_cache_size", ctypes.c_longlong),
        ("clock_rate_khz", ctypes.c_int),
        ("memory_clock_rate_khz", ctypes.c_int),
        ("memory_bus_width", ctypes.c_int),
    ]


_lib = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I = ctypes.c_int
_SZ = ctypes.c_size_t


def _declare(lib):
    sig = {
        "mxfp4_abi_version": (_I, []),
        "mxfp4_device_info_get": (_I, [_I, ctypes.POINTER(DeviceInfo)]),
        "mxfp4_device_error": (_I, [_I, ctypes.POINTER(ctypes.c_uint)]),
        "mxfp4_error_string": (ctypes.c_char_p, [_I]),
        "mxfp4_test_hooks": (_I, [_I, ctypes.c_ulonglong]),
        "mxfp4_quantize": (_I, [_P, _I, _I, _I, _I, _P, _P, _P]),
        "mxfp4_dequantize": (_I, [_P, _P, _I, _I, _I, _P, _I, _P]),
        "mxfp4_prepacked_bytes": (_SZ, [_I, _I]),
        "mxfp4_prepack": (_I, [_P, _P, _I, _I, _I, _P, _P]),
        "mxfp4_dequantize_prepacked": (_I, [_P, _I, _I, _P, _P]),
        "mxfp4_select_path": (_I, [_I, _I, _I]),
        "mxfp4_shape_supported": (_I, [_I, _I, _I, _I]),
        "mxfp4_gemm_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
        "mxfp4_gemm": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _SZ, _P]),
        "mxfp4_gemm_noalloc": (_I, [_P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P]),
        "mxfp4_gemm_allgather": (_I, [_P, _P, ctypes.POINTER(_P), _I, _I, _I, _I, _I, _I, _I, _I, _P, _SZ, _P]),
        "mxfp4_ipc_handle_bytes": (_SZ, []),
        "mxfp4_ipc_export": (_I, [_P, _P, ctypes.POINTER(_SZ)]),
        "mxfp4_ipc_open": (_I, [_P, _SZ, ctypes.POINTER(_P)]),
        "mxfp4_ipc_close": (_I, [_P, _SZ]),
        "mxfp4_copy_columns": (_I, [_P, _SZ, _P, _SZ, _SZ, _I, _P]),
        "mxfp4_mx_weight_bytes": (_SZ, [_I, _I]),
        "mxfp4_prepack_mx": (_I, [_P, _P, _I, _I, _I, _P, _P]),
        "mxfp4_mx_workspace_bytes": (_SZ, [_I, _I, _I, _I]),
        "mxfp4_quantize_act_mx8": (_I, [_P, _I, _I, _I, _P, _P]),
        "mxfp4_gemm_mx": (_I, [_P, _P, _P, _I, _I, _I, _I, _I, _P, _SZ, _P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def lib():
    """The loaded library (loads it on first use; raises if it was not built)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"{LIB_PATH} is missing: build it with `python -m mxfp4_b200.build` "
                        "(there is no CPU fallback)"
                    )
                handle = ctypes.CDLL(LIB_PATH)
                _declare(handle)
                _lib = handle
    return _lib


def error_string(code: int) -> str:
    return lib().mxfp4_error_string(int(code)).decode()


def check(code: int, what: str) -> None:
    """Raise RuntimeError for a non-zero status (the reference's TORCH_CHECK convention)."""
    if code != 0:
        raise RuntimeError(f"{what}: {error_string(code)} (code {code})")

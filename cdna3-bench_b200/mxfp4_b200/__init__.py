"""mxfp4_b200: MXFP4-weight x BF16-activation GEMM for NVIDIA B200 (sm_100a).

Drop-in for the operator surface of the reference package ``mxfp4_cdna3``
(python/mxfp4_cdna3/__init__.py:1-22): the same names resolve lazily to the CUDA
implementations in :mod:`mxfp4_b200.kernels`, so importing the package needs neither
torch nor a GPU; calling an operator without a CUDA device raises RuntimeError.
"""

__version__ = "0.1.0"

_OPS = (
    "quantize_mxfp4",
    "quantize_mxfp4_ocp",
    "dequantize_mxfp4",
    "ref_gemm",
    "preshuffle_b",
    "prepack_b_mxfp4",
    "prepack_b200",
    "dequantize_prepacked",
    "MXFP4Weight",
    "gemm",
    "gemm_packed",
    "workspace_bytes",
    "gemm_auto",
    "gemm_a",
    "gemm_b",
    "gemm_c",
    "gemm_d",
    "gemm_e",
    "gemm_f",
    "gemm_g",
    "gemm_h",
    "gemm_i",
    "gemm_j",
    "gemm_k",
    "gemm_m",
    "select_path",
    "shape_supported",
    "shape_supported_c",
    "shape_supported_d",
    "shape_supported_e",
    "shape_supported_f",
    "shape_supported_g",
    "device_info",
    "device_error",
    "MXWeight",
    "prepack_mx",
    "quantize_act_mx8",
    "gemm_mx",
)

__all__ = list(_OPS)


def __getattr__(name):
    if name in _OPS:
        from . import kernels

        return getattr(kernels, name)
    raise AttributeError(name)

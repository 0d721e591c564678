"""Torch-facing operator surface of the B200 library.

Mirrors the reference package's operator module (python/mxfp4_cdna3/kernels.py:11-94 and
csrc/mxfp4_ext.cpp:11-225): ``gemm_a .. gemm_m``, ``gemm_g``, ``gemm_auto``,
``shape_supported_{c,d,e,f,g}``, ``device_info`` and ``prepack_b_mxfp4`` keep their names,
argument meaning and error behaviour (invalid inputs raise RuntimeError, C is fp32 [M, N]
and is allocated when not given).  Every call runs on the current CUDA stream through the
C ABI in ``include/mxfp4_b200.h``; there is no CPU path.

B200 additions: ``prepack_b200`` / :class:`MXFP4Weight` (weights re-laid once for the
tensor-core kernels), ``gemm`` (bf16 or fp32 output, explicit path choice), GPU
quantisers (reference rule and OCP MX rule) and dequantisers.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

_GROUP = 32


# ----------------------------------------------------------------------------- helpers
def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _require_cuda():
    if not torch.cuda.is_available():
        raise RuntimeError("mxfp4_b200 needs a CUDA device (sm_100); there is no CPU fallback")


def _to_device(x, dtype=None) -> torch.Tensor:
    _require_cuda()
    if isinstance(x, np.ndarray):
        x = torch.from_numpy(np.ascontiguousarray(x))
    if dtype is not None and x.dtype != dtype:
        x = x.to(dtype)
    if not x.is_cuda:
        x = x.cuda()
    return x.contiguous()


def _check(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


# ----------------------------------------------------------------------------- formats
def quantize_mxfp4(x, axis=-1, rule: str = "ref"):
    """MXFP4-quantise a 2-D float array along ``axis`` on the GPU.

    ``rule="ref"`` is byte-identical to the reference quantiser (ref.py:14-47);
    ``rule="ocp"`` is the OCP MX rule (floor(log2 amax) - 2, RNE, saturate at 6).
    NumPy input returns NumPy arrays, tensor input returns CUDA tensors.
    """
    as_numpy = isinstance(x, np.ndarray)
    xt = _to_device(x, torch.float32)
    _check(xt.dim() == 2, "quantize_mxfp4: only 2-D inputs are supported")
    ax = axis % 2
    rows, cols = xt.shape
    qlen = rows if ax == 0 else cols
    if qlen % _GROUP:
        raise ValueError(f"axis {axis} length {qlen} not divisible by {_GROUP}")
    if ax == 0:
        packed = torch.empty((rows // 2, cols), dtype=torch.uint8, device=xt.device)
        scales = torch.empty((rows // _GROUP, cols), dtype=torch.uint8, device=xt.device)
    else:
        packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=xt.device)
        scales = torch.empty((rows, cols // _GROUP), dtype=torch.uint8, device=xt.device)
    r = {"ref": _lib.RULE_REF, "ocp": _lib.RULE_OCP}[rule]
    _lib.check(
        _lib.lib().mxfp4_quantize(_ptr(xt), rows, cols, ax, r, _ptr(packed), _ptr(scales), _stream()),
        "mxfp4_quantize",
    )
    if as_numpy:
        return packed.cpu().numpy(), scales.cpu().numpy()
    return packed, scales


def quantize_mxfp4_ocp(x, axis=-1):
    return quantize_mxfp4(x, axis=axis, rule="ocp")


def dequantize_mxfp4(packed, scales, axis=-1, dtype=torch.float32):
    """GPU dequantiser (ref.py:50-72).  2-D only: axis 0 is the reference weight layout
    ([K/2, N] -> [K, N]); axis 1/-1 is row-major weights ([N, K/2] -> [N, K])."""
    as_numpy = isinstance(packed, np.ndarray)
    p = _to_device(packed, torch.uint8)
    s = _to_device(scales, torch.uint8)
    _check(p.dim() == 2 and s.dim() == 2, "dequantize_mxfp4: only 2-D inputs are supported")
    ax = axis % 2
    if ax == 0:
        K, N = p.shape[0] * 2, p.shape[1]
        _check(tuple(s.shape) == (K // _GROUP, N), "dequantize_mxfp4: scales shape")
        out = torch.empty((K, N), dtype=dtype, device=p.device)
        layout = _lib.LAYOUT_REF
    else:
        N, K = p.shape[0], p.shape[1] * 2
        _check(tuple(s.shape) == (N, K // _GROUP), "dequantize_mxfp4: scales shape")
        out = torch.empty((N, K), dtype=dtype, device=p.device)
        layout = _lib.LAYOUT_NK
    od = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}[dtype]
    _lib.check(
        _lib.lib().mxfp4_dequantize(_ptr(p), _ptr(s), K, N, layout, _ptr(out), od, _stream()),
        "mxfp4_dequantize",
    )
    return out.cpu().numpy() if as_numpy else out


def ref_gemm(A_bf16, B_packed, B_scales):
    """fp32 A @ dequant(B) (ref.py:75-78) on the GPU: exact dequant, then an fp32 library
    matmul.  A plain reference product for checking, not the fused hot path."""
    as_numpy = isinstance(A_bf16, np.ndarray)
    A = _to_device(A_bf16)
    A32 = A.float()
    Bd = dequantize_mxfp4(_to_device(B_packed), _to_device(B_scales), axis=0)
    C = A32 @ Bd
    return C.cpu().numpy() if as_numpy else C


def preshuffle_b(B_packed, B_scales, N_tile=128, K_tile=128):
    """Identity, kept for interface parity with the reference (ref.py:81-82)."""
    return B_packed, B_scales


def prepack_b_mxfp4(B_packed, B_scales, n_tile=128):
    """The reference's strategy-G layout (ref.py:85-101), computed with tensor ops.

    Returns flat uint8 (B_prep, Bs_prep) of the same type as the input (NumPy or torch)."""
    as_numpy = isinstance(B_packed, np.ndarray)
    bp = torch.as_tensor(np.ascontiguousarray(B_packed)) if as_numpy else B_packed.contiguous()
    bs = torch.as_tensor(np.ascontiguousarray(B_scales)) if as_numpy else B_scales.contiguous()
    K2, N = bp.shape
    if N % n_tile:
        raise AssertionError("N must be a multiple of n_tile")
    nb = N // n_tile
    prep = bp.reshape(K2 // 4, 4, nb, n_tile).permute(2, 0, 3, 1).contiguous().reshape(-1)
    sprep = bs.reshape(-1, nb, n_tile).permute(1, 0, 2).contiguous().reshape(-1)
    if as_numpy:
        return prep.numpy(), sprep.numpy()
    return prep, sprep


@dataclass
class MXFP4Weight:
    """Weights in the B200 chunk layout (see include/mxfp4_b200.h), ready for :func:`gemm`."""

    data: torch.Tensor  # uint8, mxfp4_prepacked_bytes(N, K) bytes
    N: int
    K: int

    def nbytes_streamed(self) -> int:
        return self.N * self.K // 2 + self.N * self.K // _GROUP


_LAYOUTS = {"ref": _lib.LAYOUT_REF, "nk": _lib.LAYOUT_NK, "g": _lib.LAYOUT_G, "prepacked": _lib.LAYOUT_PREPACKED}


def prepack_b200(B_packed, B_scales, layout: str = "ref", N: int | None = None, K: int | None = None):
    """Re-lay MXFP4 weights into the chunk layout the tensor-core kernels stream.

    layout "ref": B_packed [K/2, N], B_scales [K/32, N] (reference layout);
    layout "nk":  [N, K/2], [N, K/32];  layout "g": the strategy-G flat arrays (give N, K).
    """
    p = _to_device(B_packed, torch.uint8)
    s = _to_device(B_scales, torch.uint8)
    if layout == "ref":
        K, N = p.shape[0] * 2, p.shape[1]
    elif layout == "nk":
        N, K = p.shape[0], p.shape[1] * 2
    else:
        _check(N is not None and K is not None, "prepack_b200: layout 'g' needs N and K")
    L = _lib.lib()
    out = torch.empty(L.mxfp4_prepacked_bytes(N, K), dtype=torch.uint8, device=p.device)
    _lib.check(L.mxfp4_prepack(_ptr(p), _ptr(s), N, K, _LAYOUTS[layout], _ptr(out), _stream()), "mxfp4_prepack")
    return MXFP4Weight(out, N, K)


def dequantize_prepacked(w: MXFP4Weight) -> torch.Tensor:
    """bf16 [N, K] produced by the tensor-core kernel's own dequant routine."""
    out = torch.empty((w.N, w.K), dtype=torch.bfloat16, device=w.data.device)
    _lib.check(
        _lib.lib().mxfp4_dequantize_prepacked(_ptr(w.data), w.N, w.K, _ptr(out), _stream()),
        "mxfp4_dequantize_prepacked",
    )
    return out


# ----------------------------------------------------------------------------- GEMMs
_ODT = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _check_A(A: torch.Tensor, K: int | None = None):
    _check(isinstance(A, torch.Tensor) and A.is_cuda, "all tensors must be on GPU")
    _check(A.dtype == torch.bfloat16, "A must be bfloat16")
    _check(A.dim() == 2, "A shape")
    _check(A.is_contiguous(), "tensors must be contiguous")
    if K is not None:
        _check(A.shape[1] == K, "A shape")


def gemm(A: torch.Tensor, w: MXFP4Weight, out_dtype=torch.bfloat16, path: str = "auto", C=None):
    """C[M, N] = A[M, K] @ dequant(w)^T with fp32 accumulation (bf16 or fp32 output)."""
    _check_A(A, w.K)
    M = A.shape[0]
    if C is None:
        C = torch.empty((M, w.N), dtype=out_dtype, device=A.device)
    _check(C.is_cuda and C.dtype in _ODT and tuple(C.shape) == (M, w.N) and C.is_contiguous(), "C shape/contig")
    L = _lib.lib()
    # decode shapes: room for the activations converted once per call (torch's caching allocator)
    nws = L.mxfp4_gemm_workspace_bytes(M, w.N, w.K, _lib.LAYOUT_PREPACKED)
    ws = torch.empty(nws, dtype=torch.uint8, device=A.device) if nws else None
    _lib.check(
        L.mxfp4_gemm(
            _ptr(A), _ptr(w.data), None, _ptr(C), _ODT[C.dtype], M, w.N, w.K,
            _lib.LAYOUT_PREPACKED, _lib.PATH_NAMES[path], _ptr(ws) if ws is not None else None, nws, _stream(),
        ),
        "mxfp4_gemm",
    )
    return C


def gemm_allgather(A: torch.Tensor, w: MXFP4Weight, dst_ptrs, n_off: int, ldc: int,
                   out_dtype=torch.bfloat16, path: str = "auto"):
    """This GPU's columns of C = A @ dequant(w)^T, written straight into every buffer in
    `dst_ptrs` (device addresses of the [M, ldc] outputs of all GPUs, peers' opened with
    :func:`ipc_open`) at columns n_off .. n_off + w.N - 1.  Returns nothing; the caller orders
    later reads of the peers' writes (a collective on the same stream on every GPU)."""
    _check_A(A, w.K)
    M = A.shape[0]
    L = _lib.lib()
    arr = (ctypes.c_void_p * len(dst_ptrs))(*[int(p) for p in dst_ptrs])
    nws = L.mxfp4_gemm_workspace_bytes(M, w.N, w.K, _lib.LAYOUT_PREPACKED)
    ws = torch.empty(nws, dtype=torch.uint8, device=A.device) if nws else None
    _lib.check(
        L.mxfp4_gemm_allgather(_ptr(A), _ptr(w.data), arr, len(dst_ptrs), n_off, ldc, _ODT[out_dtype], M, w.N, w.K,
                               _lib.PATH_NAMES[path], _ptr(ws) if ws is not None else None, nws, _stream()),
        "mxfp4_gemm_allgather",
    )


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """(handle, offset) through which another process on this node maps `t`'s memory."""
    L = _lib.lib()
    h = ctypes.create_string_buffer(L.mxfp4_ipc_handle_bytes())
    off = ctypes.c_size_t(0)
    _lib.check(L.mxfp4_ipc_export(_ptr(t), h, ctypes.byref(off)), "mxfp4_ipc_export")
    return h.raw, off.value


def ipc_open(handle: bytes, offset: int) -> int:
    """Device address, in this process, of memory another process exported."""
    p = ctypes.c_void_p(0)
    _lib.check(_lib.lib().mxfp4_ipc_open(handle, offset, ctypes.byref(p)), "mxfp4_ipc_open")
    return int(p.value)


def ipc_close(ptr: int, offset: int) -> None:
    _lib.check(_lib.lib().mxfp4_ipc_close(ctypes.c_void_p(ptr), offset), "mxfp4_ipc_close")


def copy_columns(dst_ptr: int, dst_pitch: int, src_ptr: int, src_pitch: int, width_bytes: int, rows: int,
                 stream: torch.cuda.Stream | None = None) -> None:
    """Pitched device-to-device copy of `rows` rows of `width_bytes` on `stream` (default: the
    current stream) by the copy engines; `dst_ptr` may be a peer's buffer from :func:`ipc_open`."""
    s = ctypes.c_void_p(stream.cuda_stream) if stream is not None else _stream()
    _lib.check(_lib.lib().mxfp4_copy_columns(ctypes.c_void_p(int(dst_ptr)), dst_pitch, ctypes.c_void_p(int(src_ptr)),
                                             src_pitch, width_bytes, rows, s),
               "mxfp4_copy_columns")


def _gemm_layout(A, B, Bs, C, layout: int, N: int, K: int, path: int, name: str):
    M = A.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    _check(C.is_cuda and C.dtype == torch.float32, "C must be float32")
    _check(C.dim() == 2 and tuple(C.shape) == (M, N), "C shape")
    _check(C.is_contiguous(), "tensors must be contiguous")
    L = _lib.lib()
    ws = torch.empty(max(1, L.mxfp4_gemm_workspace_bytes(M, N, K, layout)), dtype=torch.uint8, device=A.device)
    _lib.check(
        L.mxfp4_gemm(_ptr(A), _ptr(B), _ptr(Bs), _ptr(C), _lib.DTYPE_F32, M, N, K, layout, path,
                     _ptr(ws), ws.numel(), _stream()),
        name,
    )
    return C


def workspace_bytes(M: int, N: int, K: int, layout: str = "ref") -> int:
    return int(_lib.lib().mxfp4_gemm_workspace_bytes(M, N, K, _LAYOUTS[layout]))


def gemm_packed(A, B_packed, B_scales, out_dtype=torch.bfloat16, layout: str = "ref", C=None,
                workspace=None, path: str = "auto"):
    """C = A @ dequant(B) for weights in the reference ([K/2,N]) or row-major ([N,K/2]) layout,
    bf16 or fp32 output.  The weights are re-laid into ``workspace`` (allocated when not given,
    ``workspace_bytes`` long) inside the same call, so this is the one-call drop-in path."""
    _check_A(A)
    M, K = A.shape
    N = B_packed.shape[1] if layout == "ref" else B_packed.shape[0]
    if C is None:
        C = torch.empty((M, N), dtype=out_dtype, device=A.device)
    _check(C.is_cuda and C.dtype in _ODT and tuple(C.shape) == (M, N) and C.is_contiguous(), "C shape/contig")
    need = workspace_bytes(M, N, K, layout)
    if workspace is None:
        workspace = torch.empty(max(1, need), dtype=torch.uint8, device=A.device)
    _check(workspace.numel() >= need, "workspace too small")
    _lib.check(
        _lib.lib().mxfp4_gemm(_ptr(A), _ptr(B_packed), _ptr(B_scales), _ptr(C), _ODT[C.dtype], M, N, K,
                              _LAYOUTS[layout], _lib.PATH_NAMES[path], _ptr(workspace), workspace.numel(),
                              _stream()),
        "mxfp4_gemm",
    )
    return C


def _check_ref_inputs(A, B_packed, B_scales):
    for t in (A, B_packed, B_scales):
        _check(isinstance(t, torch.Tensor) and t.is_cuda, "all tensors must be on GPU")
    _check_A(A)
    _check(B_packed.dtype == torch.uint8, "B_packed must be uint8")
    _check(B_scales.dtype == torch.uint8, "B_scales must be uint8")
    M, K = A.shape
    N = B_packed.shape[1] if B_packed.dim() == 2 else -1
    _check(B_packed.dim() == 2 and B_packed.shape[0] == K // 2, "B_packed shape")
    _check(B_scales.dim() == 2 and tuple(B_scales.shape) == (K // _GROUP, N), "B_scales shape")
    _check(B_packed.is_contiguous() and B_scales.is_contiguous(), "tensors must be contiguous")
    _check(K % _GROUP == 0, "K must be a multiple of 32")
    return M, N, K


def gemm_auto(A, B_packed, B_scales, C=None):
    """Reference-layout entry point: C (fp32) = A @ dequant(B); the cost model picks the path."""
    M, N, K = _check_ref_inputs(A, B_packed, B_scales)
    return _gemm_layout(A, B_packed, B_scales, C, _lib.LAYOUT_REF, N, K, _lib.PATH_AUTO, "gemm_auto")


def gemm_a(A, B_packed, B_scales, C=None):
    """Two-pass path (the reference's strategy A, strategy_a_two_pass.cu:39-116): dequantise B
    exactly into a scratch matrix, then a library GEMM that accumulates and writes fp32.

    The scratch holds the dequantised weights in fp32 and the GEMM runs in fp32 with TF32 off:
    every product of a bf16 activation and a dequantised weight is exact in fp32, so C is the
    fp32-accumulated product the reference's strategy A writes, not a bf16-rounded one.  Like
    the reference it allocates its scratch on every call; it is the unfused baseline, not a
    fast path."""
    M, N, K = _check_ref_inputs(A, B_packed, B_scales)
    if C is None:
        C = torch.empty((M, N), dtype=torch.float32, device=A.device)
    _check(C.is_cuda and C.dtype == torch.float32, "C must be float32")
    _check(tuple(C.shape) == (M, N) and C.is_contiguous(), "C shape/contig")
    Bd = dequantize_mxfp4(B_packed, B_scales, axis=0, dtype=torch.float32)  # [K, N], exact
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        torch.matmul(A.float(), Bd, out=C)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return C


def _fused(path: int, name: str):
    def fn(A, B_packed, B_scales, C=None):
        M, N, K = _check_ref_inputs(A, B_packed, B_scales)
        return _gemm_layout(A, B_packed, B_scales, C, _lib.LAYOUT_REF, N, K, path, name)

    fn.__name__ = name
    fn.__doc__ = (
        f"Drop-in for the reference's {name}: fused dequant + tensor-core GEMM, fp32 C. "
        "The reference's variants B..M (different CDNA3 schedules of one op) all map to the "
        "B200 kernel the cost model picks."
    )
    return fn


gemm_b = _fused(_lib.PATH_AUTO, "gemm_b")
gemm_c = _fused(_lib.PATH_AUTO, "gemm_c")
gemm_d = _fused(_lib.PATH_AUTO, "gemm_d")
gemm_e = _fused(_lib.PATH_AUTO, "gemm_e")
gemm_f = _fused(_lib.PATH_AUTO, "gemm_f")
gemm_h = _fused(_lib.PATH_AUTO, "gemm_h")
gemm_i = _fused(_lib.PATH_AUTO, "gemm_i")
gemm_k = _fused(_lib.PATH_AUTO, "gemm_k")
gemm_j = _fused(_lib.PATH_AUTO, "gemm_j")
gemm_m = _fused(_lib.PATH_AUTO, "gemm_m")


def gemm_g(A, B_prep, Bs_prep, C=None):
    """Strategy-G entry point: weights in the reference's prepacked layout, N inferred from
    the byte count (csrc/mxfp4_ext.cpp:127-154)."""
    for t in (A, B_prep, Bs_prep):
        _check(isinstance(t, torch.Tensor) and t.is_cuda, "all tensors on GPU")
    _check(A.dtype == torch.bfloat16, "A bf16")
    _check(B_prep.dtype == torch.uint8, "B_prep uint8")
    _check(Bs_prep.dtype == torch.uint8, "Bs_prep uint8")
    M, K = A.shape
    _check(K % 2 == 0 and B_prep.numel() % (K // 2) == 0, "B_prep size not consistent with K/2 byte stride")
    N = B_prep.numel() // (K // 2)
    _check(Bs_prep.numel() == K * N // 32, "Bs_prep size != K*N/32")
    _check(N % 128 == 0 and K % 64 == 0, "Strategy G requires N%128==0, K%64==0")
    _check(A.is_contiguous() and B_prep.is_contiguous() and Bs_prep.is_contiguous(), "tensors contiguous")
    return _gemm_layout(A, B_prep, Bs_prep, C, _lib.LAYOUT_G, N, K, _lib.PATH_AUTO, "gemm_g")


# ----------------------------------------------------------------------------- queries
def select_path(M: int, N: int, K: int) -> str:
    code = _lib.lib().mxfp4_select_path(M, N, K)
    return {v: k for k, v in _lib.PATH_NAMES.items()}[code]


def shape_supported(path: str, M: int, N: int, K: int) -> bool:
    return bool(_lib.lib().mxfp4_shape_supported(_lib.PATH_NAMES[path], M, N, K))


def shape_supported_c(M, N, K):
    return shape_supported("auto", M, N, K)


shape_supported_d = shape_supported_e = shape_supported_f = shape_supported_g = shape_supported_c


def device_info(dev_id=0) -> dict:
    info = _lib.DeviceInfo()
    _lib.check(_lib.lib().mxfp4_device_info_get(int(dev_id), ctypes.byref(info)), "mxfp4_device_info_get")
    return {
        "name": info.name.decode(),
        "gcn_arch_name": f"sm_{info.major}{info.minor}",
        "multi_processor_count": info.multi_processor_count,
        "total_global_mem": info.total_global_mem,
        "shared_mem_per_block": info.shared_mem_per_block,
        "warp_size": info.warp_size,
        "shared_mem_per_block_optin": info.shared_mem_per_block_optin,
        "l2_cache_size": info.l2_cache_size,
        "clock_rate_khz": info.clock_rate_khz,
        "memory_clock_rate_khz": info.memory_clock_rate_khz,
        "memory_bus_width": info.memory_bus_width,
    }


def device_error(clear: bool = True) -> int:
    """Device error word set by a kernel's bounded wait giving up (0 = none)."""
    code = ctypes.c_uint(0)
    _lib.check(_lib.lib().mxfp4_device_error(int(clear), ctypes.byref(code)), "mxfp4_device_error")
    return code.value


# ----------------------------------------------------------------------------- block-scaled paths
# Activations coded as E4M3 pieces with E8M0 scales, both operands' scales applied by the
# tensor core's block-scaled MMA.  mode "q8": one OCP MXFP8 piece; "split2": hi + residual,
# every element within 2**-8 of its group max.  Reference: oracle.ref_gemm_mx.


@dataclass
class MXWeight:
    """Weights in the block-scaled layout (nibbles [Np][Kp/2] + scale blocks)."""

    data: torch.Tensor  # uint8, mxfp4_mx_weight_bytes(N, K) bytes
    N: int
    K: int


def prepack_mx(B_packed, B_scales, layout: str = "ref") -> MXWeight:
    """Re-lay MXFP4 weights (layout "ref": [K/2, N] + [K/32, N]; "nk": [N, K/2] + [N, K/32])
    for :func:`gemm_mx`."""
    p = _to_device(B_packed, torch.uint8)
    s = _to_device(B_scales, torch.uint8)
    _check(layout in ("ref", "nk"), "prepack_mx: layout must be 'ref' or 'nk'")
    if layout == "ref":
        K, N = p.shape[0] * 2, p.shape[1]
    else:
        N, K = p.shape[0], p.shape[1] * 2
    L = _lib.lib()
    out = torch.empty(L.mxfp4_mx_weight_bytes(N, K), dtype=torch.uint8, device=p.device)
    _lib.check(L.mxfp4_prepack_mx(_ptr(p), _ptr(s), N, K, _LAYOUTS[layout], _ptr(out), _stream()), "mxfp4_prepack_mx")
    return MXWeight(out, N, K)


def mx_code_rows(M: int, mode: str) -> int:
    """Code rows of the coded-activation operand (see include/mxfp4_b200.h)."""
    if M <= 16:
        return 32
    return -(-M // 256) * 256 if mode == "q8" else 2 * (-(-M // 128) * 128)


def quantize_act_mx8(A: torch.Tensor, mode: str = "q8"):
    """The block-scaled GEMM's activation coding of bf16 A[M, K].
    Returns (codes uint8 [rows, Kp], scale blocks uint8 [Kp/128, rows_sf/128, 512])."""
    _check_A(A)
    _check(mode in _lib.MX_MODES, "mode must be 'q8' or 'split2'")
    M, K = A.shape
    L = _lib.lib()
    Kp, rows = -(-K // 128) * 128, mx_code_rows(M, mode)
    rows_sf = -(-rows // 128) * 128
    codes_bytes = -(-(rows * Kp) // 256) * 256
    ws = torch.empty(L.mxfp4_mx_workspace_bytes(M, 8, K, _lib.MX_MODES[mode]), dtype=torch.uint8, device=A.device)
    _lib.check(L.mxfp4_quantize_act_mx8(_ptr(A), M, K, _lib.MX_MODES[mode], _ptr(ws), _stream()),
               "mxfp4_quantize_act_mx8")
    codes = ws[: rows * Kp].view(rows, Kp)
    blocks = ws[codes_bytes: codes_bytes + rows_sf * Kp // 32].view(Kp // 128, rows_sf // 128, 512)
    return codes, blocks


def gemm_mx(A: torch.Tensor, w: MXWeight, out_dtype=torch.bfloat16, mode: str = "q8", C=None):
    """C[M, N] = A' @ dequant(w)^T on the block-scaled tensor-core path (A' = A coded per `mode`)."""
    _check_A(A, w.K)
    _check(mode in _lib.MX_MODES, "mode must be 'q8' or 'split2'")
    M = A.shape[0]
    if C is None:
        C = torch.empty((M, w.N), dtype=out_dtype, device=A.device)
    _check(C.is_cuda and C.dtype in _ODT and tuple(C.shape) == (M, w.N) and C.is_contiguous(), "C shape/contig")
    L = _lib.lib()
    md = _lib.MX_MODES[mode]
    nws = L.mxfp4_mx_workspace_bytes(M, w.N, w.K, md)
    ws = torch.empty(nws, dtype=torch.uint8, device=A.device)
    _lib.check(
        L.mxfp4_gemm_mx(_ptr(A), _ptr(w.data), _ptr(C), _ODT[C.dtype], M, w.N, w.K, md, _ptr(ws), nws, _stream()),
        "mxfp4_gemm_mx",
    )
    return C

"""Zero-copy PyTorch entry points over the C ABI (``xrgpu_mmnb_forward``).

Tensors stay on the device; the kernels run on the current torch CUDA stream. torch
supplies device memory and streams only: every numerical step runs in this package's
CUDA kernels.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _native
from ._native import check

_PATHS = {"auto": _native.PATH_AUTO, "generic": _native.PATH_GENERIC, "gemv": _native.PATH_GEMV,
          "gemm": _native.PATH_GEMM}


def _dtype_code(t: torch.dtype) -> int:
    if t == torch.float32:
        return _native.FLOAT32
    if t == torch.float16:
        return _native.FLOAT16
    raise ValueError(f"MatMulNBits T1 must be float32 or float16, got {t}")


def _zp_code(zp: Optional[torch.Tensor]) -> int:
    if zp is None:
        return _native.UNSPECIFIED
    if zp.dtype == torch.uint8:
        return _native.UINT8
    if zp.dtype == torch.float32:
        return _native.FLOAT32
    if zp.dtype == torch.float16:
        return _native.FLOAT16
    raise ValueError("zero_points must be float32/float16 (contract) or packed uint8")


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _problem(a, b, scales, zero_points, bias, y, *, K, N, bits, block_size, path, ldy=0, dtype=None):
    p = _native.Problem_()
    p.dtype = _dtype_code(dtype if dtype is not None else a.dtype)
    p.zero_point_dtype = _zp_code(zero_points)
    p.path = _PATHS[path]
    p.M = 0 if a is None else a.numel() // K
    p.K, p.N, p.block_size, p.bits = int(K), int(N), int(block_size), int(bits)
    p.a, p.b, p.scales = _ptr(a), _ptr(b), _ptr(scales)
    p.zero_points, p.bias, p.y = _ptr(zero_points), _ptr(bias), _ptr(y)
    p.ldy = int(ldy)
    return p


def _require(t: Optional[torch.Tensor], name: str, device):
    if t is None:
        return
    if not t.is_cuda or t.device != device:
        raise ValueError(f"{name} must be a CUDA tensor on {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def matmul_nbits(a: torch.Tensor, b: torch.Tensor, scales: torch.Tensor, zero_points: Optional[torch.Tensor] = None,
                 bias: Optional[torch.Tensor] = None, *, K: Optional[int] = None, N: Optional[int] = None,
                 bits: int = 4, block_size: int = 32, out: Optional[torch.Tensor] = None, path: str = "auto",
                 workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Y = A . dequant(B)^T (+ bias) for com.microsoft.MatMulNBits on the current CUDA stream.

    Shapes: a [..., K] (T1), b uint8 [N, ceil(K/bs), ceil(bs*bits/8)], scales [N, ceil(K/bs)] (T1),
    zero_points float [N, ceil(K/bs)] or packed uint8 [N, ceil(ceil(K/bs)*bits/8)], bias [N] (T1).
    ``out`` may be a [..., >=N] view whose last-dim stride is 1 (rows may be strided).
    """
    K = int(a.shape[-1]) if K is None else int(K)
    N = int(b.shape[0]) if N is None else int(N)
    dev = a.device
    for t, name in ((a, "a"), (b, "b"), (scales, "scales"), (zero_points, "zero_points"), (bias, "bias")):
        _require(t, name, dev)
    if out is None:
        out = torch.empty(tuple(a.shape[:-1]) + (N,), dtype=a.dtype, device=dev)
        ldy = N
    else:
        if out.dtype != a.dtype or out.device != dev or out.stride(-1) != 1 or out.shape[-1] != N:
            raise ValueError("out must match a's dtype/device, end with N columns and have unit column stride")
        ldy = out.stride(-2) if out.dim() >= 2 else N
    p = _problem(a, b, scales, zero_points, bias, out, K=K, N=N, bits=bits, block_size=block_size, path=path, ldy=ldy)
    lib = _native.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        ws_ptr, ws_bytes = ctypes.c_void_p(workspace.data_ptr()), workspace.numel() * workspace.element_size()
    if torch.cuda.current_device() == dev.index:
        check(lib.xrgpu_mmnb_forward(ctypes.byref(p), ws_ptr, ws_bytes, ctypes.c_void_p(stream)))
    else:
        with torch.cuda.device(dev):
            check(lib.xrgpu_mmnb_forward(ctypes.byref(p), ws_ptr, ws_bytes, ctypes.c_void_p(stream)))
    return out


def workspace_size(a_rows: int, *, K: int, N: int, bits: int = 4, block_size: int = 32, dtype=torch.float16,
                   zero_points_dtype=None, path: str = "auto") -> int:
    """Device scratch bytes ``matmul_nbits`` needs for this shape (0 when none)."""
    p = _native.Problem_()
    p.dtype = _dtype_code(dtype)
    p.zero_point_dtype = {None: _native.UNSPECIFIED, torch.uint8: _native.UINT8, torch.float32: _native.FLOAT32,
                          torch.float16: _native.FLOAT16}[zero_points_dtype]
    p.path = _PATHS[path]
    p.M, p.K, p.N, p.block_size, p.bits = int(a_rows), int(K), int(N), int(block_size), int(bits)
    p.a = p.b = p.scales = p.y = ctypes.c_void_p(256)
    if zero_points_dtype is not None:
        p.zero_points = ctypes.c_void_p(256)
    need = ctypes.c_uint64(0)
    check(_native.load().xrgpu_mmnb_workspace_size(ctypes.byref(p), ctypes.byref(need)))
    return int(need.value)


def select_path(a: torch.Tensor, b, scales, zero_points=None, *, K=None, N=None, bits=4, block_size=32,
                path: str = "auto") -> str:
    K = int(a.shape[-1]) if K is None else int(K)
    N = int(b.shape[0]) if N is None else int(N)
    p = _problem(a, b, scales, zero_points, None, None, K=K, N=N, bits=bits, block_size=block_size, path=path)
    buf = ctypes.create_string_buffer(32)
    check(_native.load().xrgpu_mmnb_select_path(ctypes.byref(p), buf, len(buf)))
    return buf.value.decode()


def dequantize(b: torch.Tensor, scales: torch.Tensor, zero_points: Optional[torch.Tensor] = None, *, K: int,
               bits: int = 4, block_size: int = 32) -> torch.Tensor:
    """Exact float32 W[N, K] = (float(q) - z) * s on the device (nbitWeight)."""
    N = int(b.shape[0])
    dev = b.device
    for t, name in ((b, "b"), (scales, "scales"), (zero_points, "zero_points")):
        _require(t, name, dev)
    w = torch.empty((N, K), dtype=torch.float32, device=dev)
    p = _problem(None, b, scales, zero_points, None, None, K=K, N=N, bits=bits, block_size=block_size, path="auto",
                 dtype=scales.dtype)
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        check(_native.load().xrgpu_mmnb_dequantize(ctypes.byref(p), ctypes.c_void_p(w.data_ptr()),
                                                    ctypes.c_void_p(stream)))
    return w


def device_error(device: int = 0, clear: bool = True) -> int:
    code = ctypes.c_uint32(0)
    check(_native.load().xrgpu_device_error(int(device), ctypes.byref(code), int(clear)))
    return int(code.value)

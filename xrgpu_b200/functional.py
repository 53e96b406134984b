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


# ---------------------------------------------------------------------------------------------
# Operators around MatMulNBits (zero-copy, current CUDA stream).
_ACTIVATIONS = {"none": 0, "identity": 0, "relu": 1, "silu": 2, "swish": 2, "gelu": 3, "tanh": 4, "sigmoid": 5,
                "swiglu": 6}


def _act_code(activation) -> int:
    if isinstance(activation, int):
        return activation
    if activation not in _ACTIVATIONS:
        raise ValueError(f"Unknown fused activation: {activation}")
    return _ACTIVATIONS[activation]


def _workspace(nbytes: int, device) -> Optional[torch.Tensor]:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device) if nbytes else None


def _call(fn, prob, ws, device):
    stream = torch.cuda.current_stream(device).cuda_stream
    args = [ctypes.byref(prob)]
    if ws is not False:
        args += [ctypes.c_void_p(ws.data_ptr()) if ws is not None else None,
                 (ws.numel() if ws is not None else 0)]
    args.append(ctypes.c_void_p(stream))
    with torch.cuda.device(device):
        check(fn(*args))


def matmul_nbits_mlp(a, gate_b, gate_scales, up_b, up_scales, *, skip=None, norm_scale=None, gate_bias=None,
                     up_bias=None, K: Optional[int] = None, N: Optional[int] = None, bits: int = 4, block_size: int = 32,
                     activation="silu", epsilon: float = 1e-5, want_residual: bool = False):
    """com.microsoft.MatMulNBitsMlp: y = fused(x.gate^T + gate_bias) * (x.up^T + up_bias), x = a + skip,
    RMS-normalised by norm_scale when given. Returns y, or (y, residual) with want_residual."""
    K = int(a.shape[-1]) if K is None else int(K)
    N = int(gate_b.shape[0]) if N is None else int(N)
    dev = a.device
    for t, n in ((a, "a"), (gate_b, "gate_b"), (gate_scales, "gate_scales"), (up_b, "up_b"), (up_scales, "up_scales"),
                 (skip, "skip"), (norm_scale, "norm_scale"), (gate_bias, "gate_bias"), (up_bias, "up_bias")):
        _require(t, n, dev)
    y = torch.empty(tuple(a.shape[:-1]) + (N,), dtype=a.dtype, device=dev)
    res = torch.empty_like(a) if want_residual else None
    p = _native.MlpProblem_()
    p.dtype = _dtype_code(a.dtype)
    p.activation = _act_code(activation)
    p.M, p.K, p.N, p.block_size, p.bits = a.numel() // K, K, N, int(block_size), int(bits)
    p.epsilon = float(epsilon)
    p.a, p.skip, p.norm_scale = _ptr(a), _ptr(skip), _ptr(norm_scale)
    p.gate_b, p.gate_scales, p.gate_bias = _ptr(gate_b), _ptr(gate_scales), _ptr(gate_bias)
    p.up_b, p.up_scales, p.up_bias = _ptr(up_b), _ptr(up_scales), _ptr(up_bias)
    p.y, p.residual = _ptr(y), _ptr(res)
    lib = _native.load()
    need = ctypes.c_uint64(0)
    check(lib.xrgpu_mlp_workspace_size(ctypes.byref(p), ctypes.byref(need)))
    _call(lib.xrgpu_mlp_forward, p, _workspace(need.value, dev), dev)
    return (y, res) if want_residual else y


def matmul_nbits_qkv(a, norm_scale, q_b, q_scales, k_b, k_scales, v_b, v_scales, *, skip=None, K: Optional[int] = None,
                     Nq: Optional[int] = None, Nkv: Optional[int] = None, bits: int = 4, block_size: int = 32,
                     epsilon: float = 1e-6, want_residual: bool = False):
    """com.microsoft.MatMulNBitsQkv: q, k, v = x.W^T with x = RMSNorm(a + skip) * norm_scale.
    Returns (q, k, v) or (q, k, v, residual)."""
    K = int(a.shape[-1]) if K is None else int(K)
    Nq = int(q_b.shape[0]) if Nq is None else int(Nq)
    Nkv = int(k_b.shape[0]) if Nkv is None else int(Nkv)
    dev = a.device
    for t, n in ((a, "a"), (norm_scale, "norm_scale"), (skip, "skip"), (q_b, "q_b"), (q_scales, "q_scales"),
                 (k_b, "k_b"), (k_scales, "k_scales"), (v_b, "v_b"), (v_scales, "v_scales")):
        _require(t, n, dev)
    lead = tuple(a.shape[:-1])
    q = torch.empty(lead + (Nq,), dtype=a.dtype, device=dev)
    k = torch.empty(lead + (Nkv,), dtype=a.dtype, device=dev)
    v = torch.empty(lead + (Nkv,), dtype=a.dtype, device=dev)
    res = torch.empty_like(a) if want_residual else None
    p = _native.QkvProblem_()
    p.dtype = _dtype_code(a.dtype)
    p.M, p.K, p.Nq, p.Nkv, p.block_size, p.bits = a.numel() // K, K, Nq, Nkv, int(block_size), int(bits)
    p.epsilon = float(epsilon)
    p.a, p.skip, p.norm_scale = _ptr(a), _ptr(skip), _ptr(norm_scale)
    p.q_b, p.q_scales, p.k_b, p.k_scales, p.v_b, p.v_scales = (_ptr(q_b), _ptr(q_scales), _ptr(k_b), _ptr(k_scales),
                                                               _ptr(v_b), _ptr(v_scales))
    p.q, p.k, p.v, p.residual = _ptr(q), _ptr(k), _ptr(v), _ptr(res)
    lib = _native.load()
    need = ctypes.c_uint64(0)
    check(lib.xrgpu_qkv_workspace_size(ctypes.byref(p), ctypes.byref(need)))
    _call(lib.xrgpu_qkv_forward, p, _workspace(need.value, dev), dev)
    return (q, k, v, res) if want_residual else (q, k, v)


def matmul_bnb4(a, b, absmax, *, K: int, N: int, block_size: int, quant_type: int = 1):
    """com.microsoft.MatMulBnb4 (transB = 1): NF4 (quant_type 1) or FP4 (0) codebook weights."""
    dev = a.device
    for t, n in ((a, "a"), (b, "b"), (absmax, "absmax")):
        _require(t, n, dev)
    y = torch.empty(tuple(a.shape[:-1]) + (int(N),), dtype=a.dtype, device=dev)
    p = _native.Bnb4Problem_()
    p.dtype = _dtype_code(a.dtype)
    p.quant_type = int(quant_type)
    p.M, p.K, p.N, p.block_size = a.numel() // int(K), int(K), int(N), int(block_size)
    p.a, p.b, p.absmax, p.y = _ptr(a), _ptr(b), _ptr(absmax), _ptr(y)
    _call(_native.load().xrgpu_bnb4_forward, p, False, dev)
    return y


def gather_block_quantized(data, indices, scales, zero_points=None, *, bits: int = 4, block_size: int = 128):
    """com.microsoft.GatherBlockQuantized (gather_axis 0, quantize_axis 1): float32 rows
    (q - z) * scale of the selected rows. Out-of-range indices leave zeros and device error 55."""
    dev = data.device
    for t, n in ((data, "data"), (indices, "indices"), (scales, "scales"), (zero_points, "zero_points")):
        _require(t, n, dev)
    if indices.dtype not in (torch.int64, torch.int32):
        raise ValueError("indices must be int64 or int32")
    width = data.shape[1] * (8 // int(bits))
    out = torch.empty((indices.numel(), width), dtype=torch.float32, device=dev)
    p = _native.GatherProblem_()
    p.bits = int(bits)
    p.index_dtype = _native.INT64 if indices.dtype == torch.int64 else _native.INT32
    p.rows, p.row_bytes, p.count, p.block_size = data.shape[0], data.shape[1], indices.numel(), int(block_size)
    p.data, p.indices, p.scales, p.zero_points, p.out = _ptr(data), _ptr(indices), _ptr(scales), _ptr(zero_points), _ptr(out)
    _call(_native.load().xrgpu_gather_block_quantized_forward, p, False, dev)
    return out


def qmoe(x, router, fc1, fc1_scales, fc2, fc2_scales, *, k: int = 1, bits: int = 4, block_size: int = 0,
         activation="relu", swiglu_fusion: int = 0, activation_alpha: float = 1.0, activation_beta: float = 0.0,
         swiglu_limit: Optional[float] = None):
    """com.microsoft.QMoE (float32): top-k routing, symmetric int4/int8 expert weights, relu or swiglu."""
    dev = x.device
    for t, n in ((x, "x"), (router, "router"), (fc1, "fc1"), (fc1_scales, "fc1_scales"), (fc2, "fc2"),
                 (fc2_scales, "fc2_scales")):
        _require(t, n, dev)
    hidden = int(x.shape[-1])
    out = torch.empty_like(x)
    p = _native.QmoeProblem_()
    p.bits, p.activation, p.swiglu_fusion = int(bits), _act_code(activation), int(swiglu_fusion)
    p.has_swiglu_limit = int(swiglu_limit is not None)
    p.tokens, p.hidden, p.experts, p.k = x.numel() // hidden, hidden, int(router.shape[1]), int(k)
    p.fc1_rows, p.block_size = int(fc1.shape[1]), int(block_size)
    p.activation_alpha, p.activation_beta = float(activation_alpha), float(activation_beta)
    p.swiglu_limit = float(swiglu_limit or 0.0)
    p.input, p.router, p.fc1, p.fc1_scales = _ptr(x), _ptr(router), _ptr(fc1), _ptr(fc1_scales)
    p.fc2, p.fc2_scales, p.output = _ptr(fc2), _ptr(fc2_scales), _ptr(out)
    lib = _native.load()
    need = ctypes.c_uint64(0)
    check(lib.xrgpu_qmoe_workspace_size(ctypes.byref(p), ctypes.byref(need)))
    _call(lib.xrgpu_qmoe_forward, p, _workspace(need.value, dev), dev)
    return out

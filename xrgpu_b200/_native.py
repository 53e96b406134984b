"""ctypes binding of ``libxrgpu_mmnb.so`` (the C ABI in ``include/xrgpu_mmnb.h``).

Loading fails loudly when the library is missing: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "libxrgpu_mmnb.so"

MAX_RANK = 16

# xrgpu_dtype (operators.h:9 order)
FLOAT32, FLOAT16, INT32, UINT32, INT16, INT8, UINT8, INT64, BOOL, UNSPECIFIED = range(10)
# xrgpu_status
OK, INVALID_ARGUMENT, RUNTIME_ERROR, TIMEOUT, DEVICE_ERROR, UNAVAILABLE = range(6)
# xrgpu_mmnb_path
PATH_AUTO, PATH_GENERIC, PATH_GEMV, PATH_GEMM = range(4)

EXPORTED = (
    "xrgpu_last_error", "xrgpu_default_options", "xrgpu_probe", "xrgpu_plan", "xrgpu_prepare", "xrgpu_run",
    "xrgpu_read_outputs", "xrgpu_info", "xrgpu_close", "xrgpu_destroy", "xrgpu_write_input", "xrgpu_run_async",
    "xrgpu_sync", "xrgpu_output_device_ptr", "xrgpu_mmnb_workspace_size", "xrgpu_mmnb_forward",
    "xrgpu_mmnb_dequantize", "xrgpu_mmnb_select_path", "xrgpu_device_error", "xrgpu_version",
    "xrgpu_p2p_create", "xrgpu_p2p_connect", "xrgpu_p2p_allgather", "xrgpu_p2p_destroy",
    "xrgpu_p2p_forward_supported", "xrgpu_p2p_forward_send", "xrgpu_p2p_forward_recv", "xrgpu_p2p_forward_recv_many",
    "xrgpu_stream_capture_id",
    "xrgpu_plan_ex", "xrgpu_prepare_ex", "xrgpu_mlp_workspace_size", "xrgpu_mlp_forward", "xrgpu_mlp_forward_static",
    "xrgpu_qkv_workspace_size",
    "xrgpu_qkv_forward", "xrgpu_bnb4_forward", "xrgpu_gather_block_quantized_forward", "xrgpu_qmoe_workspace_size",
    "xrgpu_qmoe_forward",
)
# xrgpu_activation
ACT_NONE, ACT_RELU, ACT_SILU, ACT_GELU, ACT_TANH, ACT_SIGMOID, ACT_SWIGLU = range(7)
P2P_HANDLE_BYTES = 64
P2P_MAX_WORLD = 16
STATIC_SCRATCH_BYTES = 4 << 20  # XRGPU_STATIC_SCRATCH_BYTES (xrgpu_mlp_forward_static)


class Tensor_(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("shape", ctypes.c_int64 * MAX_RANK), ("data", ctypes.c_void_p), ("nbytes", ctypes.c_uint64)]


class IntAttr_(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("value", ctypes.c_int64)]


class Request_(ctypes.Structure):
    _fields_ = [("operation", ctypes.c_char_p), ("inputs", ctypes.POINTER(Tensor_)), ("num_inputs", ctypes.c_int32),
                ("attrs", ctypes.POINTER(IntAttr_)), ("num_attrs", ctypes.c_int32),
                ("args", ctypes.POINTER(IntAttr_)), ("num_args", ctypes.c_int32)]


class Options_(ctypes.Structure):
    _fields_ = [("profiling", ctypes.c_int32), ("timeout_ns", ctypes.c_uint64),
                ("memory_limit_bytes", ctypes.c_uint64), ("device", ctypes.c_int32)]


class Problem_(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("zero_point_dtype", ctypes.c_int32), ("path", ctypes.c_int32),
                ("reserved", ctypes.c_int32), ("M", ctypes.c_int64), ("K", ctypes.c_int64), ("N", ctypes.c_int64),
                ("block_size", ctypes.c_int64), ("bits", ctypes.c_int64), ("a", ctypes.c_void_p),
                ("b", ctypes.c_void_p), ("scales", ctypes.c_void_p), ("zero_points", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64)]


class FloatAttr_(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("value", ctypes.c_double)]


class StringAttr_(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("value", ctypes.c_char_p)]


class RequestEx_(ctypes.Structure):
    _fields_ = [("operation", ctypes.c_char_p), ("inputs", ctypes.POINTER(Tensor_)), ("num_inputs", ctypes.c_int32),
                ("attrs", ctypes.POINTER(IntAttr_)), ("num_attrs", ctypes.c_int32),
                ("args", ctypes.POINTER(IntAttr_)), ("num_args", ctypes.c_int32),
                ("float_attrs", ctypes.POINTER(FloatAttr_)), ("num_float_attrs", ctypes.c_int32),
                ("string_attrs", ctypes.POINTER(StringAttr_)), ("num_string_attrs", ctypes.c_int32),
                ("requested_outputs", ctypes.POINTER(ctypes.c_char_p)), ("num_requested_outputs", ctypes.c_int32)]


_vp, _i64 = ctypes.c_void_p, ctypes.c_int64


class MlpProblem_(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("activation", ctypes.c_int32), ("M", _i64), ("K", _i64), ("N", _i64),
                ("block_size", _i64), ("bits", _i64), ("epsilon", ctypes.c_float), ("reserved", ctypes.c_int32),
                ("a", _vp), ("skip", _vp), ("norm_scale", _vp), ("gate_b", _vp), ("gate_scales", _vp),
                ("gate_bias", _vp), ("up_b", _vp), ("up_scales", _vp), ("up_bias", _vp), ("y", _vp), ("residual", _vp)]


class QkvProblem_(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32), ("M", _i64), ("K", _i64), ("Nq", _i64),
                ("Nkv", _i64), ("block_size", _i64), ("bits", _i64), ("epsilon", ctypes.c_float),
                ("reserved2", ctypes.c_int32), ("a", _vp), ("skip", _vp), ("norm_scale", _vp), ("q_b", _vp),
                ("q_scales", _vp), ("k_b", _vp), ("k_scales", _vp), ("v_b", _vp), ("v_scales", _vp), ("q", _vp),
                ("k", _vp), ("v", _vp), ("residual", _vp)]


class Bnb4Problem_(ctypes.Structure):
    _fields_ = [("dtype", ctypes.c_int32), ("quant_type", ctypes.c_int32), ("M", _i64), ("K", _i64), ("N", _i64),
                ("block_size", _i64), ("a", _vp), ("b", _vp), ("absmax", _vp), ("y", _vp)]


class GatherProblem_(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int32), ("index_dtype", ctypes.c_int32), ("rows", _i64), ("row_bytes", _i64),
                ("count", _i64), ("block_size", _i64), ("data", _vp), ("indices", _vp), ("scales", _vp),
                ("zero_points", _vp), ("out", _vp)]


class QmoeProblem_(ctypes.Structure):
    _fields_ = [("bits", ctypes.c_int32), ("activation", ctypes.c_int32), ("swiglu_fusion", ctypes.c_int32),
                ("has_swiglu_limit", ctypes.c_int32), ("tokens", _i64), ("hidden", _i64), ("experts", _i64),
                ("k", _i64), ("fc1_rows", _i64), ("block_size", _i64), ("activation_alpha", ctypes.c_float),
                ("activation_beta", ctypes.c_float), ("swiglu_limit", ctypes.c_float), ("reserved", ctypes.c_int32),
                ("input", _vp), ("router", _vp), ("fc1", _vp), ("fc1_scales", _vp), ("fc2", _vp),
                ("fc2_scales", _vp), ("output", _vp)]


_lib = None


def load(path: os.PathLike | None = None):
    """Load (once) and return the CUDA library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    so = Path(path) if path else LIBRARY
    if not so.exists():
        raise RuntimeError(f"xrgpu_b200 CUDA library not built: {so} is missing (run xrgpu_b200.build.build())")
    lib = ctypes.CDLL(str(so))
    P = ctypes.POINTER
    vp, u64, i32 = ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int32
    sig = {
        "xrgpu_last_error": ([], ctypes.c_char_p),
        "xrgpu_version": ([], ctypes.c_char_p),
        "xrgpu_default_options": ([P(Options_)], None),
        "xrgpu_probe": ([ctypes.c_char_p, u64, P(u64)], ctypes.c_int),
        "xrgpu_plan": ([P(Request_), P(Tensor_), i32, P(i32)], ctypes.c_int),
        "xrgpu_prepare": ([ctypes.c_char_p, P(Request_), P(Options_), P(vp)], ctypes.c_int),
        "xrgpu_run": ([vp], ctypes.c_int),
        "xrgpu_read_outputs": ([vp, i32, vp, u64], ctypes.c_int),
        "xrgpu_info": ([vp, ctypes.c_char_p, u64, P(u64)], ctypes.c_int),
        "xrgpu_close": ([vp], ctypes.c_int),
        "xrgpu_destroy": ([vp], None),
        "xrgpu_write_input": ([vp, ctypes.c_char_p, vp, u64], ctypes.c_int),
        "xrgpu_run_async": ([vp, vp], ctypes.c_int),
        "xrgpu_sync": ([vp], ctypes.c_int),
        "xrgpu_output_device_ptr": ([vp, i32, P(vp)], ctypes.c_int),
        "xrgpu_mmnb_workspace_size": ([P(Problem_), P(u64)], ctypes.c_int),
        "xrgpu_mmnb_forward": ([P(Problem_), vp, u64, vp], ctypes.c_int),
        "xrgpu_mmnb_dequantize": ([P(Problem_), vp, vp], ctypes.c_int),
        "xrgpu_mmnb_select_path": ([P(Problem_), ctypes.c_char_p, u64], ctypes.c_int),
        "xrgpu_device_error": ([i32, P(ctypes.c_uint32), i32], ctypes.c_int),
        "xrgpu_p2p_create": ([i32, i32, i32, u64, P(vp), vp], ctypes.c_int),
        "xrgpu_p2p_connect": ([vp, vp], ctypes.c_int),
        "xrgpu_p2p_allgather": ([vp, vp, ctypes.c_int64, ctypes.c_int64, vp, ctypes.c_int64, ctypes.c_int64, vp],
                                ctypes.c_int),
        "xrgpu_p2p_destroy": ([vp], ctypes.c_int),
        "xrgpu_p2p_forward_supported": ([vp, P(Problem_), ctypes.c_int64, P(i32)], ctypes.c_int),
        "xrgpu_p2p_forward_send": ([vp, P(Problem_), ctypes.c_int64, vp, vp], ctypes.c_int),
        "xrgpu_p2p_forward_recv": ([vp, ctypes.c_int64, vp, ctypes.c_int64, vp], ctypes.c_int),
        "xrgpu_p2p_forward_recv_many": ([i32, P(vp), P(ctypes.c_int64), P(vp), P(ctypes.c_int64), vp], ctypes.c_int),
        "xrgpu_stream_capture_id": ([vp, P(u64)], ctypes.c_int),
        "xrgpu_plan_ex": ([P(RequestEx_), P(Tensor_), i32, P(i32)], ctypes.c_int),
        "xrgpu_prepare_ex": ([ctypes.c_char_p, P(RequestEx_), P(Options_), P(vp)], ctypes.c_int),
        "xrgpu_mlp_workspace_size": ([P(MlpProblem_), P(u64)], ctypes.c_int),
        "xrgpu_mlp_forward": ([P(MlpProblem_), vp, u64, vp], ctypes.c_int),
        "xrgpu_mlp_forward_static": ([P(MlpProblem_), vp], ctypes.c_int),
        "xrgpu_qkv_workspace_size": ([P(QkvProblem_), P(u64)], ctypes.c_int),
        "xrgpu_qkv_forward": ([P(QkvProblem_), vp, u64, vp], ctypes.c_int),
        "xrgpu_bnb4_forward": ([P(Bnb4Problem_), vp], ctypes.c_int),
        "xrgpu_gather_block_quantized_forward": ([P(GatherProblem_), vp], ctypes.c_int),
        "xrgpu_qmoe_workspace_size": ([P(QmoeProblem_), P(u64)], ctypes.c_int),
        "xrgpu_qmoe_forward": ([P(QmoeProblem_), vp, u64, vp], ctypes.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = res
    _lib = lib
    return lib


class XrgpuError(RuntimeError):
    """Runtime/timeout/device failure from the CUDA backend (the reference's std::runtime_error)."""

    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int):
    """Raise the Python counterpart of a nonzero xrgpu_status.

    INVALID_ARGUMENT -> ValueError (the reference's std::invalid_argument);
    everything else -> XrgpuError (std::runtime_error).
    """
    if status == OK:
        return
    msg = load().xrgpu_last_error().decode(errors="replace")
    if status == INVALID_ARGUMENT:
        raise ValueError(msg)
    raise XrgpuError(status, msg)

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
)
P2P_HANDLE_BYTES = 64
P2P_MAX_WORLD = 16


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

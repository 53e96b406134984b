"""ctypes wrappers for the compiled CPU checkers (TEST INFRASTRUCTURE ONLY).

``OracleC`` wraps this directory's own C restatement (``mmnb_oracle.c``);
``ReferenceC`` wraps the reference's own GLSL algorithm compiled as C++
(``oracle/_ref/libmmnb_ref.so``, see ``oracle/build.py``). Both take NumPy
arrays and return Y in A's dtype.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build
from .mmnb_oracle import k_blocks

DT_F32, DT_F16, DT_U8, DT_NONE = 0, 1, 6, -1
_c_i64 = ctypes.c_int64
_vp = ctypes.c_void_p


def _dt(arr) -> int:
    if arr is None:
        return DT_NONE
    return {np.dtype(np.float32): DT_F32, np.dtype(np.float16): DT_F16, np.dtype(np.uint8): DT_U8}[arr.dtype]


def _ptr(arr):
    return None if arr is None else arr.ctypes.data_as(_vp)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


class _Matmul:
    prefix = ""

    def _bind(self, lib):
        fn = getattr(lib, self.prefix + "matmul")
        fn.argtypes = [_vp, ctypes.c_int, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, ctypes.c_int, _vp,
                       _c_i64, _c_i64, _vp, _c_i64, _c_i64, ctypes.c_int]
        fn.restype = ctypes.c_int
        self._matmul = fn

    def matmul(self, a, b, scales, zero_points=None, bias=None, *, K, N, bits=4, block_size,
               columns=None, threads=1, out=None):
        a = np.ascontiguousarray(a)
        b = np.ascontiguousarray(b, dtype=np.uint8)
        scales = np.ascontiguousarray(scales, dtype=a.dtype)
        zp = None if zero_points is None else np.ascontiguousarray(zero_points)
        bias = None if bias is None else np.ascontiguousarray(bias, dtype=a.dtype)
        rows = int(np.prod(a.shape[:-1], dtype=np.int64))
        c0, c1 = (0, N) if columns is None else (columns.start or 0, N if columns.stop is None else columns.stop)
        y = out if out is not None else np.zeros(tuple(a.shape[:-1]) + (N,), dtype=a.dtype)
        code = self._matmul(_ptr(a), _dt(a), rows, K, N, _ptr(b), _ptr(scales), _ptr(zp), _dt(zp),
                            _ptr(bias), block_size, bits, _ptr(y), c0, c1, int(threads))
        if code != 0:
            raise RuntimeError(f"{type(self).__name__}.matmul failed with code {code}")
        return y


class OracleC(_Matmul):
    """This repository's serial float32 C restatement (``mmnb_oracle.c``)."""

    prefix = "mmnb_oracle_"

    def __init__(self):
        self.lib = ctypes.CDLL(str(_build.build_oracle()))
        self._bind(self.lib)
        self.lib.mmnb_oracle_dequantize.argtypes = [ctypes.c_int, _c_i64, _c_i64, _vp, _vp, _vp,
                                                    ctypes.c_int, _c_i64, _c_i64, _vp, ctypes.c_int]
        self.lib.mmnb_oracle_dequantize.restype = ctypes.c_int
        self.lib.mmnb_oracle_f32_to_f16_array.argtypes = [_vp, _vp, _c_i64]
        self.lib.mmnb_oracle_f16_to_f32_array.argtypes = [_vp, _vp, _c_i64]

    def dequantize(self, b, scales, zero_points=None, *, K, N, bits=4, block_size, threads=1):
        b = np.ascontiguousarray(b, dtype=np.uint8)
        scales = np.ascontiguousarray(scales)
        zp = None if zero_points is None else np.ascontiguousarray(zero_points)
        w = np.empty((N, K), dtype=np.float32)
        code = self.lib.mmnb_oracle_dequantize(_dt(scales), K, N, _ptr(b), _ptr(scales), _ptr(zp),
                                               _dt(zp), block_size, bits, _ptr(w), int(threads))
        if code:
            raise RuntimeError(f"dequantize failed with code {code}")
        return w

    def f32_to_f16_bits(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.shape, dtype=np.uint16)
        self.lib.mmnb_oracle_f32_to_f16_array(_ptr(x), _ptr(out), x.size)
        return out

    def f16_bits_to_f32(self, h):
        h = np.ascontiguousarray(h, dtype=np.uint16)
        out = np.empty(h.shape, dtype=np.float32)
        self.lib.mmnb_oracle_f16_to_f32_array(_ptr(h), _ptr(out), h.size)
        return out


class ReferenceC(_Matmul):
    """The reference's own ``packedMatmul``/``nbitWeight`` compiled as C++.

    Float zero points only (the reference contract): packed uint8 zero points
    are an extension the reference does not accept.
    """

    prefix = "mmnb_ref_"

    def __init__(self):
        path = _build.build_reference()
        if path is None or not path.exists():
            raise FileNotFoundError("oracle/_ref/libmmnb_ref.so is not built (needs the reference checkout)")
        self.lib = ctypes.CDLL(str(path))
        self._bind(self.lib)
        self.lib.mmnb_ref_half_to_float_bits.argtypes = [ctypes.c_uint32]
        self.lib.mmnb_ref_half_to_float_bits.restype = ctypes.c_uint32
        self.lib.mmnb_ref_float_bits_to_half.argtypes = [ctypes.c_uint32]
        self.lib.mmnb_ref_float_bits_to_half.restype = ctypes.c_uint32

    def matmul(self, a, b, scales, zero_points=None, bias=None, **kw):
        if zero_points is not None and np.asarray(zero_points).dtype == np.uint8:
            raise ValueError("the reference contract takes float zero points only")
        return super().matmul(a, b, scales, zero_points, bias, **kw)


def reference_available() -> bool:
    return _build.REF_SO.exists() or (_build.DEFAULT_REFERENCE / "kernels").exists()


__all__ = ["OracleC", "ReferenceC", "host_threads", "reference_available", "k_blocks"]

"""Python mirror of the reference's standalone operator API, backed by the CUDA library.

Names, argument meaning and error behaviour follow ``xrgpu::operators`` /
``xrgpu::operators::extended`` (runtime/include/xrgpu/operators.h:9-55,
runtime/include/xrgpu/extended_operators.h:8-61):

* ``plan(request)`` validates and infers outputs without touching tensor bytes;
* ``Operator.prepare(package_directory, request, options)`` copies the inputs to the
  device (the handle owns that snapshot), ``run()`` executes synchronously within
  ``options.timeout_ns``, ``read_outputs()`` returns owned host tensors, ``info()``
  returns JSON and ``close()`` releases the device memory;
* contract and planning errors raise ``ValueError`` (the reference's
  ``std::invalid_argument``); execution failures raise ``XrgpuError``, a
  ``RuntimeError`` (``std::runtime_error``); a failed run poisons the operator
  until ``close()`` (kernels/_shared/extended/vulkan.cpp:105,115).

Operations served: ``com.microsoft.MatMulNBits`` and the operators around it --
``com.microsoft.MatMulNBitsMlp``, ``MatMulNBitsQkv`` (its fused callers), ``MatMulBnb4``,
``GatherBlockQuantized`` and ``QMoE`` (the same quantized-weight formats). Their attributes may be
integers, numbers or strings, and optional outputs (``residualT``) are produced when requested,
as in ``complex_plan.cpp:54-57``.
"""
from __future__ import annotations

import ctypes
import enum
import json
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from . import _native
from ._native import check

OPERATION = "com.microsoft.MatMulNBits"


class DType(enum.IntEnum):
    """Logical dtypes in the order of operators.h:9."""

    Float32 = 0
    Float16 = 1
    Int32 = 2
    UInt32 = 3
    Int16 = 4
    Int8 = 5
    UInt8 = 6
    Int64 = 7
    Bool = 8
    Unspecified = 9


_NUMPY = {DType.Float32: np.float32, DType.Float16: np.float16, DType.Int32: np.int32, DType.UInt32: np.uint32,
          DType.Int16: np.int16, DType.Int8: np.int8, DType.UInt8: np.uint8, DType.Int64: np.int64,
          DType.Bool: np.bool_}


def dtype_from_numpy(dt) -> DType:
    dt = np.dtype(dt)
    for k, v in _NUMPY.items():
        if np.dtype(v) == dt:
            return k
    raise ValueError(f"unsupported numpy dtype {dt}")


@dataclass
class Tensor:
    """Owned little-endian contiguous bytes with a logical dtype and shape (operators.h:16-23)."""

    name: str = ""
    shape: List[int] = field(default_factory=list)
    dtype: DType = DType.Float32
    storage_dtype: DType = DType.Unspecified
    layout: str = "contiguous"
    data: bytes = b""

    @classmethod
    def from_numpy(cls, name: str, array, dtype: Optional[DType] = None) -> "Tensor":
        arr = np.ascontiguousarray(array)
        logical = dtype if dtype is not None else dtype_from_numpy(arr.dtype)
        if np.dtype(_NUMPY[logical]) != arr.dtype:
            arr = arr.astype(_NUMPY[logical])
        return cls(name=name, shape=list(arr.shape), dtype=logical, data=arr.astype(arr.dtype.newbyteorder("<")).tobytes())

    def numpy(self) -> np.ndarray:
        return np.frombuffer(self.data, dtype=np.dtype(_NUMPY[DType(self.dtype)]).newbyteorder("<")).reshape(self.shape)


@dataclass
class Options:
    """operators.h:24-28 plus the CUDA device ordinal."""

    profiling: bool = False
    timeout_ns: int = 15_000_000_000
    memory_limit_bytes: int = 268_435_456
    device: int = 0


@dataclass
class Attributes:
    """extended_operators.h:8-16 (MatMulNBits uses integer attributes only)."""

    integers: Dict[str, int] = field(default_factory=dict)
    numbers: Dict[str, float] = field(default_factory=dict)
    strings: Dict[str, str] = field(default_factory=dict)


@dataclass
class Request:
    """extended_operators.h:22-28."""

    operation: str = OPERATION
    inputs: List[Tensor] = field(default_factory=list)
    attrs: Attributes = field(default_factory=Attributes)
    args: Attributes = field(default_factory=Attributes)
    requested_outputs: List[Tensor] = field(default_factory=list)


def _int_attrs(attrs: Attributes, operation: str):
    """Integer attributes; for MatMulNBits (integer attributes only) integral numbers count too."""
    items = []
    for k, v in attrs.integers.items():
        items.append((k, int(v)))
    if operation == OPERATION:
        for k, v in attrs.numbers.items():
            if float(v) != int(v):
                raise ValueError(f"Integer attribute required: {k}")
            items.append((k, int(v)))
        if attrs.strings:
            raise ValueError("Unknown string attribute for MatMulNBits: " + ", ".join(attrs.strings))
    arr = (_native.IntAttr_ * max(1, len(items)))()
    for i, (k, v) in enumerate(items):
        arr[i].name = k.encode()
        arr[i].value = v
    return arr, len(items)


def _other_attrs(attrs: Attributes, args: Attributes, operation: str, keep: list):
    """Number and string attributes of the operators around MatMulNBits (args override attrs)."""
    if operation == OPERATION:
        return (_native.FloatAttr_ * 1)(), 0, (_native.StringAttr_ * 1)(), 0
    numbers = {**attrs.numbers, **args.numbers}
    strings = {**attrs.strings, **args.strings}
    farr = (_native.FloatAttr_ * max(1, len(numbers)))()
    for i, (k, v) in enumerate(numbers.items()):
        name = k.encode()
        keep.append(name)
        farr[i].name = name
        farr[i].value = float(v)
    sarr = (_native.StringAttr_ * max(1, len(strings)))()
    for i, (k, v) in enumerate(strings.items()):
        name, value = k.encode(), str(v).encode()
        keep += [name, value]
        sarr[i].name = name
        sarr[i].value = value
    return farr, len(numbers), sarr, len(strings)


class _CRequest:
    """Keeps the ctypes view of a Request (and its buffers) alive during a call."""

    def __init__(self, request: Request, with_data: bool):
        self.keep = []
        n = len(request.inputs)
        self.tensors = (_native.Tensor_ * max(1, n))()
        for i, t in enumerate(request.inputs):
            if len(t.shape) > _native.MAX_RANK:
                raise ValueError("Extended tensor rank exceeds 16")
            if t.layout != "contiguous":
                raise ValueError("Extended kernels require contiguous row-major tensors")
            if t.storage_dtype not in (DType.Unspecified, t.dtype):
                raise ValueError("the CUDA backend requires storage_dtype == dtype")
            ct = self.tensors[i]
            name = t.name.encode()
            self.keep.append(name)
            ct.name = name
            ct.dtype = int(t.dtype)
            ct.rank = len(t.shape)
            for j, d in enumerate(t.shape):
                ct.shape[j] = int(d)
            if with_data:
                buf = t.data if isinstance(t.data, (bytes, bytearray)) else bytes(t.data)
                cbuf = ctypes.create_string_buffer(buf, len(buf)) if buf else None
                self.keep.append(cbuf)
                ct.data = ctypes.cast(cbuf, ctypes.c_void_p) if cbuf is not None else None
                ct.nbytes = len(buf)
        self.attrs, na = _int_attrs(request.attrs, request.operation)
        self.args, nr = _int_attrs(request.args, request.operation)
        self.floats, nf, self.strings, ns = _other_attrs(request.attrs, request.args, request.operation, self.keep)
        names = [t.name.encode() for t in request.requested_outputs]
        self.keep += names
        self.requested = (ctypes.c_char_p * max(1, len(names)))(*names)
        op = request.operation.encode()
        self.keep.append(op)
        self.req = _native.RequestEx_(op, self.tensors, n, self.attrs, na, self.args, nr, self.floats, nf,
                                      self.strings, ns, self.requested, len(names))


def _check_requested(request: Request, planned: List[Tensor]):
    if not request.requested_outputs:
        return
    if len(request.requested_outputs) != len(planned):
        raise ValueError("Requested output count differs from plan")
    for want, got in zip(request.requested_outputs, planned):
        if want.name != got.name or DType(want.dtype) != got.dtype:
            raise ValueError("Requested output name/type differs from plan")
        if list(want.shape) != list(got.shape):
            raise ValueError("Requested output shape differs from plan")


def plan(request: Request) -> List[Tensor]:
    """Metadata-only validation and output inference (extended_operators.h:48)."""
    lib = _native.load()
    c = _CRequest(request, with_data=False)
    out = (_native.Tensor_ * 8)()
    count = ctypes.c_int32(0)
    check(lib.xrgpu_plan_ex(ctypes.byref(c.req), out, 8, ctypes.byref(count)))
    planned = [Tensor(name=y.name.decode(), shape=[int(y.shape[i]) for i in range(y.rank)], dtype=DType(y.dtype))
               for y in out[:count.value]]
    _check_requested(request, planned)
    return planned


def probe() -> str:
    """JSON availability report (operators.h:34); never implies CPU compute."""
    lib = _native.load()
    need = ctypes.c_uint64(0)
    lib.xrgpu_probe(None, 0, ctypes.byref(need))
    buf = ctypes.create_string_buffer(int(need.value) + 1)
    lib.xrgpu_probe(buf, len(buf), None)
    return buf.value.decode()


class Operator:
    """A prepared MatMulNBits call on one CUDA device (extended_operators.h:49-61)."""

    def __init__(self, handle, planned: List[Tensor]):
        self._h = handle
        self._planned = planned
        self._lib = _native.load()

    @classmethod
    def prepare(cls, package_directory: Optional[str], request: Request, options: Optional[Options] = None) -> "Operator":
        lib = _native.load()
        planned = plan(request)
        options = options or Options()
        c = _CRequest(request, with_data=True)
        opts = _native.Options_(int(bool(options.profiling)), int(options.timeout_ns), int(options.memory_limit_bytes),
                                int(options.device))
        handle = ctypes.c_void_p()
        pkg = package_directory.encode() if package_directory else None
        check(lib.xrgpu_prepare_ex(pkg, ctypes.byref(c.req), ctypes.byref(opts), ctypes.byref(handle)))
        return cls(handle, planned)

    def _handle(self):
        if self._h is None:
            raise RuntimeError("Operator handle destroyed")
        return self._h

    def run(self) -> None:
        check(self._lib.xrgpu_run(self._handle()))

    def run_async(self, stream: int = 0) -> None:
        """Enqueue without waiting on a cudaStream_t (extension)."""
        check(self._lib.xrgpu_run_async(self._handle(), ctypes.c_void_p(stream or None)))

    def sync(self) -> None:
        check(self._lib.xrgpu_sync(self._handle()))

    def write_input(self, name: str, data) -> None:
        """Replace one prepared input's bytes (same size) without re-preparing (extension)."""
        buf = data if isinstance(data, (bytes, bytearray)) else np.ascontiguousarray(data).tobytes()
        cbuf = ctypes.create_string_buffer(bytes(buf), len(buf))
        check(self._lib.xrgpu_write_input(self._handle(), name.encode(), ctypes.cast(cbuf, ctypes.c_void_p), len(buf)))

    def write_input_ptr(self, name: str, host_ptr: int, nbytes: int) -> None:
        """Like write_input, from a raw (e.g. pinned) host pointer."""
        check(self._lib.xrgpu_write_input(self._handle(), name.encode(), ctypes.c_void_p(host_ptr), int(nbytes)))

    def read_outputs(self) -> List[Tensor]:
        outs = []
        for i, t in enumerate(self._planned):
            n = int(np.prod(t.shape, dtype=np.int64)) * np.dtype(_NUMPY[t.dtype]).itemsize
            buf = ctypes.create_string_buffer(max(1, n))
            check(self._lib.xrgpu_read_outputs(self._handle(), i, buf, n))
            outs.append(Tensor(name=t.name, shape=list(t.shape), dtype=t.dtype, data=buf.raw[:n]))
        return outs

    def read_output_into(self, index: int, host_ptr: int, nbytes: int) -> None:
        """Copy output `index` into a raw (e.g. pinned) host buffer."""
        check(self._lib.xrgpu_read_outputs(self._handle(), index, ctypes.c_void_p(host_ptr), int(nbytes)))

    def output_device_ptr(self, index: int = 0) -> int:
        ptr = ctypes.c_void_p()
        check(self._lib.xrgpu_output_device_ptr(self._handle(), index, ctypes.byref(ptr)))
        return int(ptr.value or 0)

    def info(self) -> str:
        need = ctypes.c_uint64(0)
        check(self._lib.xrgpu_info(self._handle(), None, 0, ctypes.byref(need)))
        buf = ctypes.create_string_buffer(int(need.value) + 1)
        check(self._lib.xrgpu_info(self._handle(), buf, len(buf), None))
        return buf.value.decode()

    def info_dict(self) -> dict:
        return json.loads(self.info())

    def close(self) -> None:
        if self._h is not None:
            check(self._lib.xrgpu_close(self._h))

    def __del__(self):
        try:
            if self._h is not None:
                self._lib.xrgpu_destroy(self._h)
                self._h = None
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

"""B200-native (sm_100a) backend for xrGPU's com.microsoft.MatMulNBits operator.

Public surface:
  * ``xrgpu_b200.operators`` -- the reference's operator API (plan / Operator.prepare / run /
    read_outputs / info / close) over host tensors;
  * ``xrgpu_b200.functional`` -- zero-copy torch entry points (``matmul_nbits``, ``dequantize``);
  * ``xrgpu_b200.sharded`` -- N-column sharding across GPUs with one all-gather of Y;
  * ``xrgpu_b200.catalog`` -- the operator descriptor/registration for the ``cuda`` backend.
The kernels live in ``libxrgpu_mmnb.so`` (C ABI: include/xrgpu_mmnb.h).
"""
from . import _native  # noqa: F401
from .operators import (OPERATION, Attributes, DType, Operator, Options, Request, Tensor, plan,  # noqa: F401
                        probe)

__all__ = ["OPERATION", "Attributes", "DType", "Operator", "Options", "Request", "Tensor", "plan", "probe"]

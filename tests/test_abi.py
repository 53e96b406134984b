"""Host-only checks of the C ABI: the library builds, loads, exports every declared entry point,
and its planner validates requests like the reference (no GPU needed: planning reads no CUDA state).
"""
import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def declared_functions():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = header.read_text()
        names |= set(re.findall(r"XRGPU_API[^;(]*?\b(xrgpu_\w+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported(cuda_lib):
    declared = declared_functions()
    assert len(declared) >= 20
    for name in sorted(declared):
        assert hasattr(cuda_lib, name), name


def test_binding_covers_header(cuda_lib):
    from xrgpu_b200 import _native
    assert set(_native.EXPORTED) <= declared_functions()


def test_version_and_options(cuda_lib):
    from xrgpu_b200 import _native
    assert b"sm_100a" in cuda_lib.xrgpu_version()
    o = _native.Options_()
    cuda_lib.xrgpu_default_options(ctypes.byref(o))
    assert (o.profiling, o.timeout_ns, o.memory_limit_bytes, o.device) == (0, 15_000_000_000, 268_435_456, 0)


def _request(a_shape=(2, 64), N=8, K=None, bs=32, bits=4, a_dt=None, extra=None, drop=(), zp=None, bias=True, **attrs):
    from xrgpu_b200.operators import Attributes, DType, Request, Tensor
    K = a_shape[-1] if K is None else K
    kb = -(-K // bs)
    blob = (bs * bits + 7) // 8
    a_dt = DType.Float16 if a_dt is None else a_dt
    t = [Tensor("aT", list(a_shape), a_dt), Tensor("bT", [N, kb, blob], DType.UInt8), Tensor("scalesT", [N, kb], a_dt)]
    if zp == "packed":
        t.append(Tensor("zeroPointsT", [N, (kb * bits + 7) // 8], DType.UInt8))
    elif zp is not None:
        t.append(Tensor("zeroPointsT", [N, kb], zp))
    if bias:
        t.append(Tensor("biasT", [N], a_dt))
    t = [x for x in t if x.name not in drop] + list(extra or [])
    ints = {"K": K, "N": N, "block_size": bs, "bits": bits}
    ints.update(attrs)
    ints = {k: v for k, v in ints.items() if v is not None}
    return Request(inputs=t, attrs=Attributes(integers=ints))


def test_plan_infers_output(cuda_lib):
    from xrgpu_b200.operators import DType, plan
    (y,) = plan(_request((2, 3, 64), N=8))
    assert y.name == "yT" and y.shape == [2, 3, 8] and y.dtype == DType.Float16
    (y,) = plan(_request((5, 64), N=3, a_dt=DType.Float32, zp=DType.Float32))
    assert y.shape == [5, 3] and y.dtype == DType.Float32
    (y,) = plan(_request((0, 32), N=4, bias=False))  # empty rows (upstream empty_zero_dim)
    assert y.shape == [0, 4]
    (y,) = plan(_request((1, 64), N=8, zp="packed"))
    assert y.shape == [1, 8]


def test_plan_defaults_follow_reference(cuda_lib):
    from xrgpu_b200.operators import plan
    # K defaults to A's last dim, block_size to 32, bits to 4 (complex_plan.cpp:118).
    r = _request((1, 64), N=8)
    for key in ("K", "block_size", "bits"):
        r.attrs.integers.pop(key)
    (y,) = plan(r)
    assert y.shape == [1, 8]
    r.inputs[1].shape = [8, 1, 32]  # block_size 64 does not match the default of 32
    r.inputs[2].shape = [8, 1]
    with pytest.raises(ValueError, match="bT shape"):
        plan(r)


def test_args_override_attrs(cuda_lib):
    from xrgpu_b200.operators import Attributes, plan
    r = _request((1, 64), N=8)
    r.attrs.integers["N"] = 99
    r.args = Attributes(integers={"N": 8})
    assert plan(r)[0].shape == [1, 8]


@pytest.mark.parametrize("mutate,message", [
    (lambda r: setattr(r, "operation", "com.microsoft.Nope"), "Unsupported extended operator"),
    (lambda r: r.inputs.pop(1), "Missing required frozen-contract input: bT"),
    (lambda r: r.inputs.append(r.inputs[0]), "Duplicate"),
    (lambda r: setattr(r.inputs[1], "name", "weights"), "Unknown input outside frozen contract"),
    (lambda r: setattr(r.inputs[2], "dtype", 0), "Type variable differs"),
    (lambda r: setattr(r.inputs[1], "dtype", 5), "Logical dtype outside frozen contract: bT"),
    (lambda r: setattr(r.inputs[0], "dtype", 2), "Logical dtype outside frozen contract: aT"),
    (lambda r: setattr(r.inputs[1], "shape", [8, 2]), "Rank outside frozen contract: bT"),
    (lambda r: setattr(r.inputs[1], "shape", [8, 2, 15]), "bT shape"),
    (lambda r: setattr(r.inputs[2], "shape", [8, 3]), "scalesT shape"),
    (lambda r: r.attrs.integers.pop("N"), "Packed matmul N required"),
    (lambda r: r.attrs.integers.update(bits=3), "bits must be 2, 4 or 8"),
    (lambda r: r.attrs.integers.update(block_size=24), "power of two"),
    (lambda r: r.attrs.integers.update(block_size=8), "power of two"),
    (lambda r: r.attrs.integers.update(accuracy_level=5), "accuracy_level"),
    (lambda r: r.attrs.integers.update(K=32), "last dimension"),
    (lambda r: setattr(r.inputs[3], "shape", [9]), "biasT shape"),
])
def test_plan_rejects_contract_violations(cuda_lib, mutate, message):
    from xrgpu_b200.operators import plan
    r = _request((2, 64), N=8)
    mutate(r)
    with pytest.raises(ValueError, match=message):
        plan(r)


def test_probe_reports_json(cuda_lib):
    from xrgpu_b200.operators import probe
    info = json.loads(probe())
    assert info["backend"] == "cuda" and info["cpu_compute_fallback"] is False
    assert isinstance(info["available"], bool)


def test_prepare_without_gpu_is_unavailable_not_cpu(cuda_lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from xrgpu_b200._native import XrgpuError
    from xrgpu_b200.operators import Operator, Tensor
    r = _request((1, 64), N=8, bias=False)
    r.inputs = [Tensor.from_numpy(t.name, np.zeros(t.shape, dtype={1: np.float16, 6: np.uint8}[int(t.dtype)]))
                for t in r.inputs]
    with pytest.raises(XrgpuError):
        Operator.prepare(None, r)


def test_product_never_imports_oracle():
    pkg = ROOT / "xrgpu_b200"
    for f in list(pkg.rglob("*.py")) + list(pkg.rglob("*.cu")) + list(pkg.rglob("*.h")):
        text = f.read_text()
        assert "oracle" not in re.sub(r"#.*|//.*", "", text).replace("oracle/", ""), f

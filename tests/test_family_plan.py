"""Planning of the operators around MatMulNBits through the C ABI (xrgpu_plan_ex; no GPU needed).

Mirrors the reference's plan_complex branches (kernels/_shared/extended/complex_plan.cpp:117-129)
and validate_contract (contracts.cpp:14-20): output shapes/dtypes, optional outputs only when
requested, requested order, and the reference's error messages for bad requests.
"""
import numpy as np
import pytest

from xrgpu_b200.operators import Attributes, DType, Request, Tensor, plan


def T(name, shape, dtype):
    return Tensor(name=name, shape=list(shape), dtype=dtype)


def mlp_inputs(M=2, K=64, N=8, bs=32, dt=DType.Float16, norm=True, skip=True, bias=True):
    kb = K // bs
    ins = [T("aT", (M, K), dt), T("gateBT", (N, kb, bs // 2), DType.UInt8), T("gateScalesT", (N, kb), dt),
           T("upBT", (N, kb, bs // 2), DType.UInt8), T("upScalesT", (N, kb), dt)]
    if norm:
        ins.append(T("normScaleT", (K,), dt))
    if skip:
        ins.append(T("skipT", (M, K), dt))
    if bias:
        ins += [T("gateBiasT", (N,), dt), T("upBiasT", (N,), dt)]
    return ins


def test_mlp_plan_and_requested_residual(cuda_lib):
    r = Request("com.microsoft.MatMulNBitsMlp", mlp_inputs(), Attributes(integers={"K": 64, "N": 8, "block_size": 32},
                                                                         strings={"activation": "silu"}))
    out = plan(r)
    assert [(t.name, t.shape, t.dtype) for t in out] == [("yT", [2, 8], DType.Float16)]
    r.requested_outputs = [T("residualT", (2, 64), DType.Float16), T("yT", (2, 8), DType.Float16)]
    out = plan(r)
    assert [t.name for t in out] == ["residualT", "yT"]


def test_qkv_plan_shapes(cuda_lib):
    K, Nq, Nkv, bs = 64, 32, 16, 32
    ins = [T("aT", (1, 3, K), DType.Float32), T("normScaleT", (K,), DType.Float32)]
    for p, n in (("q", Nq), ("k", Nkv), ("v", Nkv)):
        ins += [T(f"{p}BT", (n, K // bs, bs // 2), DType.UInt8), T(f"{p}ScalesT", (n, K // bs), DType.Float32)]
    out = plan(Request("com.microsoft.MatMulNBitsQkv", ins, Attributes(integers={"K": K, "Nq": Nq, "Nkv": Nkv,
                                                                                 "block_size": bs})))
    assert [(t.name, t.shape) for t in out] == [("qT", [1, 3, Nq]), ("kT", [1, 3, Nkv]), ("vT", [1, 3, Nkv])]


def test_qkv_requires_norm_scale(cuda_lib):
    ins = [T("aT", (1, 32), DType.Float32), T("qBT", (4, 1, 16), DType.UInt8), T("qScalesT", (4, 1), DType.Float32),
           T("kBT", (4, 1, 16), DType.UInt8), T("kScalesT", (4, 1), DType.Float32),
           T("vBT", (4, 1, 16), DType.UInt8), T("vScalesT", (4, 1), DType.Float32)]
    with pytest.raises(ValueError, match="Missing required frozen-contract input: normScaleT"):
        plan(Request("com.microsoft.MatMulNBitsQkv", ins, Attributes(integers={"K": 32, "Nq": 4, "Nkv": 4})))


def test_bnb4_plan(cuda_lib):
    ins = [T("aT", (3, 64), DType.Float16), T("bT", (64 * 10 // 2,), DType.UInt8), T("absmaxT", (10,), DType.Float16)]
    out = plan(Request("com.microsoft.MatMulBnb4", ins, Attributes(integers={"K": 64, "N": 10, "block_size": 64,
                                                                             "quant_type": 0})))
    assert [(t.name, t.shape, t.dtype) for t in out] == [("yT", [3, 10], DType.Float16)]
    with pytest.raises(ValueError, match="quant_type"):
        plan(Request("com.microsoft.MatMulBnb4", ins, Attributes(integers={"K": 64, "N": 10, "block_size": 64,
                                                                           "quant_type": 2})))


def test_gather_plan_and_geometry_checks(cuda_lib):
    ins = [T("dataT", (6, 9), DType.UInt8), T("indicesT", (3,), DType.Int64), T("scalesT", (6, 2), DType.Float32),
           T("zeroPointsT", (6, 1), DType.UInt8)]
    out = plan(Request("com.microsoft.GatherBlockQuantized", ins, Attributes(integers={"bits": 4, "block_size": 16})))
    assert [(t.name, t.shape, t.dtype) for t in out] == [("outputT", [3, 18], DType.Float32)]
    with pytest.raises(ValueError, match="Unsupported GatherBlockQuantized geometry"):
        plan(Request("com.microsoft.GatherBlockQuantized", ins, Attributes(integers={"bits": 2, "block_size": 16})))
    bad = [T("dataT", (6, 9), DType.UInt8), T("indicesT", (3,), DType.Int32), T("scalesT", (6, 2), DType.Float32)]
    with pytest.raises(ValueError, match="Logical dtype outside frozen contract: indicesT"):
        plan(Request("com.microsoft.GatherBlockQuantized", bad, Attributes(integers={"bits": 4, "block_size": 16})))


def qmoe_inputs(tokens=3, hidden=32, experts=4, inter=16, bits=4, bs=0, swiglu=False):
    rows = 2 * inter if swiglu else inter
    per = 8 // bits
    s1 = (experts, rows) if not bs else (experts, rows, hidden // bs)
    s2 = (experts, hidden) if not bs else (experts, hidden, inter // bs)
    return [T("inputT", (tokens, hidden), DType.Float32), T("routerT", (tokens, experts), DType.Float32),
            T("fc1T", (experts, rows, hidden // per), DType.UInt8), T("fc1ScalesT", s1, DType.Float32),
            T("fc2T", (experts, hidden, inter // per), DType.UInt8), T("fc2ScalesT", s2, DType.Float32)]


def test_qmoe_plan_and_checks(cuda_lib):
    out = plan(Request("com.microsoft.QMoE", qmoe_inputs(), Attributes(integers={"k": 2})))
    assert [(t.name, t.shape) for t in out] == [("outputT", [3, 32])]
    sw = Request("com.microsoft.QMoE", qmoe_inputs(swiglu=True, bs=16),
                 Attributes(integers={"k": 2, "swiglu_fusion": 1, "block_size": 16},
                            strings={"activation_type": "swiglu"}, numbers={"swiglu_limit": 7.0}))
    assert plan(sw)[0].shape == [3, 32]
    with pytest.raises(ValueError, match="Invalid MoE input or routing geometry"):
        plan(Request("com.microsoft.QMoE", qmoe_inputs(), Attributes(integers={"k": 5})))
    with pytest.raises(ValueError, match="Invalid quantized SwiGLU fusion"):
        plan(Request("com.microsoft.QMoE", qmoe_inputs(), Attributes(integers={"k": 1},
                                                                     strings={"activation_type": "swiglu"})))
    with pytest.raises(ValueError, match="Unsupported QMoE integer layout"):
        plan(Request("com.microsoft.QMoE", qmoe_inputs(), Attributes(strings={"quant_type": "fp"})))


def test_unknown_input_and_activation_rejected(cuda_lib):
    ins = mlp_inputs() + [T("zeroPointsT", (8, 1), DType.UInt8)]
    with pytest.raises(ValueError, match="Unknown input outside frozen contract: zeroPointsT"):
        plan(Request("com.microsoft.MatMulNBitsMlp", ins, Attributes(integers={"K": 64, "N": 8})))
    with pytest.raises(ValueError, match="Unknown fused activation: mish"):
        plan(Request("com.microsoft.MatMulNBitsMlp", mlp_inputs(),
                     Attributes(integers={"K": 64, "N": 8}, strings={"activation": "mish"})))

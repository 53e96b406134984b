"""The family oracle (oracle/family_oracle.py) against the reference's known-answer vectors.

tests/golden/family_cases.* hold the reference test module's own cases for MatMulNBitsMlp,
MatMulNBitsQkv, MatMulBnb4, GatherBlockQuantized and QMoE (published upstream outputs and the
reference's independent hand-built cases; see tests/golden/make_family_golden.py). Each output is
compared with the case's own tolerance: |got - expected| <= atol + rtol * |expected|.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import family_oracle as FO

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "family_cases.json").read_text())
ARRAYS = np.load(GOLDEN / "family_cases.npz")


def case_arrays(entry):
    i = entry["index"]
    ins = {d["name"]: ARRAYS[f"{i}/in/{d['name']}"] for d in entry["inputs"]}
    outs = {d["name"]: ARRAYS[f"{i}/out/{d['name']}"] for d in entry["outputs"]}
    return ins, outs


def run_oracle(entry, ins):
    op, at = entry["operation"], {**entry["attrs"], **entry["args"]}
    g = ins.get
    if op == "com.microsoft.MatMulNBitsMlp":
        y, res = FO.matmul_nbits_mlp(g("aT"), g("skipT"), g("normScaleT"), g("gateBT"), g("gateScalesT"), g("gateBiasT"),
                                     g("upBT"), g("upScalesT"), g("upBiasT"), K=at["K"], N=at["N"],
                                     bits=at.get("bits", 4), block_size=at["block_size"],
                                     activation=at.get("activation", "silu"), epsilon=at.get("epsilon", 1e-5))
        return {"yT": y, "residualT": res}
    if op == "com.microsoft.MatMulNBitsQkv":
        q, k, v, res = FO.matmul_nbits_qkv(g("aT"), g("skipT"), g("normScaleT"), g("qBT"), g("qScalesT"), g("kBT"),
                                           g("kScalesT"), g("vBT"), g("vScalesT"), K=at["K"], Nq=at["Nq"],
                                           Nkv=at["Nkv"], bits=at.get("bits", 4), block_size=at["block_size"],
                                           epsilon=at.get("epsilon", 1e-6))
        return {"qT": q, "kT": k, "vT": v, "residualT": res}
    if op == "com.microsoft.MatMulBnb4":
        return {"yT": FO.matmul_bnb4(g("aT"), g("bT"), g("absmaxT"), K=at["K"], N=at["N"], block_size=at["block_size"],
                                     quant_type=at["quant_type"], transB=at.get("transB", 1))}
    if op == "com.microsoft.GatherBlockQuantized":
        out, _ = FO.gather_block_quantized(g("dataT"), g("indicesT"), g("scalesT"), g("zeroPointsT"),
                                           bits=at.get("bits", 4), block_size=at.get("block_size", 128))
        return {"outputT": out}
    if op == "com.microsoft.QMoE":
        return {"outputT": FO.qmoe(g("inputT"), g("routerT"), g("fc1T"), g("fc1ScalesT"), g("fc2T"), g("fc2ScalesT"),
                                   k=at.get("k", 1), bits=at.get("expert_weight_bits", 4),
                                   block_size=at.get("block_size", 0), activation=at.get("activation_type", "relu"),
                                   swiglu_fusion=at.get("swiglu_fusion", 0),
                                   activation_alpha=at.get("activation_alpha", 1.0),
                                   activation_beta=at.get("activation_beta", 0.0),
                                   swiglu_limit=at.get("swiglu_limit"))}
    raise AssertionError(op)


def close(got, exp, tol):
    got = np.asarray(got, np.float64)
    exp = np.asarray(exp, np.float64)
    atol, rtol = (tol or {}).get("atol", 0.0), (tol or {}).get("rtol", 0.0)
    return got.shape == exp.shape and bool(np.all(np.abs(got - exp) <= atol + rtol * np.abs(exp)))


@pytest.mark.parametrize("entry", META, ids=lambda e: e["operation"].split(".")[-1] + ":" + e["name"])
def test_family_oracle_matches_reference_known_answers(entry):
    ins, outs = case_arrays(entry)
    got = run_oracle(entry, ins)
    for d in entry["outputs"]:
        assert close(got[d["name"]], outs[d["name"]], d["tolerance"]), (d["name"], got[d["name"]], outs[d["name"]])


def test_bnb4_codebooks_are_the_reference_tables():
    assert FO.NF4[7] == 0.0 and FO.NF4[0] == -1.0 and FO.NF4[15] == 1.0
    assert FO.FP4[3] == 1.0 and FO.FP4[11] == -1.0 and np.signbit(FO.FP4[8])


def test_gather_out_of_range_index_fails_and_leaves_row_zero():
    data = np.arange(8, dtype=np.uint8).reshape(2, 4)
    scales = np.ones((2, 1), np.float32)
    out, failed = FO.gather_block_quantized(data, np.array([1, 5, -1]), scales, bits=4, block_size=16)
    assert failed and np.all(out[1] == 0) and np.all(out[2] == 0) and np.any(out[0] != 0)

"""Loader for the committed MatMulNBits golden fixtures.

``upstream_cases.json`` holds every case of the reference's frozen MatMulNBits suite
(kernels/_provenance/upstream/com.microsoft.MatMulNBits/build/webgpu/test.json) as a
generator spec; ``upstream_outputs.npz`` holds the expected Y of each case, computed by the
reference's own algorithm (GLSL ``packedMatmul``/``nbitWeight`` compiled as C++, see
oracle/build.py) -- plus, where the suite publishes one, its explicit expected output.

Inputs are regenerated here from the specs. The suite's generators ``values``, ``constant``,
``cycle`` and ``linspace`` are materialised with the semantics of the reference harness
(kernels/_shared/verify_upstream.py:90-122). Its ``fillFloat32`` generator has no documented
semantics (testing.md:391-394), so those inputs are replaced by seeded normal values whose
seed is stored in the spec; the expected outputs were computed from exactly these inputs.
"""
from __future__ import annotations

import json
import zlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
CASES = HERE / "upstream_cases.json"
OUTPUTS = HERE / "upstream_outputs.npz"

_DT = {"float32": np.float32, "float16": np.float16, "uint8": np.uint8}


def seeded_normal(seed: int, count: int, scale: float) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return (rng.standard_normal(count) * scale).astype(np.float64)


def materialize(spec: dict) -> np.ndarray:
    """verify_upstream.materialize semantics for values/constant/cycle/linspace, plus 'seeded_normal'."""
    dtype = np.dtype(_DT[spec["dtype"]])
    shape = tuple(spec["shape"])
    count = int(np.prod(shape, dtype=np.int64)) if shape else 1
    gen = spec["data"]
    kind = gen["kind"]
    if kind == "values":
        arr = np.asarray(gen["values"], dtype=np.float64).astype(dtype)
        if arr.size != count:
            raise ValueError("values count differs from shape")
    elif kind == "constant":
        arr = np.full(count, gen["value"], dtype=np.float64).astype(dtype)
    elif kind == "cycle":
        arr = np.resize(np.asarray(gen["values"], dtype=np.float64).astype(dtype), count)
    elif kind == "linspace":
        arr = np.linspace(gen["start"], gen["end"], count, dtype=np.float64).astype(dtype)
    elif kind == "seeded_normal":
        arr = seeded_normal(int(gen["seed"]), count, float(gen.get("scale", 1.0))).astype(dtype)
    else:
        raise ValueError(f"unknown generator {kind}")
    return np.ascontiguousarray(arr).reshape(shape)


def case_seed(name: str, tensor: str) -> int:
    return zlib.crc32(f"{name}/{tensor}".encode()) & 0x7FFFFFFF


def load_cases():
    """Return a list of dicts: name, attrs, inputs (name -> ndarray), expected (dict), tolerance."""
    specs = json.loads(CASES.read_text())
    outputs = np.load(OUTPUTS)
    cases = []
    for spec in specs["cases"]:
        inputs = {k: materialize(v) for k, v in spec["inputs"].items()}
        name = spec["name"]
        exp = {"mode": spec["expected_mode"], "dtype": spec["output"]["dtype"], "shape": tuple(spec["output"]["shape"])}
        if exp["mode"] == "full":
            exp["y"] = outputs[f"{name}/y"]
        else:
            exp["index"] = outputs[f"{name}/index"]
            exp["values"] = outputs[f"{name}/values"]
            exp["sum"] = float(outputs[f"{name}/sum"])
            exp["sumsq"] = float(outputs[f"{name}/sumsq"])
        if f"{name}/published" in outputs:
            exp["published"] = outputs[f"{name}/published"]
        cases.append({"name": name, "attrs": spec["attrs"], "inputs": inputs, "expected": exp,
                      "atol": float(spec["output"].get("tolerance", 0.0)),
                      "rtol": float(spec["output"].get("relTolerance", 0.0)),
                      "substituted": spec.get("substituted", [])})
    return cases


def compare(actual, expected, atol: float, rtol: float) -> dict:
    """verify_upstream.compare semantics (kernels/_shared/verify_upstream.py:137-151)."""
    actual = np.asarray(actual)
    expected = np.asarray(expected)
    if actual.dtype != expected.dtype or actual.shape != expected.shape:
        return dict(passed=False, reason="Output shape or dtype mismatch")
    finite = np.isfinite(actual) & np.isfinite(expected)
    special = (actual == expected) & ~finite
    err = np.abs(actual[finite].astype(np.float64) - expected[finite].astype(np.float64))
    limit = atol + rtol * np.abs(expected[finite].astype(np.float64))
    ok = bool(np.all(finite | special) and np.all(err <= limit))
    return dict(passed=ok, max_absolute_error=float(err.max()) if err.size else 0.0,
                nonfinite_mismatches=int(np.count_nonzero(~finite & ~special)))


def check_against(actual: np.ndarray, exp: dict, atol: float, rtol: float) -> dict:
    """Compare a computed Y with a fixture's expected data (full array or sampled entries)."""
    actual = np.asarray(actual)
    if actual.shape != exp["shape"]:
        return dict(passed=False, reason=f"shape {actual.shape} != {exp['shape']}")
    if exp["mode"] == "full":
        return compare(actual, exp["y"], atol, rtol)
    flat = actual.reshape(-1)
    res = compare(flat[exp["index"]], exp["values"], atol, rtol)
    a64 = flat.astype(np.float64)
    n = max(1, a64.size)
    # Checksums: mean and RMS must agree to the case tolerance (scaled by the spread).
    mean_tol = atol + rtol * abs(exp["sum"] / n) + 1e-6 * np.sqrt(exp["sumsq"] / n)
    res["mean_ok"] = bool(abs(a64.sum() / n - exp["sum"] / n) <= max(mean_tol, 1e-12))
    res["passed"] = bool(res["passed"] and res["mean_ok"])
    return res

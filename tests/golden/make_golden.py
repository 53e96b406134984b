"""Regenerates tests/golden/upstream_cases.json and upstream_outputs.npz.

Run in a checkout that has the xrGPU reference (default /root/reference, override with
XRGPU_REFERENCE_ROOT):  python tests/golden/make_golden.py

For every case of the reference's frozen MatMulNBits suite
(kernels/_provenance/upstream/com.microsoft.MatMulNBits/build/webgpu/test.json):
  * the generator specs are resolved ($ref into fixtureArrays) and recorded; ``fillFloat32``
    inputs are replaced by seeded normal values (its semantics are undocumented,
    testing.md:391-394) and listed under "substituted";
  * the expected Y is computed by the reference's own algorithm compiled from its sources
    (oracle/_ref/libmmnb_ref.so: packedMatmul/nbitWeight of complex_kernel.glsl:80-83 with
    half.glsl's conversions), and, where the suite publishes an explicit output, that output is
    stored too and must agree with the reference computation.
Outputs with more than SAMPLE_LIMIT elements are stored as a seeded sample of entries plus a
sum and a sum of squares.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from fixtures import CASES, OUTPUTS, case_seed, compare, materialize  # noqa: E402
from oracle.native import ReferenceC  # noqa: E402

REFERENCE = Path(os.environ.get("XRGPU_REFERENCE_ROOT", "/root/reference"))
SUITE = REFERENCE / "kernels/_provenance/upstream/com.microsoft.MatMulNBits/build/webgpu/test.json"
SAMPLE_LIMIT = 16384
SAMPLE_COUNT = 4096
INPUT_ORDER = ("aT", "bT", "scalesT", "zeroPointsT", "biasT")


def resolve(values, doc):
    if isinstance(values, dict) and "$ref" in values:
        ref = values["$ref"]
        assert ref.startswith("#/fixtureArrays/")
        return doc["fixtureArrays"][ref.split("/")[-1]]
    return values


def main():
    doc = json.loads(SUITE.read_text())
    ref = ReferenceC()
    specs, arrays = [], {}
    for case in doc["cases"]:
        name = case["name"]
        inputs, substituted = {}, []
        for tname in INPUT_ORDER:
            if tname not in case["inputs"]:
                continue
            t = case["inputs"][tname]
            gen = dict(t["data"])
            if gen["kind"] == "fillFloat32":
                gen = {"kind": "seeded_normal", "seed": case_seed(name, tname), "scale": float(gen.get("scale", 1.0))}
                substituted.append(tname)
            elif "values" in gen:
                gen["values"] = resolve(gen["values"], doc)
            inputs[tname] = {"dtype": t["dtype"], "shape": t["shape"], "data": gen}
        attrs = {k: int(v) for k, v in case["attrs"].items()}
        out = case["outputs"]["yT"]
        arr = {k: materialize(v) for k, v in inputs.items()}
        K, N = attrs["K"], attrs["N"]
        bits, bs = attrs.get("bits", 4), attrs["block_size"]
        y = ref.matmul(arr["aT"], arr["bT"], arr["scalesT"], arr.get("zeroPointsT"), arr.get("biasT"), K=K, N=N,
                       bits=bits, block_size=bs, threads=8)
        assert list(y.shape) == list(out["shape"]), (name, y.shape, out["shape"])
        spec = {"name": name, "attrs": attrs, "inputs": inputs, "substituted": substituted,
                "output": {k: out[k] for k in ("dtype", "shape", "tolerance", "relTolerance") if k in out}}
        if "data" in out:
            published = materialize({"dtype": out["dtype"], "shape": out["shape"], "data": out["data"]})
            res = compare(y, published, out.get("tolerance", 0), out.get("relTolerance", 0))
            assert res["passed"], (name, res)
            arrays[f"{name}/published"] = published
        if y.size <= SAMPLE_LIMIT:
            spec["expected_mode"] = "full"
            arrays[f"{name}/y"] = y
        else:
            spec["expected_mode"] = "sampled"
            rng = np.random.default_rng(case_seed(name, "sample"))
            idx = np.sort(rng.choice(y.size, SAMPLE_COUNT, replace=False)).astype(np.int64)
            flat = y.reshape(-1)
            arrays[f"{name}/index"] = idx
            arrays[f"{name}/values"] = flat[idx]
            arrays[f"{name}/sum"] = np.float64(flat.astype(np.float64).sum())
            arrays[f"{name}/sumsq"] = np.float64((flat.astype(np.float64) ** 2).sum())
        specs.append(spec)
    CASES.write_text(json.dumps({"source": "kernels/_provenance/upstream/com.microsoft.MatMulNBits/build/webgpu/test.json",
                                 "expected_by": "oracle/_ref (reference packedMatmul compiled as C++)",
                                 "cases": specs}, indent=1))
    np.savez_compressed(OUTPUTS, **arrays)
    print(f"{len(specs)} cases -> {CASES.name}, {OUTPUTS.name} ({OUTPUTS.stat().st_size} bytes)")


if __name__ == "__main__":
    main()

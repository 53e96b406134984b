"""Regenerates tests/golden/family_cases.json and family_cases.npz.

Known-answer vectors for the operators that call or share MatMulNBits' quantized formats:
com.microsoft.MatMulNBitsMlp, MatMulNBitsQkv, MatMulBnb4, GatherBlockQuantized and QMoE.
They are taken from the reference's own independent test module
(kernels/_shared/extended/complex_reference.py), imported from the reference checkout
(XRGPU_REFERENCE_ROOT):

  * ``published_cases(full=True)``: the frozen upstream suites' cases that publish explicit
    outputs (kernels/_provenance/upstream/<op>/build/webgpu/test.json);
  * ``custom_cases()`` and ``advanced_cases()``: the reference's hand-built independent cases
    (its NumPy ``moe_reference`` for QMoE, closed-form expectations for the others).

Each case keeps its inputs, expected outputs, attributes and per-output tolerance exactly as the
reference module produced them. Run:  python tests/golden/make_family_golden.py
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REFERENCE = Path(os.environ.get("XRGPU_REFERENCE_ROOT", "/root/reference"))
OPS = ("com.microsoft.MatMulNBitsMlp", "com.microsoft.MatMulNBitsQkv", "com.microsoft.MatMulBnb4",
       "com.microsoft.GatherBlockQuantized", "com.microsoft.QMoE")


def _jsonable(v):
    if isinstance(v, (np.integer,)):
        return int(v)
    if isinstance(v, (np.floating,)):
        return float(v)
    if isinstance(v, dict):
        return {k: _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    return v


def main():
    for sub in ("kernels/_shared/extended", "kernels/_shared", "."):
        sys.path.insert(0, str(REFERENCE / sub))
    import complex_reference as cr  # the reference's own test module

    cases = []
    for source, rows in (("published", cr.published_cases(full=True)), ("custom", cr.custom_cases()),
                         ("advanced", cr.advanced_cases())):
        for row in rows:
            if row["operation"] in OPS:
                cases.append((source, row))
    arrays, meta = {}, []
    for i, (source, row) in enumerate(cases):
        entry = {"index": i, "source": source, "operation": row["operation"], "name": row["name"],
                 "attrs": _jsonable(row.get("attrs", {})), "args": _jsonable(row.get("args", {})),
                 "inputs": [], "outputs": []}
        for name, value in row["inputs"].items():
            arrays[f"{i}/in/{name}"] = np.asarray(value)
            desc = row.get("input_descriptors", {}).get(name, {})
            entry["inputs"].append({"name": name, "dtype": str(np.asarray(value).dtype),
                                    "logical_dtype": desc.get("dtype"), "source_dtype": desc.get("source_dtype")})
        for name, value in row["expected"].items():
            arrays[f"{i}/out/{name}"] = np.asarray(value)
            tol = row.get("comparisons", {}).get(name) if row.get("comparisons") else None
            entry["outputs"].append({"name": name, "dtype": str(np.asarray(value).dtype),
                                     "tolerance": _jsonable(tol) if tol else None})
        meta.append(entry)
    np.savez_compressed(HERE / "family_cases.npz", **arrays)
    (HERE / "family_cases.json").write_text(json.dumps(meta, indent=1) + "\n")
    counts = {}
    for e in meta:
        counts[e["operation"]] = counts.get(e["operation"], 0) + 1
    print(json.dumps(counts))


if __name__ == "__main__":
    main()

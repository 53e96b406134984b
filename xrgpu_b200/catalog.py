"""Registration of the CUDA backend for com.microsoft.MatMulNBits.

``kernels/catalog.json`` lists the operators this backend serves, keyed by backend, with the
sha256 of each descriptor; ``load()`` validates it the way the reference's Vulkan catalog loader
validates its entries (kernels/catalog.py:85-248): catalog identity digest, descriptor paths and
digests, that the contract rejects unsupported execution (``cpu_fallback`` and
``silent_type_conversion`` false), that the catalog's ``native`` record matches the contract's,
and that the portable contract (inputs, outputs, attributes, constraints) is present. The
Vulkan catalog's own invariants (221 ids, 315 SPIR-V variants, backend "vulkan") are untouched:
this is an additional catalog for backend "cuda".
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

KERNELS = Path(__file__).resolve().parent / "kernels"
BACKEND, TARGET = "cuda", "sm_100a"
PORTABLE_KEYS = ("inputs", "outputs", "attributes", "attribute_constraints", "type_constraints")


def _sha(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def _digest(value) -> str:
    return hashlib.sha256(json.dumps(value, sort_keys=True, separators=(",", ":")).encode()).hexdigest()


def load(root: Path = KERNELS) -> dict:
    """Validate and return the CUDA backend catalog."""
    root = Path(root)
    value = json.loads((root / "catalog.json").read_text())
    if value.get("schema_version") != 1 or value.get("kind") != "xrgpu.native-kernel-catalog":
        raise ValueError("Unsupported native catalog")
    if _digest({k: v for k, v in value.items() if k != "catalog_sha256"}) != value.get("catalog_sha256"):
        raise ValueError("Native catalog identity mismatch")
    if (value.get("backend"), value.get("target")) != (BACKEND, TARGET):
        raise ValueError("Unsupported native catalog target")
    entries = value.get("entries", [])
    if len(entries) != value.get("operator_count") or len({e["id"] for e in entries}) != len(entries):
        raise ValueError("Native catalog operator count mismatch")
    for entry in entries:
        identity = entry["id"]
        if entry["path"] != identity or entry["contract"] != identity + "/contract.json":
            raise ValueError("Native operator descriptor path mismatch")
        file = root / entry["contract"]
        if _sha(file) != entry["descriptor_digests"]["contract"]:
            raise ValueError("Native descriptor checksum mismatch: " + entry["contract"])
        contract = json.loads(file.read_text())
        if (contract.get("kind"), contract.get("id"), contract.get("backend"), contract.get("target")) != (
                "xrgpu.native-operator", identity, BACKEND, TARGET):
            raise ValueError("Native descriptor target/identity mismatch")
        if contract["native"] != entry["native"]:
            raise ValueError("Native catalog and contract differ: " + identity)
        caps = contract.get("capabilities", {})
        if caps.get("cpu_fallback") is not False or caps.get("silent_type_conversion") is not False:
            raise ValueError("Native contract must reject unsupported execution")
        for key in PORTABLE_KEYS:
            if key not in contract:
                raise ValueError("Native portable contract incomplete: " + key)
    return value


def contract(identity: str = "com.microsoft.MatMulNBits", root: Path = KERNELS) -> dict:
    load(root)
    return json.loads((Path(root) / identity / "contract.json").read_text())


def refresh(root: Path = KERNELS) -> dict:
    """Regenerate catalog.json digests from the descriptors (maintainer tool)."""
    root = Path(root)
    entries = []
    for file in sorted(root.glob("*/contract.json")):
        c = json.loads(file.read_text())
        entries.append({"id": c["id"], "path": c["id"], "contract": c["id"] + "/contract.json",
                        "descriptor_digests": {"contract": _sha(file)}, "native": c["native"]})
    value = {"schema_version": 1, "kind": "xrgpu.native-kernel-catalog", "backend": BACKEND, "target": TARGET,
             "operator_count": len(entries), "entries": entries}
    value["catalog_sha256"] = _digest(value)
    (root / "catalog.json").write_text(json.dumps(value, indent=2, sort_keys=True) + "\n")
    return value


if __name__ == "__main__":
    print(json.dumps(refresh(), indent=2)[:400])

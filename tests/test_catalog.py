"""Registration: the CUDA backend catalog validates like the reference's catalog loader and
its portable contract is the reference operator's contract."""
import json
import shutil
from pathlib import Path

import pytest

from oracle.build import DEFAULT_REFERENCE  # XRGPU_REFERENCE_ROOT, the checkout the checkers use
from xrgpu_b200 import catalog

REFERENCE_CONTRACT = DEFAULT_REFERENCE / "kernels/com.microsoft.MatMulNBits/contract.json"


def test_catalog_loads():
    value = catalog.load()
    assert value["backend"] == "cuda" and value["operator_count"] == 1
    c = catalog.contract()
    assert c["capabilities"]["cpu_fallback"] is False


def test_catalog_rejects_tampering(tmp_path):
    root = tmp_path / "kernels"
    shutil.copytree(catalog.KERNELS, root)
    path = root / "com.microsoft.MatMulNBits" / "contract.json"
    c = json.loads(path.read_text())
    c["capabilities"]["cpu_fallback"] = True
    path.write_text(json.dumps(c))
    with pytest.raises(ValueError, match="checksum"):
        catalog.load(root)
    catalog.refresh(root)  # digests now match, but the contract itself is invalid
    with pytest.raises(ValueError, match="reject unsupported execution"):
        catalog.load(root)


def test_native_entry_points_exported(cuda_lib):
    c = catalog.contract()
    for name in c["native"]["operator_entry_points"] + c["native"]["device_entry_points"]:
        assert hasattr(cuda_lib, name), name


@pytest.mark.skipif(not REFERENCE_CONTRACT.exists(), reason="reference checkout not present")
def test_portable_contract_equals_reference():
    ours = catalog.contract()
    ref = json.loads(REFERENCE_CONTRACT.read_text())
    for key in catalog.PORTABLE_KEYS:
        assert ours[key] == ref[key], key
    assert ref["capabilities"]["cpu_fallback"] is False

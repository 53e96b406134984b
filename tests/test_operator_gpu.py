"""Operator-API semantics on the GPU: the reference's prepare/run/read_outputs/info/close
lifecycle (extended_operators.h:49-61, vulkan.cpp:105-123), ownership, limits and poisoning."""
import json

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import mmnb_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def api(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from xrgpu_b200 import operators
    return operators


def request(api, M=2, K=256, N=64, bs=32, dt=np.float16, seed=0, a_shape=None, zp=None):
    rng = np.random.default_rng(seed)
    kb = K // bs
    a = rng.standard_normal(a_shape or (M, K)).astype(dt)
    b = rng.integers(0, 256, (N, kb, bs // 2), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, (N, kb)).astype(dt)
    bias = rng.standard_normal(N).astype(dt)
    T = api.Tensor.from_numpy
    inputs = [T("aT", a), T("bT", b), T("scalesT", s), T("biasT", bias)]
    if zp is not None:
        inputs.insert(3, T("zeroPointsT", zp))
    r = api.Request(inputs=inputs, attrs=api.Attributes(integers={"K": K, "N": N, "block_size": bs}))
    return r, (a, b, s, zp, bias)


def test_lifecycle_and_info(api):
    r, (a, b, s, zp, bias) = request(api, a_shape=(2, 3, 256))
    op = api.Operator.prepare(None, r, api.Options(profiling=True))
    op.run()
    (y,) = op.read_outputs()
    assert y.name == "yT" and y.shape == [2, 3, 64] and y.dtype == api.DType.Float16
    ref = O.matmul_nbits(a, b, s, None, bias, K=256, N=64, block_size=32)
    assert np.abs(y.numpy().astype(np.float32) - ref.astype(np.float32)).max() <= 2e-2
    info = json.loads(op.info())
    assert info["backend"] == "cuda" and info["cpu_compute_fallback"] is False
    assert info["dispatch_count"] == 1 and info["executed"] and not info["closed"]
    assert info["gpu_ms"] is not None and info["execution_ms"] >= 0
    op.run()  # repeated runs reuse the prepared snapshot
    (y2,) = op.read_outputs()
    assert y2.data == y.data
    op.close()
    assert json.loads(op.info())["closed"] is True
    with pytest.raises(RuntimeError, match="closed"):
        op.run()


def test_prepare_snapshots_inputs_and_write_input_replaces(api):
    r, (a, b, s, zp, bias) = request(api, M=1, K=512, N=32, seed=3)
    op = api.Operator.prepare(None, r)
    r.inputs[0].data = b"\x00" * len(r.inputs[0].data)  # mutating the request does not affect the handle
    op.run()
    (y,) = op.read_outputs()
    ref = O.matmul_nbits(a, b, s, None, bias, K=512, N=32, block_size=32)
    assert np.abs(y.numpy().astype(np.float32) - ref.astype(np.float32)).max() <= 2e-2
    a2 = (a * 2).astype(np.float16)
    op.write_input("aT", a2)
    op.run()
    (y2,) = op.read_outputs()
    ref2 = O.matmul_nbits(a2, b, s, None, bias, K=512, N=32, block_size=32)
    assert np.abs(y2.numpy().astype(np.float32) - ref2.astype(np.float32)).max() <= 4e-2
    with pytest.raises(ValueError, match="byte count"):
        op.write_input("aT", a2[:, :10])
    op.close()


def test_empty_rows_run(api):
    for dt in (np.float32, np.float16):
        r, _ = request(api, M=0, K=32, N=4, dt=dt)
        op = api.Operator.prepare(None, r)
        op.run()
        (y,) = op.read_outputs()
        assert y.shape == [0, 4] and y.data == b""
        op.close()


def test_memory_limit_is_enforced_and_raisable(api):
    r, _ = request(api, M=1, K=4096, N=4096)
    with pytest.raises(ValueError, match="memory limit"):
        api.Operator.prepare(None, r, api.Options(memory_limit_bytes=1 << 20))
    op = api.Operator.prepare(None, r, api.Options(memory_limit_bytes=1 << 30))
    op.run()
    op.close()


def test_timeout_poisons_until_close(api):
    # A 1 ns budget expires before the kernel can complete: run() reports TIMEOUT and the
    # handle stays poisoned (vulkan.cpp:105,115); close() still releases it. No GPU fault is
    # involved: the kernel finishes normally in the background.
    from xrgpu_b200._native import TIMEOUT, XrgpuError
    r, _ = request(api, M=1, K=4096, N=8192)
    op = api.Operator.prepare(None, r, api.Options(timeout_ns=1, memory_limit_bytes=1 << 30))
    with pytest.raises(XrgpuError) as e:
        op.run()
    assert e.value.status == TIMEOUT
    with pytest.raises(RuntimeError, match="failed earlier"):
        op.run()
    op.close()


def test_invalid_device_ordinal(api):
    r, _ = request(api)
    with pytest.raises(ValueError, match="device"):
        api.Operator.prepare(None, r, api.Options(device=1000))


def test_packed_and_float_zero_points_agree(api):
    rng = np.random.default_rng(9)
    K, N, bs = 1024, 48, 32
    kb = K // bs
    codes = rng.integers(0, 16, (N, kb))
    packed = np.zeros((N, (kb + 1) // 2), np.uint8)
    for j in range(kb):
        packed[:, j // 2] |= (codes[:, j] << (4 * (j % 2))).astype(np.uint8)
    r1, (a, b, s, _, bias) = request(api, M=1, K=K, N=N, zp=codes.astype(np.float16), seed=9)
    r2, _ = request(api, M=1, K=K, N=N, zp=packed, seed=9)
    ys = []
    for r in (r1, r2):
        op = api.Operator.prepare(None, r)
        op.run()
        ys.append(op.read_outputs()[0].numpy())
        op.close()
    ref = O.matmul_nbits(a, b, s, codes.astype(np.float16), bias, K=K, N=N, block_size=bs)
    for y in ys:
        assert np.abs(y.astype(np.float32) - ref.astype(np.float32)).max() <= 2e-2

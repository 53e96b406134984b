"""GPU parity of the operators around MatMulNBits (MatMulNBitsMlp, MatMulNBitsQkv, MatMulBnb4,
GatherBlockQuantized, QMoE) through the C ABI.

* The reference's known-answer vectors (tests/golden/family_cases.*) through the operator API
  (xrgpu_prepare_ex / run / read_outputs), each within its own tolerance.
* Seeded inputs at decode and prefill shapes through the zero-copy API against the family oracle
  (oracle/family_oracle.py), within BASELINE.json's tolerances: max|dY| <= 1e-2 max|Y_ref|,
  relative Frobenius <= 2e-3.
"""
import json
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import family_oracle as FO
from xrgpu_b200 import _native
from xrgpu_b200.operators import Attributes, DType, Operator, Request, Tensor

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "family_cases.json").read_text())
ARRAYS = np.load(GOLDEN / "family_cases.npz")


@pytest.fixture(scope="module")
def F(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from xrgpu_b200 import functional
    return functional


def dev(x):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).cuda()


def within(got, ref, max_rel=1e-2, frob=2e-3):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return got.shape == ref.shape
    d = got - ref
    scale = max(np.abs(ref).max(), 1e-30)
    return (got.shape == ref.shape and np.abs(d).max() <= max_rel * scale
            and np.linalg.norm(d) <= frob * max(np.linalg.norm(ref), 1e-30))


# ----------------------------------------------------------------- golden vectors, operator API
def _attrs(entry):
    ints, nums, strs = {}, {}, {}
    for k, v in {**entry["attrs"], **entry["args"]}.items():
        if isinstance(v, bool) or isinstance(v, int):
            ints[k] = int(v)
        elif isinstance(v, float):
            nums[k] = v
        else:
            strs[k] = str(v)
    return Attributes(integers=ints, numbers=nums, strings=strs)


@pytest.mark.parametrize("entry", META, ids=lambda e: e["operation"].split(".")[-1] + ":" + e["name"])
def test_reference_known_answers_through_operator_api(F, entry):
    i = entry["index"]
    tensors = []
    for d in entry["inputs"]:
        arr = ARRAYS[f"{i}/in/{d['name']}"]
        if d["name"] == "indicesT":  # contract dtype int64 (the suite stores its uint32 storage form)
            arr = arr.astype(np.int64)
        tensors.append(Tensor.from_numpy(d["name"], arr))
    outs = [(d["name"], ARRAYS[f"{i}/out/{d['name']}"], d["tolerance"]) for d in entry["outputs"]]
    req = Request(entry["operation"], tensors, _attrs(entry),
                  requested_outputs=[Tensor(name=n, shape=list(a.shape), dtype=DType.Float32 if a.dtype == np.float32
                                            else DType.Float16) for n, a, _ in outs])
    with Operator.prepare(None, req) as op:
        op.run()
        got = {t.name: t.numpy() for t in op.read_outputs()}
        assert json.loads(op.info())["cpu_compute_fallback"] is False
    for name, exp, tol in outs:
        atol, rtol = (tol or {}).get("atol", 0.0), (tol or {}).get("rtol", 0.0)
        g = got[name].astype(np.float64)
        assert g.shape == exp.shape, name
        assert np.all(np.abs(g - exp) <= atol + rtol * np.abs(exp.astype(np.float64))), (name, g, exp)
    assert F.device_error(0) == 0


# ----------------------------------------------------------------- seeded problems, zero-copy API
def _weights(rng, N, K, bs, bits=4, dt=np.float16):
    kb = K // bs
    b = rng.integers(0, 256, (N, kb, bs * bits // 8), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, (N, kb)).astype(dt)
    return b, s


@pytest.mark.parametrize("M,K,N,bs,dt", [(1, 4096, 1024, 32, np.float16), (3, 1024, 640, 64, np.float16),
                                         (64, 2048, 512, 32, np.float16), (2, 512, 96, 32, np.float32)])
@pytest.mark.parametrize("norm,skip,bias", [(True, True, True), (False, False, False), (True, False, False)])
def test_mlp_matches_oracle(F, M, K, N, bs, dt, norm, skip, bias):
    rng = np.random.default_rng(M * 7 + K + N + 3 * norm + 5 * skip)
    a = rng.standard_normal((M, K)).astype(dt)
    sk = rng.standard_normal((M, K)).astype(dt) if skip else None
    ns = rng.uniform(0.5, 1.5, K).astype(dt) if norm else None
    gb, gs = _weights(rng, N, K, bs, dt=dt)
    ub, us = _weights(rng, N, K, bs, dt=dt)
    gbias = rng.standard_normal(N).astype(dt) if bias else None
    ubias = rng.standard_normal(N).astype(dt) if bias else None
    y, res = F.matmul_nbits_mlp(dev(a), dev(gb), dev(gs), dev(ub), dev(us), skip=dev(sk), norm_scale=dev(ns),
                                gate_bias=dev(gbias), up_bias=dev(ubias), K=K, N=N, block_size=bs, want_residual=True)
    torch.cuda.synchronize()
    ry, rres = FO.matmul_nbits_mlp(a, sk, ns, gb, gs, gbias, ub, us, ubias, K=K, N=N, block_size=bs)
    assert within(y.cpu().numpy(), ry) and within(res.cpu().numpy(), rres, 1e-3, 1e-3)
    assert F.device_error(0) == 0


@pytest.mark.parametrize("M,K,Nq,Nkv,dt", [(1, 4096, 4096, 1024, np.float16), (5, 2048, 512, 128, np.float16),
                                           (96, 1024, 256, 128, np.float16), (2, 256, 64, 32, np.float32)])
def test_qkv_matches_oracle(F, M, K, Nq, Nkv, dt):
    rng = np.random.default_rng(M + K + Nq)
    bs = 32
    a = rng.standard_normal((M, K)).astype(dt)
    sk = rng.standard_normal((M, K)).astype(dt)
    ns = rng.uniform(0.5, 1.5, K).astype(dt)
    w = [_weights(rng, n, K, bs, dt=dt) for n in (Nq, Nkv, Nkv)]
    q, k, v, res = F.matmul_nbits_qkv(dev(a), dev(ns), dev(w[0][0]), dev(w[0][1]), dev(w[1][0]), dev(w[1][1]),
                                      dev(w[2][0]), dev(w[2][1]), skip=dev(sk), K=K, block_size=bs, want_residual=True)
    torch.cuda.synchronize()
    rq, rk, rv, rres = FO.matmul_nbits_qkv(a, sk, ns, w[0][0], w[0][1], w[1][0], w[1][1], w[2][0], w[2][1], K=K,
                                           Nq=Nq, Nkv=Nkv, block_size=bs)
    for got, ref in ((q, rq), (k, rk), (v, rv)):
        assert within(got.cpu().numpy(), ref)
    assert within(res.cpu().numpy(), rres, 1e-3, 1e-3)


@pytest.mark.parametrize("M,K,N,bs,qt,dt", [(1, 4096, 1024, 64, 1, np.float16), (4, 1024, 300, 128, 0, np.float16),
                                            (3, 100, 17, 16, 1, np.float32), (2, 512, 64, 32, 0, np.float32)])
def test_bnb4_matches_oracle(F, M, K, N, bs, qt, dt):
    rng = np.random.default_rng(K + N + qt)
    a = rng.standard_normal((M, K)).astype(dt)
    b = rng.integers(0, 256, (N * K + 1) // 2, dtype=np.uint8)
    absmax = rng.uniform(0.5, 2.0, (N * K + bs - 1) // bs).astype(dt)
    y = F.matmul_bnb4(dev(a), dev(b), dev(absmax), K=K, N=N, block_size=bs, quant_type=qt)
    torch.cuda.synchronize()
    ref = FO.matmul_bnb4(a, b, absmax, K=K, N=N, block_size=bs, quant_type=qt)
    assert within(y.cpu().numpy(), ref)


@pytest.mark.parametrize("bits,bs,zp,idx", [(4, 128, True, torch.int64), (4, 32, False, torch.int32),
                                            (8, 64, True, torch.int64), (8, 16, False, torch.int64)])
def test_gather_block_quantized_bit_exact(F, bits, bs, zp, idx):
    rng = np.random.default_rng(bits * bs)
    rows, width = 1000, 4096
    data = rng.integers(0, 256, (rows, width * bits // 8), dtype=np.uint8)
    blocks = width // bs
    scales = rng.uniform(0.01, 0.1, (rows, blocks)).astype(np.float32)
    z = rng.integers(0, 256, (rows, (blocks * bits + 7) // 8), dtype=np.uint8) if zp else None
    ind = rng.integers(0, rows, 37)
    out = F.gather_block_quantized(dev(data), torch.from_numpy(ind).to(idx).cuda(), dev(scales), dev(z), bits=bits,
                                   block_size=bs)
    torch.cuda.synchronize()
    ref, failed = FO.gather_block_quantized(data, ind, scales, z, bits=bits, block_size=bs)
    assert not failed and np.array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))
    assert F.device_error(0) == 0


def test_gather_out_of_range_index_reports_code_55(F):
    rng = np.random.default_rng(55)
    data = rng.integers(0, 256, (8, 32), dtype=np.uint8)
    scales = rng.uniform(0.01, 0.1, (8, 4)).astype(np.float32)
    ind = np.array([3, 8, -1, 0], dtype=np.int64)
    F.device_error(0, clear=True)
    out = F.gather_block_quantized(dev(data), dev(ind), dev(scales), bits=4, block_size=16)
    torch.cuda.synchronize()
    assert F.device_error(0, clear=True) == 55
    ref, failed = FO.gather_block_quantized(data, ind, scales, bits=4, block_size=16)
    assert failed and np.array_equal(out.cpu().numpy(), ref)
    # through the operator API the same failure is a device error that poisons the handle
    req = Request("com.microsoft.GatherBlockQuantized",
                  [Tensor.from_numpy("dataT", data), Tensor.from_numpy("indicesT", ind),
                   Tensor.from_numpy("scalesT", scales)], Attributes(integers={"bits": 4, "block_size": 16}))
    with Operator.prepare(None, req) as op:
        with pytest.raises(_native.XrgpuError, match="code 55"):
            op.run()
        with pytest.raises(_native.XrgpuError, match="failed earlier"):
            op.run()


@pytest.mark.parametrize("bits,bs,act,k", [(4, 0, "relu", 2), (4, 32, "swiglu", 2), (8, 0, "swiglu", 1),
                                           (8, 64, "relu", 3)])
def test_qmoe_matches_oracle(F, bits, bs, act, k):
    rng = np.random.default_rng(bits + bs + k)
    tokens, hidden, experts, inter = 5, 256, 8, 128
    rows = 2 * inter if act == "swiglu" else inter
    per = 8 // bits
    x = rng.standard_normal((tokens, hidden)).astype(np.float32)
    router = rng.standard_normal((tokens, experts)).astype(np.float32)
    fc1 = rng.integers(0, 256, (experts, rows, hidden // per), dtype=np.uint8)
    fc2 = rng.integers(0, 256, (experts, hidden, inter // per), dtype=np.uint8)
    s1 = rng.uniform(0.01, 0.03, (experts, rows) if not bs else (experts, rows, hidden // bs)).astype(np.float32)
    s2 = rng.uniform(0.01, 0.03, (experts, hidden) if not bs else (experts, hidden, inter // bs)).astype(np.float32)
    kw = dict(k=k, bits=bits, block_size=bs, activation=act, swiglu_fusion=1 if act == "swiglu" else 0,
              activation_alpha=1.702, activation_beta=1.0, swiglu_limit=7.0 if act == "swiglu" else None)
    out = F.qmoe(dev(x), dev(router), dev(fc1), dev(s1), dev(fc2), dev(s2), **kw)
    torch.cuda.synchronize()
    ref = FO.qmoe(x, router, fc1, s1, fc2, s2, **kw)
    assert within(out.cpu().numpy(), ref, 1e-4, 1e-5)
    assert F.device_error(0) == 0

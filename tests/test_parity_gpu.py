"""GPU parity: every CUDA kernel path against the CPU oracle, through the C ABI.

Bars (north star): dequantized weights bit-exact; Y within max|dY| <= 1e-2 * max|Y_ref| and
relative Frobenius error <= 2e-3 (BASELINE_TOL below); golden fixtures within each case's own
tolerance (upstream test.json, compare() semantics of kernels/_shared/verify_upstream.py:137-151).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import mmnb_oracle as O
from oracle.native import OracleC

import fixtures as G

pytestmark = pytest.mark.gpu

BASELINE_TOL = dict(max_abs_rel=1e-2, frob_rel=2e-3)


@pytest.fixture(scope="module")
def F(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from xrgpu_b200 import functional
    return functional


@pytest.fixture(scope="module")
def oc():
    return OracleC()


def dev(x):
    return None if x is None else torch.from_numpy(np.ascontiguousarray(x)).cuda()


def make(rng, M, K, N, bits, bs, dt, zp_kind=None, bias=False, a_shape=None):
    kb, blob = O.k_blocks(K, bs), O.blob_size(bs, bits)
    a = rng.standard_normal(a_shape or (M, K)).astype(dt)
    b = rng.integers(0, 256, (N, kb, blob), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, (N, kb)).astype(dt)
    if zp_kind is None:
        zp = None
    elif zp_kind == "packed":
        zp = rng.integers(0, 256, (N, (kb * bits + 7) // 8), dtype=np.uint8)
    elif zp_kind == "frac":  # non-integer float zero points (legal in the reference contract)
        zp = (rng.integers(0, 1 << bits, (N, kb)) + rng.uniform(-0.5, 0.5, (N, kb))).astype(np.float32)
    else:
        zp = rng.integers(0, 1 << bits, (N, kb)).astype(zp_kind)
    bb = rng.standard_normal(N).astype(dt) if bias else None
    return a, b, s, zp, bb


def within_baseline_tol(y, ref):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    if ref.size == 0:
        return True, {}
    scale = max(np.abs(ref).max(), 1e-30)
    max_abs = np.abs(y - ref).max()
    frob = np.linalg.norm(y - ref) / max(np.linalg.norm(ref), 1e-30)
    ok = max_abs <= BASELINE_TOL["max_abs_rel"] * scale and frob <= BASELINE_TOL["frob_rel"]
    return ok, dict(max_abs=max_abs, scale=scale, frob=frob)


def run_gpu(F, a, b, s, zp, bias, *, K, N, bits, bs, path):
    y = F.matmul_nbits(dev(a), dev(b), dev(s), dev(zp), dev(bias), K=K, N=N, bits=bits, block_size=bs, path=path)
    torch.cuda.synchronize()
    assert F.device_error(0) == 0
    return y.cpu().numpy()


# ----------------------------------------------------------------- dequantization (bit-exact)
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("dt", [np.float32, np.float16])
@pytest.mark.parametrize("zp_kind", [None, "float16", "float32", "packed", "frac"])
def test_dequantize_bit_exact(F, bits, dt, zp_kind):
    rng = np.random.default_rng(bits * 100 + (dt == np.float16))
    for K, N, bs in [(64, 8, 16), (77, 5, 32), (4096, 33, 128), (100, 3, 64)]:
        zk = {"float16": np.float16, "float32": np.float32}.get(zp_kind, zp_kind)
        a, b, s, zp, _ = make(rng, 1, K, N, bits, bs, dt, zk)
        w = F.dequantize(dev(b), dev(s), dev(zp), K=K, bits=bits, block_size=bs).cpu().numpy()
        ref = O.dequantize(b, s, zp, K=K, bits=bits, block_size=bs)
        assert np.array_equal(w.view(np.uint32), ref.view(np.uint32)), (K, N, bs)


# ----------------------------------------------------------------- generic kernel
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("dt", [np.float32, np.float16])
@pytest.mark.parametrize("zp_kind", [None, "float", "packed"])
def test_generic_matches_oracle(F, oc, bits, dt, zp_kind):
    rng = np.random.default_rng(7 * bits + (dt == np.float16))
    for (M, K, N, bs, a_shape) in [(3, 77, 19, 16, None), (8, 128, 64, 32, None), (1, 33, 5, 32, None),
                                   (6, 256, 40, 128, (2, 3, 256)), (17, 64, 9, 64, None)]:
        zk = dt if zp_kind == "float" else zp_kind
        a, b, s, zp, bias = make(rng, M, K, N, bits, bs, dt, zk, bias=True, a_shape=a_shape)
        y = run_gpu(F, a, b, s, zp, bias, K=K, N=N, bits=bits, bs=bs, path="generic")
        ref = oc.matmul(a, b, s, zp, bias, K=K, N=N, bits=bits, block_size=bs)
        assert y.shape == ref.shape and y.dtype == ref.dtype
        ok, st = within_baseline_tol(y, ref)
        assert ok, (M, K, N, bs, st)
        tol = 1e-4 if dt == np.float32 else 2e-3
        assert np.abs(y.astype(np.float64) - ref).max() <= tol * max(1.0, np.abs(ref).max())


# ----------------------------------------------------------------- decode GEMV (tensor cores)
GEMV_SHAPES = [
    # (M, K, N, bs)
    (1, 64, 16, 32), (1, 4096, 4096, 32), (1, 4096, 1024, 32), (4, 4096, 1000, 128), (1, 1024, 7, 64),
    (8, 2048, 300, 32), (9, 512, 64, 64), (16, 4096, 512, 128), (2, 14336, 256, 32), (3, 768, 4100, 256),
]


@pytest.mark.parametrize("M,K,N,bs", GEMV_SHAPES)
@pytest.mark.parametrize("zp_kind", [None, "float16", "packed", "frac"])
def test_gemv_matches_oracle(F, M, K, N, bs, zp_kind):
    rng = np.random.default_rng(M * 131 + K + N + bs)
    zk = {"float16": np.float16}.get(zp_kind, zp_kind)
    a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, zk, bias=(N % 2 == 0))
    assert F.select_path(dev(a), dev(b), dev(s), dev(zp), K=K, N=N, bits=4, block_size=bs) == "gemv"
    y = run_gpu(F, a, b, s, zp, bias, K=K, N=N, bits=4, bs=bs, path="gemv")
    ref = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=4, block_size=bs)
    ok, st = within_baseline_tol(y, ref)
    assert ok, st
    # float16 output: allow one float16 rounding plus float32 reassociation
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    assert np.all(err <= 2e-3 * np.abs(ref.astype(np.float64)) + 1e-3 * np.abs(ref).max() + 1e-6)


def test_gemv_deterministic_and_linear_full_size(F):
    """Size-independent properties at the Llama-3-8B decode shapes (full size)."""
    rng = np.random.default_rng(11)
    for K, N in [(4096, 4096), (4096, 1024), (4096, 14336), (14336, 4096)]:
        a, b, s, zp, _ = make(rng, 1, K, N, 4, 32, np.float16, "packed")
        da, db, ds, dz = dev(a), dev(b), dev(s), dev(zp)
        y1 = F.matmul_nbits(da, db, ds, dz, K=K, N=N, block_size=32)
        y2 = F.matmul_nbits(da, db, ds, dz, K=K, N=N, block_size=32)
        y_2a = F.matmul_nbits(da * 2, db, ds, dz, K=K, N=N, block_size=32)
        torch.cuda.synchronize()
        assert torch.equal(y1, y2)                     # fixed-order split-K reduction
        normal = y1.abs() >= 2.0 ** -14                # doubling is exact except float16 subnormals
        assert torch.equal(y_2a[normal], (y1 * 2)[normal])
        cols = slice(0, 512)                           # oracle on a column sample
        ref = O.matmul_nbits(a, b, s, zp, K=K, N=N, bits=4, block_size=32, columns=cols)
        ok, st = within_baseline_tol(y1.cpu().numpy()[:, cols], ref)
        assert ok, (K, N, st)


def test_gemv_caller_workspace_reused_across_calls(F):
    """The GEMV needs no global scratch (its split-K partial sums meet in shared memory), so the
    reported workspace size is 0; a caller-owned workspace argument is accepted and ignored, and
    repeated calls give identical (deterministic) results within the tolerance of the oracle."""
    rng = np.random.default_rng(21)
    for (M, K, N, bs) in [(1, 4096, 4096, 32), (3, 14336, 1000, 64), (1, 576, 70, 32)]:
        a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, "packed", bias=True)
        need = F.workspace_size(M, K=K, N=N, bits=4, block_size=bs)
        assert need == 0
        ws = torch.zeros(64, dtype=torch.uint8, device="cuda")
        ys = [F.matmul_nbits(dev(a), dev(b), dev(s), dev(zp), dev(bias), K=K, N=N, block_size=bs, workspace=ws)
              for _ in range(3)]
        torch.cuda.synchronize()
        assert F.device_error(0) == 0
        assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])
        ref = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=4, block_size=bs)
        assert within_baseline_tol(ys[0].cpu().numpy(), ref)[0]


def test_gemv_writes_strided_output_slice(F):
    rng = np.random.default_rng(5)
    M, K, N, bs = 3, 1024, 96, 32
    a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, None, bias=True)
    big = torch.full((M, 3 * N), 7.0, dtype=torch.float16, device="cuda")
    F.matmul_nbits(dev(a), dev(b), dev(s), None, dev(bias), K=K, N=N, block_size=bs, out=big[:, N:2 * N])
    torch.cuda.synchronize()
    ref = O.matmul_nbits(a, b, s, None, bias, K=K, N=N, bits=4, block_size=bs)
    out = big.cpu().numpy()
    assert np.all(out[:, :N] == 7.0) and np.all(out[:, 2 * N:] == 7.0)
    assert within_baseline_tol(out[:, N:2 * N], ref)[0]


# Multi-row staged GEMV (block size 128 / 256, K % 512 == 0): M = 1..16 with one or two 8-row
# activation tiles, ragged N, every zero-point form, strided output rows, full config-3 width.
MR_SHAPES = [
    # (M, K, N, bs)
    (2, 4096, 1000, 128), (5, 2048, 777, 256), (8, 4096, 14336, 128), (9, 1024, 300, 128),
    (16, 4096, 14336, 128), (12, 1024, 64, 256), (1, 4096, 2048, 128), (16, 512, 17, 128),
]


@pytest.mark.parametrize("M,K,N,bs", MR_SHAPES)
@pytest.mark.parametrize("zp_kind", [None, "float16", "packed", "frac"])
def test_gemv_multirow_staged_matches_oracle(F, M, K, N, bs, zp_kind):
    rng = np.random.default_rng(M * 977 + K + N + bs)
    zk = {"float16": np.float16}.get(zp_kind, zp_kind)
    a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, zk, bias=(N % 2 == 0))
    y = run_gpu(F, a, b, s, zp, bias, K=K, N=N, bits=4, bs=bs, path="gemv")
    cols = slice(0, min(N, 2048))  # oracle on a column sample at full width
    ref = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=4, block_size=bs, columns=cols)
    ok, st = within_baseline_tol(y[:, cols], ref)
    assert ok, st
    err = np.abs(y[:, cols].astype(np.float64) - ref.astype(np.float64))
    assert np.all(err <= 2e-3 * np.abs(ref.astype(np.float64)) + 1e-3 * np.abs(ref).max() + 1e-6)
    y2 = run_gpu(F, a, b, s, zp, bias, K=K, N=N, bits=4, bs=bs, path="gemv")
    assert np.array_equal(y, y2)  # fixed-order sums of cut tiles


def test_gemv_multirow_staged_strided_output_rows(F):
    rng = np.random.default_rng(8)
    M, K, N, bs = 6, 2048, 96, 128
    a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, "packed", bias=True)
    big = torch.full((M, 3 * N), 7.0, dtype=torch.float16, device="cuda")
    F.matmul_nbits(dev(a), dev(b), dev(s), dev(zp), dev(bias), K=K, N=N, block_size=bs, out=big[:, N:2 * N])
    torch.cuda.synchronize()
    ref = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=4, block_size=bs)
    out = big.cpu().numpy()
    assert np.all(out[:, :N] == 7.0) and np.all(out[:, 2 * N:] == 7.0)
    assert within_baseline_tol(out[:, N:2 * N], ref)[0]


# ----------------------------------------------------------------- prefill GEMM (tcgen05)
GEMM_SHAPES = [
    # (M, K, N, bs): ragged M and N tiles, bs 16..128, one and many K steps, several tiles per CTA
    (1, 1024, 128, 32), (17, 2048, 100, 64), (64, 1024, 256, 16), (300, 1024, 384, 32),
    (129, 4096, 200, 128), (2048, 2048, 4096, 64), (520, 4096, 1056, 64), (40, 512, 64, 64),
]


def gemm_geometry_ok(K, bs, zp_kind):
    """The GEMM's TMA windows need 16-byte rows of scales (ceil(K/bs) % 8 == 0) and, for packed
    zero points, of zero-point bytes (ceil(K/bs) % 32 == 0); other shapes run the generic kernel."""
    kb = K // bs
    return K % 64 == 0 and kb % 8 == 0 and (zp_kind != "packed" or kb % 32 == 0)


@pytest.mark.parametrize("M,K,N,bs", GEMM_SHAPES)
@pytest.mark.parametrize("zp_kind", [None, "float16", "packed"])
def test_gemm_matches_oracle(F, M, K, N, bs, zp_kind):
    rng = np.random.default_rng(M * 7 + K + N * 3 + bs)
    zk = {"float16": np.float16}.get(zp_kind, zp_kind)
    a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, zk, bias=(M % 2 == 0))
    if not gemm_geometry_ok(K, bs, zp_kind):
        with pytest.raises(ValueError):
            F.select_path(dev(a), dev(b), dev(s), dev(zp), K=K, N=N, bits=4, block_size=bs, path="gemm")
        assert F.select_path(dev(a), dev(b), dev(s), dev(zp), K=K, N=N, bits=4, block_size=bs) == (
            "gemv" if M <= 16 else "generic")
        return
    assert F.select_path(dev(a), dev(b), dev(s), dev(zp), K=K, N=N, bits=4, block_size=bs, path="gemm") == "gemm"
    if M > 16:
        assert F.select_path(dev(a), dev(b), dev(s), dev(zp), K=K, N=N, bits=4, block_size=bs) == "gemm"
    y = run_gpu(F, a, b, s, zp, bias, K=K, N=N, bits=4, bs=bs, path="gemm")
    ref = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=4, block_size=bs)
    ok, st = within_baseline_tol(y, ref)
    assert ok, st
    # weights rounded once to float16 (the exact float32 weight's nearest float16) before the
    # float32 tensor-core sum, plus the float16 output rounding
    err = np.abs(y.astype(np.float64) - ref.astype(np.float64))
    assert np.all(err <= 4e-3 * np.abs(ref.astype(np.float64)) + 2e-3 * np.abs(ref).max() + 1e-6)


def test_gemm_prefill_full_size_properties(F):
    """Config 4 (M=2048, K=4096, N=14336, bs=64, no zero points) at full size: deterministic,
    exactly linear in A, and within the tolerance of the oracle on a row x column sample."""
    rng = np.random.default_rng(4)
    M, K, N, bs = 2048, 4096, 14336, 64
    a, b, s, _, _ = make(rng, M, K, N, 4, bs, np.float16, None)
    da, db, ds = dev(a), dev(b), dev(s)
    assert F.select_path(da, db, ds, None, K=K, N=N, block_size=bs) == "gemm"
    y1 = F.matmul_nbits(da, db, ds, None, K=K, N=N, block_size=bs)
    y2 = F.matmul_nbits(da, db, ds, None, K=K, N=N, block_size=bs)
    y_2a = F.matmul_nbits(da * 2, db, ds, None, K=K, N=N, block_size=bs)
    torch.cuda.synchronize()
    assert F.device_error(0) == 0
    assert torch.equal(y1, y2)
    # Exactly linear in A (every product and partial sum doubles), except where y1 was rounded
    # into the float16 subnormal range, whose absolute grid (2^-24) does not scale.
    normal = y1.float().abs() >= 2.0 ** -14
    assert torch.equal(y_2a[normal], (y1 * 2)[normal])
    assert torch.all((y_2a.float() - 2 * y1.float()).abs()[~normal] <= 2.0 ** -24)
    rows = np.r_[0:64, M - 64:M]
    y_host = y1.cpu().numpy()
    for cs in (slice(0, 256), slice(N - 256, N)):
        ref = O.matmul_nbits(a[rows], b, s, None, K=K, N=N, bits=4, block_size=bs, columns=cs)
        ok, st = within_baseline_tol(y_host[rows][:, cs], ref)
        assert ok, st


@pytest.mark.parametrize("M", [1, 4096])
def test_config5_shard_full_size(F, M):
    """Config 5 (70B-scale, bs 32, packed zero points): one GPU's 1/8 shard of the lm_head
    projection, (K, N) = (8192, 16032), at decode (GEMV) and prefill (GEMM) size: deterministic
    and within the tolerance of the oracle on a row x column sample."""
    rng = np.random.default_rng(5)
    K, N, bs = 8192, 16032, 32
    a, b, s, zp, _ = make(rng, M, K, N, 4, bs, np.float16, "packed")
    da, db, ds, dz = dev(a), dev(b), dev(s), dev(zp)
    assert F.select_path(da, db, ds, dz, K=K, N=N, block_size=bs) == ("gemv" if M == 1 else "gemm")
    y1 = F.matmul_nbits(da, db, ds, dz, K=K, N=N, block_size=bs)
    y2 = F.matmul_nbits(da, db, ds, dz, K=K, N=N, block_size=bs)
    torch.cuda.synchronize()
    assert F.device_error(0) == 0
    assert torch.equal(y1, y2)
    rows = np.r_[0:min(M, 32), max(0, M - 32):M] if M > 1 else np.r_[0:1]
    y_host = y1.cpu().numpy()
    for cs in (slice(0, 256), slice(N - 256, N)):
        ref = O.matmul_nbits(a[rows], b, s, zp, K=K, N=N, bits=4, block_size=bs, columns=cs)
        ok, st = within_baseline_tol(y_host[rows][:, cs], ref)
        assert ok, (M, cs, st)


def test_gemm_writes_strided_output_slice(F):
    rng = np.random.default_rng(6)
    M, K, N, bs = 80, 1024, 160, 32
    a, b, s, zp, bias = make(rng, M, K, N, 4, bs, np.float16, "packed", bias=True)
    assert F.select_path(dev(a), dev(b), dev(s), dev(zp), K=K, N=N, block_size=bs) == "gemm"
    big = torch.full((M, 3 * N), 7.0, dtype=torch.float16, device="cuda")
    F.matmul_nbits(dev(a), dev(b), dev(s), dev(zp), dev(bias), K=K, N=N, block_size=bs, out=big[:, N:2 * N])
    torch.cuda.synchronize()
    ref = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=4, block_size=bs)
    out = big.cpu().numpy()
    assert np.all(out[:, :N] == 7.0) and np.all(out[:, 2 * N:] == 7.0)
    assert within_baseline_tol(out[:, N:2 * N], ref)[0]


def test_gemm_unsupported_forms_fall_back_to_generic(F):
    rng = np.random.default_rng(8)
    # K not a multiple of 64; float32 activations; 8-bit codes: the planner keeps the generic kernel
    for (K, dt, bits) in [(96, np.float16, 4), (512, np.float32, 4), (512, np.float16, 8)]:
        a, b, s, zp, _ = make(rng, 32, K, 64, bits, 32, dt, None)
        assert F.select_path(dev(a), dev(b), dev(s), None, K=K, N=64, bits=bits, block_size=32) == "generic"
        with pytest.raises(ValueError):
            F.select_path(dev(a), dev(b), dev(s), None, K=K, N=64, bits=bits, block_size=32, path="gemm")


def test_f16_accumulator_cancellation_gemv(F):
    K, N, bs = 8192, 8, 32
    kb = K // bs
    for M in (1, 8):
        a = np.full((M, K), 8.0, np.float16)
        b = np.full((N, kb, 16), 255, np.uint8)
        s = np.where(np.arange(kb) < kb // 2, 16.0, -16.0).astype(np.float16)[None, :].repeat(N, 0)
        y = run_gpu(F, a, b, s, None, None, K=K, N=N, bits=4, bs=bs, path="auto")
        assert np.all(np.abs(y.astype(np.float32)) <= 0.05)


# ----------------------------------------------------------------- golden fixtures via the operator API
def _request(case):
    from xrgpu_b200.operators import Attributes, Request, Tensor
    order = ("aT", "bT", "scalesT", "zeroPointsT", "biasT")
    inputs = [Tensor.from_numpy(k, case["inputs"][k]) for k in order if k in case["inputs"]]
    return Request(inputs=inputs, attrs=Attributes(integers=dict(case["attrs"])))


def test_golden_fixtures_operator_api(cuda_lib):
    from xrgpu_b200.operators import Operator
    failures = []
    for case in G.load_cases():
        op = Operator.prepare(None, _request(case))
        op.run()
        (y,) = op.read_outputs()
        info = op.info_dict()
        op.close()
        assert info["backend"] == "cuda" and info["cpu_compute_fallback"] is False
        res = G.check_against(y.numpy(), case["expected"], case["atol"], case["rtol"])
        if not res["passed"]:
            failures.append((case["name"], info["path"], res))
        if "published" in case["expected"]:
            assert G.compare(y.numpy(), case["expected"]["published"], case["atol"], case["rtol"])["passed"]
    assert not failures, failures


def test_golden_fixtures_every_applicable_path(F):
    for case in G.load_cases():
        x, at = case["inputs"], case["attrs"]
        K, N, bits, bs = at["K"], at["N"], at.get("bits", 4), at["block_size"]
        args = [dev(x["aT"]), dev(x["bT"]), dev(x["scalesT"]), dev(x.get("zeroPointsT")), dev(x.get("biasT"))]
        for path in ("generic", "gemv", "gemm"):
            try:
                chosen = F.select_path(args[0], args[1], args[2], args[3], K=K, N=N, bits=bits, block_size=bs, path=path)
            except ValueError:
                continue  # path does not support this case
            assert chosen == path
            y = F.matmul_nbits(*args, K=K, N=N, bits=bits, block_size=bs, path=path).cpu().numpy()
            res = G.check_against(y, case["expected"], case["atol"], case["rtol"])
            assert res["passed"], (case["name"], path, res)


# ----------------------------------------------------------------- config 1 at full size
def test_config1_full_size_against_c_oracle(F, oc):
    rng = np.random.default_rng(1)
    M, K, N, bs = 1, 4096, 4096, 32
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.integers(0, 256, (N, K // bs, 16), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, (N, K // bs)).astype(np.float32)
    y = run_gpu(F, a, b, s, None, None, K=K, N=N, bits=4, bs=bs, path="auto")
    ref = oc.matmul(a, b, s, K=K, N=N, bits=4, block_size=bs, threads=8)
    ok, st = within_baseline_tol(y, ref)
    assert ok, st
    assert np.abs(y - ref).max() <= 1e-4 * np.abs(ref).max()

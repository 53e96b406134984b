"""GPU parity at the BASELINE.json configurations' own shapes (configs 3 and 5).

Full-size outputs are checked on a seeded sample of rows and output columns against the oracle
(float64 restatement of complex_kernel.glsl:80,83), under BASELINE.json's tolerances, plus the
size-independent properties: a second call is bit-identical and Y(2A) = 2 Y(A) outside the float16
subnormal range (exact scaling by a power of two).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import mmnb_oracle as O

pytestmark = pytest.mark.gpu

TOL_MAX, TOL_FROB = 1e-2, 2e-3


@pytest.fixture(scope="module")
def F(cuda_lib):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from xrgpu_b200 import functional
    return functional


def _inputs(seed, M, K, N, bs, scale):
    """BASELINE distributions: A ~N(0,1) fp16, random bytes for B, scales ~U(lo, hi) fp16, packed
    zero points with uniform nibbles."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    kb = K // bs
    a = torch.randn((M, K), generator=g, device="cuda").half()
    b = torch.randint(0, 256, (N, kb, bs // 2), dtype=torch.uint8, device="cuda", generator=g)
    s = (torch.rand((N, kb), generator=g, device="cuda") * (scale[1] - scale[0]) + scale[0]).half()
    zp = torch.randint(0, 256, (N, (kb + 1) // 2), dtype=torch.uint8, device="cuda", generator=g)
    return a, b, s, zp


def _check_sample(y, a, b, s, zp, *, K, bs, rows, cols):
    npy = lambda t: t.cpu().numpy()  # noqa: E731
    ref = O.matmul_nbits(npy(a[rows]), npy(b[cols]), npy(s[cols]), npy(zp[cols]), K=K, N=len(cols), bits=4,
                         block_size=bs).astype(np.float64)
    got = y[rows][:, cols].double().cpu().numpy()
    d = got - ref
    rel_max = np.abs(d).max() / np.abs(ref).max()
    frob = np.linalg.norm(d) / np.linalg.norm(ref)
    assert rel_max <= TOL_MAX and frob <= TOL_FROB, (rel_max, frob)


def _properties(F, y, a, b, s, zp, *, K, N, bs):
    y2 = F.matmul_nbits(a, b, s, zp, K=K, N=N, block_size=bs)
    y_2a = F.matmul_nbits(a * 2, b, s, zp, K=K, N=N, block_size=bs)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)                       # deterministic
    normal = y.abs() >= 2.0 ** -13
    assert torch.equal(y_2a[normal], (y * 2)[normal])  # linear (power-of-two scaling is exact)


@pytest.mark.parametrize("M,path", [(4, "gemv"), (16, "gemv"), (64, "gemm")])
def test_config3_batched_decode_full_shape(F, M, path):
    """Config 3: M in {4, 16, 64}, K=4096, N=14336, bs 128, scales ~U(0.002, 0.01), packed zero points."""
    K, N, bs = 4096, 14336, 128
    a, b, s, zp = _inputs(300 + M, M, K, N, bs, (0.002, 0.01))
    assert F.select_path(a, b, s, zp, K=K, N=N, block_size=bs) == path
    y = F.matmul_nbits(a, b, s, zp, K=K, N=N, block_size=bs)
    torch.cuda.synchronize()
    assert F.device_error(0) == 0 and y.shape == (M, N)
    rng = np.random.default_rng(M)
    cols = np.sort(rng.choice(N, 768, replace=False))
    _check_sample(y, a, b, s, zp, K=K, bs=bs, rows=np.arange(M), cols=cols)
    _properties(F, y, a, b, s, zp, K=K, N=N, bs=bs)


# Config 5's per-GPU column shards (1/8 of N) of the 70B-scale projections.
C5_SHARDS = [("up", 8192, 3584), ("down", 28672, 1024), ("lm_head", 8192, 16032)]


@pytest.mark.parametrize("name,K,N", C5_SHARDS)
@pytest.mark.parametrize("M", [1, 4096])
def test_config5_shards_full_shape(F, name, K, N, M):
    """Config 5: bs 32, scales ~U(0.005, 0.02), packed zero points, at M = 1 (GEMV) and M = 4096 (GEMM)."""
    bs = 32
    a, b, s, zp = _inputs(500 + K + N + M, M, K, N, bs, (0.005, 0.02))
    assert F.select_path(a, b, s, zp, K=K, N=N, block_size=bs) == ("gemv" if M == 1 else "gemm")
    y = F.matmul_nbits(a, b, s, zp, K=K, N=N, block_size=bs)
    torch.cuda.synchronize()
    assert F.device_error(0) == 0 and y.shape == (M, N)
    rng = np.random.default_rng(K + N + M)
    rows = np.arange(1) if M == 1 else np.sort(rng.choice(M, 48, replace=False))
    cols = np.sort(rng.choice(N, 512 if M == 1 else 160, replace=False))
    _check_sample(y, a, b, s, zp, K=K, bs=bs, rows=rows, cols=cols)
    _properties(F, y, a, b, s, zp, K=K, N=N, bs=bs)

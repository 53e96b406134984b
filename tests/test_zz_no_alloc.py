"""MatMulNBitsMlp through xrgpu_mlp_forward_static, the entry point that allocates nothing.

Some callers cannot let the library allocate device memory while they run: a serving engine that
plans all of the GPU's memory itself, or a decode loop that must not take cudaMalloc's implicit
synchronisation. xrgpu_mlp_forward_static runs the same kernels as xrgpu_mlp_forward with its scratch
in a fixed 4 MiB array in device memory. This file is collected last (its name sorts after the
others), so a failure here comes after every other test has run; it passes alone in a fresh process
too, because the entry point's first call on a device does its own set-up.

Checked through the C ABI: two calls in a row equal the workspace entry point's result within
BASELINE.json's tolerances (max|dY| <= 1e-2 max|Y_ref|, relative Frobenius <= 2e-3), the residual
output included; a problem whose scratch exceeds the array is rejected as an invalid argument.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _within(got, ref, max_rel=1e-2, frob=2e-3):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = got - ref
    return (got.shape == ref.shape and np.abs(d).max() <= max_rel * max(np.abs(ref).max(), 1e-30)
            and np.linalg.norm(d) <= frob * max(np.linalg.norm(ref), 1e-30))


def _problem(_native, M, K, N, bs, t):
    p = _native.MlpProblem_()
    p.dtype = _native.FLOAT16
    p.activation = _native.ACT_SILU
    p.M, p.K, p.N, p.block_size, p.bits = M, K, N, bs, 4
    p.epsilon = 1e-5
    ptr = lambda x: ctypes.c_void_p(x.data_ptr()) if x is not None else None  # noqa: E731
    p.a, p.skip, p.norm_scale = ptr(t["a"]), ptr(t["skip"]), ptr(t["norm"])
    p.gate_b, p.gate_scales, p.gate_bias = ptr(t["gb"]), ptr(t["gs"]), ptr(t["gbias"])
    p.up_b, p.up_scales, p.up_bias = ptr(t["ub"]), ptr(t["us"]), ptr(t["ubias"])
    p.y, p.residual = ptr(t["y"]), ptr(t["res"])
    return p


def _tensors(M, K, N, bs, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    kb = K // bs
    half = lambda *shape: torch.randn(shape, device="cuda", generator=g).half()  # noqa: E731
    codes = lambda: torch.randint(0, 256, (N, kb, bs // 2), dtype=torch.uint8, device="cuda", generator=g)  # noqa: E731
    scales = lambda: (torch.rand((N, kb), device="cuda", generator=g) * 0.015 + 0.005).half()  # noqa: E731
    return dict(a=half(M, K), skip=half(M, K), norm=(torch.rand(K, device="cuda", generator=g) + 0.5).half(),
                gb=codes(), gs=scales(), gbias=half(N), ub=codes(), us=scales(), ubias=half(N),
                y=torch.empty((M, N), dtype=torch.float16, device="cuda"),
                res=torch.empty((M, K), dtype=torch.float16, device="cuda"))


def test_static_scratch_entry_point_matches_workspace_entry_point(cuda_lib):
    from xrgpu_b200 import _native
    lib = _native.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    M, K, N, bs = 2, 4096, 2048, 32
    t = _tensors(M, K, N, bs, seed=11)

    # the existing entry point with a caller-owned workspace
    p = _problem(_native, M, K, N, bs, t)
    need = ctypes.c_uint64(0)
    _native.check(lib.xrgpu_mlp_workspace_size(ctypes.byref(p), ctypes.byref(need)))
    assert 0 < need.value <= _native.STATIC_SCRATCH_BYTES
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    _native.check(lib.xrgpu_mlp_forward(ctypes.byref(p), ctypes.c_void_p(ws.data_ptr()), need.value, stream))
    torch.cuda.synchronize()
    y_ref, res_ref = t["y"].cpu().numpy().copy(), t["res"].cpu().numpy().copy()

    # the static-scratch entry point, twice in a row (the array keeps the first call's contents)
    for call in range(2):
        t["y"].fill_(float("nan"))
        t["res"].fill_(float("nan"))
        _native.check(lib.xrgpu_mlp_forward_static(ctypes.byref(p), stream))
        torch.cuda.synchronize()
        y, res = t["y"].cpu().numpy(), t["res"].cpu().numpy()
        assert np.isfinite(y).all() and np.isfinite(res).all(), call
        assert _within(y, y_ref), call
        assert _within(res, res_ref, 1e-3, 1e-3), call

    code = ctypes.c_uint32(0)
    _native.check(lib.xrgpu_device_error(0, ctypes.byref(code), 1))
    assert code.value == 0


def test_static_scratch_rejects_problems_larger_than_the_array(cuda_lib):
    from xrgpu_b200 import _native
    lib = _native.load()
    # scratch = (M K + 2 M N) float16 values: 64 x (8192 + 2 x 28672) x 2 bytes, about 8.4 MB > 4 MiB
    M, K, N, bs = 64, 8192, 28672, 32
    small = _tensors(1, 256, 16, bs, seed=3)  # valid device pointers; nothing is launched
    p = _problem(_native, M, K, N, bs, small)
    need = ctypes.c_uint64(0)
    _native.check(lib.xrgpu_mlp_workspace_size(ctypes.byref(p), ctypes.byref(need)))
    assert need.value > _native.STATIC_SCRATCH_BYTES
    st = lib.xrgpu_mlp_forward_static(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == _native.INVALID_ARGUMENT
    assert b"static scratch" in lib.xrgpu_last_error()

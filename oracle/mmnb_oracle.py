"""NumPy restatement of the reference MatMulNBits algorithm (CPU oracle).

TEST INFRASTRUCTURE ONLY: used by ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline legs of ``bench.py`` as the checker. The product path never
imports it.

Semantics restated (paths relative to the xrGPU project root):

* ``kernels/_shared/extended/shaders/complex_kernel.glsl:80`` (``nbitWeight``):
  ``blocks = ceil(K/bs)``, ``blockBytes = ceil(bs*bits/8)``,
  ``element = k % bs``, ``byte = (n*blocks + k/bs)*blockBytes + element*bits/8``,
  ``shift = (element*bits) % 8`` (codes packed low-first),
  ``q = (B[byte] >> shift) & (2^bits - 1)``,
  ``z = zero_points[n*blocks + k/bs]`` read as float, else ``2^(bits-1)``,
  ``w = (float(q) - z) * scales[n*blocks + k/bs]`` in float32.
* ``complex_kernel.glsl:83`` (``packedMatmul``, opcode 1025): rows = numel(A)/K
  (rank-3 A folds its leading axes into rows), ``sum += a*w`` over ascending k
  in float32, then ``sum += bias[n]`` and one store converted to A's dtype.
* ``kernels/_shared/shaders/half.glsl:17-45``: float32 -> float16 storage
  conversion rounds to nearest even, overflows to +-inf. NumPy's
  ``astype(np.float16)`` implements the same IEEE rounding.
* Packed uint8 zero points (the ONNX Runtime form, an extension here: the
  reference contract takes float zero points) are unpacked low-first with row
  stride ``ceil(blocks*bits/8)``, the order the reference already uses for
  packed zero points in ``gatherQuant`` (``complex_kernel.glsl:85``).

Two accumulation modes: ``"float64"`` (vectorised, for all sizes) and
``"float32"`` (serial ascending-k float32 like the shader; small sizes only).
"""
from __future__ import annotations

import numpy as np


def k_blocks(K: int, block_size: int) -> int:
    """``kBlocksExpected`` = ceil(K / block_size) (upstream manifest.json:47)."""
    return (int(K) + int(block_size) - 1) // int(block_size)


def blob_size(block_size: int, bits: int) -> int:
    """``blobSizeExpected`` = ceil(block_size * bits / 8) (upstream manifest.json:48)."""
    return (int(block_size) * int(bits) + 7) // 8


def default_zero_point(bits: int) -> float:
    """``2^(bits-1)``: 2, 8 or 128 (complex_kernel.glsl:80; manifest.json:134)."""
    return float(1 << (int(bits) - 1))


def unpack_codes(b: np.ndarray, K: int, bits: int, block_size: int) -> np.ndarray:
    """Integer codes q[n, k] for k < K, as uint8 [N, K] (complex_kernel.glsl:80)."""
    b = np.ascontiguousarray(b, dtype=np.uint8)
    N = b.shape[0]
    kb, blob = k_blocks(K, block_size), blob_size(block_size, bits)
    if b.shape != (N, kb, blob):
        raise ValueError(f"bT shape {b.shape} != {(N, kb, blob)}")
    k = np.arange(K, dtype=np.int64)
    element = k % block_size
    byte = (k // block_size) * blob + (element * bits) // 8
    shift = ((element * bits) % 8).astype(np.uint8)
    flat = b.reshape(N, kb * blob)
    return (flat[:, byte] >> shift) & np.uint8((1 << bits) - 1)


def unpack_packed_zero_points(zp: np.ndarray, N: int, kb: int, bits: int) -> np.ndarray:
    """Packed uint8 zero points [N, ceil(kb*bits/8)] -> float32 [N, kb].

    Low-first within each byte, the packing ``gatherQuant`` reads
    (complex_kernel.glsl:85). Codes 0..2^bits-1 are exact in float32.
    """
    zp = np.ascontiguousarray(zp, dtype=np.uint8)
    stride = (kb * bits + 7) // 8
    if zp.shape != (N, stride):
        raise ValueError(f"packed zeroPointsT shape {zp.shape} != {(N, stride)}")
    j = np.arange(kb, dtype=np.int64)
    byte = (j * bits) // 8
    shift = ((j * bits) % 8).astype(np.uint8)
    return ((zp[:, byte] >> shift) & np.uint8((1 << bits) - 1)).astype(np.float32)


def zero_point_matrix(zero_points, N: int, kb: int, bits: int) -> np.ndarray:
    """Per-block zero points as float32 [N, kb], whatever form was supplied."""
    if zero_points is None:
        return np.full((N, kb), default_zero_point(bits), dtype=np.float32)
    zp = np.asarray(zero_points)
    if zp.dtype == np.uint8:
        return unpack_packed_zero_points(zp, N, kb, bits)
    if zp.dtype not in (np.float32, np.float16):
        raise ValueError("zero points must be float32/float16 (contract) or packed uint8")
    if zp.shape != (N, kb):
        raise ValueError(f"zeroPointsT shape {zp.shape} != {(N, kb)}")
    return zp.astype(np.float32)


def dequantize(b, scales, zero_points, *, K: int, bits: int, block_size: int) -> np.ndarray:
    """Dequantized weights W[n, k] = (float(q) - z) * s in float32 (complex_kernel.glsl:80).

    Each operation is one IEEE float32 operation (subtract, then multiply),
    so this is bit-exact with the shader's ``nbitWeight``.
    """
    b = np.asarray(b, dtype=np.uint8)
    N = b.shape[0]
    kb = k_blocks(K, block_size)
    s = np.asarray(scales)
    if s.shape != (N, kb):
        raise ValueError(f"scalesT shape {s.shape} != {(N, kb)}")
    q = unpack_codes(b, K, bits, block_size).astype(np.float32)
    z = zero_point_matrix(zero_points, N, kb, bits)
    block = np.arange(K) // block_size
    with np.errstate(all="ignore"):
        return (q - z[:, block]) * s.astype(np.float32)[:, block]


def output_shape(a_shape, N: int):
    """``shapes.aT[:-1] + [N]`` (complex_plan.cpp:120; contract.json:95-101)."""
    return tuple(a_shape[:-1]) + (int(N),)


def matmul_nbits(a, b, scales, zero_points=None, bias=None, *, K: int, N: int,
                 bits: int = 4, block_size: int, accumulate: str = "float64",
                 columns: slice | None = None) -> np.ndarray:
    """Y = A @ dequant(B)^T (+ bias), returned in A's dtype (complex_kernel.glsl:83).

    ``columns`` restricts the computation to a slice of output columns (used
    to time or check a bounded sample of a large problem).
    """
    a = np.asarray(a)
    if a.dtype not in (np.float32, np.float16):
        raise ValueError("aT must be float32 or float16")
    if a.shape[-1] != K:
        raise ValueError("last axis of aT must equal K")
    rows = int(np.prod(a.shape[:-1], dtype=np.int64))
    cols = range(N)[columns] if columns is not None else range(N)
    c0, c1 = cols.start, cols.stop
    b_sel = np.asarray(b)[c0:c1]
    s_sel = np.asarray(scales)[c0:c1]
    zp_sel = None if zero_points is None else np.asarray(zero_points)[c0:c1]
    w = dequantize(b_sel, s_sel, zp_sel, K=K, bits=bits, block_size=block_size)
    x = a.reshape(rows, K)
    if accumulate == "float64":
        y = x.astype(np.float64) @ w.astype(np.float64).T
        if bias is not None:
            y = y + np.asarray(bias)[c0:c1].astype(np.float64)
        y = y.astype(np.float32)
    elif accumulate == "float32":
        xf = x.astype(np.float32)
        y = np.zeros((rows, c1 - c0), dtype=np.float32)
        with np.errstate(all="ignore"):
            for k in range(K):  # serial ascending k, one float32 multiply-add each
                y += xf[:, k:k + 1] * w[:, k][None, :]
            if bias is not None:
                y += np.asarray(bias)[c0:c1].astype(np.float32)[None, :]
    else:
        raise ValueError("accumulate must be 'float64' or 'float32'")
    with np.errstate(all="ignore"):
        y = y.astype(a.dtype)
    return y.reshape(tuple(a.shape[:-1]) + (c1 - c0,))


def algorithmic_bytes(M: int, K: int, N: int, bits: int, block_size: int, act_bytes: int,
                      zp_kind: str | None, has_bias: bool) -> int:
    """Bytes one call must move: B + scales + zero points + A + Y (+ bias)."""
    kb = k_blocks(K, block_size)
    total = N * kb * blob_size(block_size, bits) + N * kb * act_bytes
    if zp_kind == "packed":
        total += N * ((kb * bits + 7) // 8)
    elif zp_kind in ("float16", "float32"):
        total += N * kb * (2 if zp_kind == "float16" else 4)
    total += M * K * act_bytes + M * N * act_bytes
    if has_bias:
        total += N * act_bytes
    return int(total)


def quantize_reference_weights(w: np.ndarray, *, bits: int, block_size: int, rng=None):
    """Helper for tests: pack an integer code matrix [N, K] into the bT layout."""
    w = np.asarray(w, dtype=np.uint8)
    N, K = w.shape
    kb, blob = k_blocks(K, block_size), blob_size(block_size, bits)
    out = np.zeros((N, kb * blob), dtype=np.uint8)
    k = np.arange(K)
    element = k % block_size
    byte = (k // block_size) * blob + (element * bits) // 8
    shift = ((element * bits) % 8).astype(np.uint8)
    for j in range(K):
        out[:, byte[j]] |= (w[:, j] & ((1 << bits) - 1)) << shift[j]
    return out.reshape(N, kb, blob)

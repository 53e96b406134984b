"""NumPy restatement of the reference's MatMulNBits family operators (CPU oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/`` (and ``bench.py``'s CPU-baseline leg) as the
checker; the product path never imports it.

Operators and the reference code each function restates (paths relative to the xrGPU project
root; ``K`` = ``complex_kernel.glsl`` = kernels/_shared/extended/shaders/complex_kernel.glsl):

* ``fused_activation``         -- ``fused`` (K:41-47) with the codes of ``activation_lower``
  (kernels/_shared/extended/complex_plan.cpp:50): 0 identity, 1 relu, 2 silu, 3 gelu (erf form for
  opcode 1027, tanh form otherwise), 4 tanh, 5 sigmoid, 6 swiglu (identity inside ``fused``).
* ``packed_input``             -- ``packedInput`` (K:81) and the residual store of ``packedMatmul``
  (K:83): h = a + skip; with a norm scale, x = h * (1/sqrt(sum(h^2)/K + eps) * normScale[k]).
* ``matmul_nbits_mlp`` (1027)  -- ``packedMatmul`` (K:83): y = fused(gate.x + gateBias) * (up.x + upBias),
  gate/up weights from ``nbitWeight`` without zero points (z = 2^(bits-1), K:80).
* ``matmul_nbits_qkv`` (1028)  -- ``packedMatmul`` (K:83): q/k/v = x.W^T, always normalised.
* ``matmul_bnb4`` (1026)       -- ``bnbWeight`` (K:82): NF4/FP4 codebooks, high nibble first,
  absmax per block of ``block_size`` flat weight indices.
* ``gather_block_quantized`` (1031) -- ``gatherQuant`` (K:85): out-of-range indices fail with
  code 55 and leave their row zero.
* ``qmoe`` (1030)              -- ``moe``/``expertRank``/``expertWeight`` (K:158-160): top-k by the
  rank rule (ties go to the higher expert index), softmax over the selected experts, symmetric
  int4/int8 expert weights with per-row or per-block scales, relu or (clamped) swiglu.

Accumulation is float64 (vectorised); results are returned in the reference's output dtypes.
"""
from __future__ import annotations

import math

import numpy as np

from .mmnb_oracle import dequantize, k_blocks

ACTIVATIONS = {"none": 0, "": 0, "identity": 0, "relu": 1, "silu": 2, "swish": 2, "gelu": 3, "tanh": 4,
               "sigmoid": 5, "swiglu": 6}

# bnbWeight's codebooks (complex_kernel.glsl:82): NF4 (quant_type 1) and FP4 (quant_type 0).
NF4 = np.array([-1.0, -0.6961928009986877, -0.5250730514526367, -0.3949174880981445, -0.28444138169288635,
                -0.18477343022823334, -0.09105003625154495, 0.0, 0.07958029955625534, 0.16093020141124725,
                0.24611230194568634, 0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
                0.7229568362236023, 1.0], dtype=np.float32)
FP4 = np.array([0.0, 0.0052083333333333, 0.6666666666666666, 1.0, 0.3333333333333333, 0.5, 0.1666666666666666,
                0.25, -0.0, -0.0052083333333333, -0.6666666666666666, -1.0, -0.3333333333333333, -0.5,
                -0.1666666666666666, -0.25], dtype=np.float32)


def activation_code(name) -> int:
    if isinstance(name, (int, np.integer)):
        return int(name)
    if name not in ACTIVATIONS:
        raise ValueError(f"Unknown fused activation: {name}")
    return ACTIVATIONS[name]


def _logistic(x):
    return 1.0 / (1.0 + np.exp(-x))


def fused_activation(x, kind: int, gelu_erf: bool = True):
    """``fused`` (complex_kernel.glsl:41-47) in float64."""
    x = np.asarray(x, np.float64)
    with np.errstate(all="ignore"):
        if kind == 1:
            return np.maximum(x, 0.0)
        if kind == 2:
            return x * _logistic(x)
        if kind == 3:
            if gelu_erf:
                return 0.5 * x * (1.0 + np.vectorize(math.erf)(x * 0.7071067811865475))
            return 0.5 * x * (1.0 + np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3)))
        if kind == 4:
            return np.tanh(x)
        if kind == 5:
            return _logistic(x)
    return x


def packed_input(a, skip=None, norm_scale=None, *, K: int, epsilon: float):
    """(x, residual) of ``packedInput`` with normalisation on (complex_kernel.glsl:81,83), float64."""
    a = np.asarray(a)
    rows = int(np.prod(a.shape[:-1], dtype=np.int64))
    h = a.reshape(rows, K).astype(np.float32).astype(np.float64)
    if skip is not None:
        h = (h + np.asarray(skip).reshape(rows, K).astype(np.float64)).astype(np.float32).astype(np.float64)
    residual = h.copy()
    if norm_scale is not None:
        inv = 1.0 / np.sqrt(np.sum(h * h, axis=1, keepdims=True) / K + np.float32(epsilon))
        h = h * inv * np.asarray(norm_scale).astype(np.float64)[None, :]
    return h, residual


def _project(x, b, scales, *, K, N, bits, block_size, bias=None):
    w = dequantize(b, scales, None, K=K, bits=bits, block_size=block_size).astype(np.float64)
    y = x @ w.T
    if bias is not None:
        y = y + np.asarray(bias).astype(np.float64)[None, :]
    return y


def matmul_nbits_mlp(a, skip, norm_scale, gate_b, gate_scales, gate_bias, up_b, up_scales, up_bias, *, K: int,
                     N: int, bits: int = 4, block_size: int, activation="silu", epsilon: float = 1e-5):
    """(yT, residualT) of opcode 1027; normalisation applies only when normScaleT is given."""
    a = np.asarray(a)
    x, residual = packed_input(a, skip, norm_scale, K=K, epsilon=epsilon)
    g = _project(x, gate_b, gate_scales, K=K, N=N, bits=bits, block_size=block_size, bias=gate_bias)
    u = _project(x, up_b, up_scales, K=K, N=N, bits=bits, block_size=block_size, bias=up_bias)
    y = fused_activation(g, activation_code(activation), gelu_erf=True) * u
    lead = tuple(a.shape[:-1])
    with np.errstate(all="ignore"):
        return y.astype(a.dtype).reshape(lead + (N,)), residual.astype(a.dtype).reshape(a.shape)


def matmul_nbits_qkv(a, skip, norm_scale, q_b, q_scales, k_b, k_scales, v_b, v_scales, *, K: int, Nq: int,
                     Nkv: int, bits: int = 4, block_size: int, epsilon: float = 1e-6):
    """(qT, kT, vT, residualT) of opcode 1028 (always normalised)."""
    a = np.asarray(a)
    x, residual = packed_input(a, skip, norm_scale, K=K, epsilon=epsilon)
    lead = tuple(a.shape[:-1])
    outs = []
    for b, s, n in ((q_b, q_scales, Nq), (k_b, k_scales, Nkv), (v_b, v_scales, Nkv)):
        y = _project(x, b, s, K=K, N=n, bits=bits, block_size=block_size)
        with np.errstate(all="ignore"):
            outs.append(y.astype(a.dtype).reshape(lead + (n,)))
    return (*outs, residual.astype(a.dtype).reshape(a.shape))


def bnb_weights(b, absmax, *, K: int, N: int, block_size: int, quant_type: int, transB: int = 1):
    """W[n, k] of ``bnbWeight`` (complex_kernel.glsl:82) as float32 [N, K]."""
    b = np.asarray(b, np.uint8).reshape(-1)
    n = np.arange(N, dtype=np.int64)[:, None]
    k = np.arange(K, dtype=np.int64)[None, :]
    idx = n * K + k if transB else k * N + n
    byte = b[idx // 2]
    code = np.where(idx % 2 == 0, byte >> 4, byte & 15)
    table = NF4 if quant_type == 1 else FP4
    return table[code] * np.asarray(absmax).astype(np.float32)[idx // block_size]


def matmul_bnb4(a, b, absmax, *, K: int, N: int, block_size: int, quant_type: int, transB: int = 1):
    a = np.asarray(a)
    w = bnb_weights(b, absmax, K=K, N=N, block_size=block_size, quant_type=quant_type, transB=transB)
    y = a.reshape(-1, K).astype(np.float64) @ w.astype(np.float64).T
    with np.errstate(all="ignore"):
        return y.astype(a.dtype).reshape(tuple(a.shape[:-1]) + (N,))


def gather_block_quantized(data, indices, scales, zero_points=None, *, bits: int = 4, block_size: int = 128):
    """(outputT float32 [len(indices), width], failed) of ``gatherQuant`` (complex_kernel.glsl:85).
    ``failed`` is True when some index was out of range (the reference's fail(55)); those rows stay 0."""
    data = np.asarray(data, np.uint8)
    rows, row_bytes = data.shape
    width = row_bytes * (8 // bits)
    blocks = (width + block_size - 1) // block_size
    zrow = (blocks * bits + 7) // 8
    idx = np.asarray(indices).astype(np.int64).reshape(-1)
    out = np.zeros((idx.size, width), np.float32)
    j = np.arange(width)
    mask = (1 << bits) - 1
    sc = np.asarray(scales, np.float32).reshape(-1)
    zp = None if zero_points is None else np.asarray(zero_points, np.uint8).reshape(-1)
    failed = False
    for r, sel in enumerate(idx):
        sel = int(np.clip(sel, -2 ** 31, 2 ** 31 - 1))  # controlIndex saturates int64 to int32
        if sel < 0 or sel >= rows:
            failed = True
            continue
        q = (data[sel, (j * bits) // 8] >> ((j * bits) % 8)) & mask
        blk = j // block_size
        if zp is not None:
            z = (zp[sel * zrow + (blk * bits) // 8] >> ((blk * bits) % 8)) & mask
        else:
            z = np.full(width, 1 << (bits - 1))
        out[r] = (q.astype(np.float32) - z.astype(np.float32)) * sc[sel * blocks + blk]
    return out, failed


def _expert_weights(w, scales, *, bits: int, block_size: int):
    """``expertWeight`` for opcode 1030: symmetric codes (q - 2^(bits-1)) times per-row or per-block
    scales, as float64 [experts, rows, cols]."""
    w = np.asarray(w, np.uint8)
    E, R, packed = w.shape
    cols = packed * (8 // bits)
    c = np.arange(cols)
    q = (w[:, :, (c * bits) // 8] >> ((c * bits) % 8)) & ((1 << bits) - 1)
    value = q.astype(np.float64) - (1 << (bits - 1))
    if value.size == 0:  # an empty expert projection (zero rows or columns)
        return value
    s = np.asarray(scales, np.float64).reshape(E, R, -1)
    per_row = s.shape[2]
    sidx = c // max(1, block_size) if per_row > 1 else np.zeros(cols, np.int64)
    return value * s[:, :, sidx]


def qmoe(x, router, fc1, fc1_scales, fc2, fc2_scales, *, k: int = 1, bits: int = 4, block_size: int = 0,
         activation="relu", swiglu_fusion: int = 0, activation_alpha: float = 1.0, activation_beta: float = 0.0,
         swiglu_limit=None):
    """outputT of opcode 1030 (``moe``, complex_kernel.glsl:160), float32 of x's shape."""
    x = np.asarray(x, np.float32)
    hidden = x.shape[-1]
    xs = x.reshape(-1, hidden).astype(np.float64)
    logits = np.asarray(router, np.float32).astype(np.float64)
    E = logits.shape[1]
    act = activation_code(activation)
    w1 = _expert_weights(fc1, fc1_scales, bits=bits, block_size=block_size)
    w2 = _expert_weights(fc2, fc2_scales, bits=bits, block_size=block_size)
    fc1_rows = w1.shape[1]
    fusion = 2 if (act == 6 and swiglu_fusion) else 1
    inter = fc1_rows // fusion
    out = np.zeros_like(xs)
    for t in range(xs.shape[0]):
        s = logits[t]
        rank = np.array([np.sum((s > s[e]) | ((s == s[e]) & (np.arange(E) > e))) for e in range(E)])
        chosen = np.nonzero(rank < k)[0]
        if chosen.size == 0:
            continue
        m = s[chosen].max()
        weights = np.exp(s[chosen] - m)
        weights /= weights.sum()
        for e, we in zip(chosen, weights):
            j = np.arange(inter)
            gate_rows = 2 * j if (act == 6 and swiglu_fusion == 1) else j
            lin_rows = 2 * j + 1 if swiglu_fusion == 1 else inter + j
            gate = w1[e, gate_rows] @ xs[t]
            if act == 6:
                linear = w1[e, lin_rows] @ xs[t] if swiglu_fusion else np.zeros(inter)
                if swiglu_limit is not None:
                    gate = np.minimum(gate, swiglu_limit)
                    linear = np.clip(linear, -swiglu_limit, swiglu_limit)
                a = gate * _logistic(activation_alpha * gate) * (linear + activation_beta)
            else:
                a = fused_activation(gate, act, gelu_erf=False)
            out[t] += we * (w2[e] @ a)
    return out.astype(np.float32).reshape(x.shape)


def k_blocks_of(K: int, block_size: int) -> int:
    return k_blocks(K, block_size)

"""Pins the CPU oracle (NumPy + C restatements) against the reference.

Sources of truth, in order:
  * the reference suite's known answers (upstream test.json: q4_block512 = 128 exactly, the
    empty-M cases, the float16 accumulator-cancellation cases whose exact result is 0);
  * the reference's own algorithm compiled from its sources (oracle/_ref/libmmnb_ref.so);
  * the committed golden fixtures (tests/golden), produced by that compiled reference.
"""
import numpy as np
import pytest

from oracle import mmnb_oracle as O
from oracle.native import OracleC, ReferenceC, reference_available

import fixtures as G


@pytest.fixture(scope="module")
def oc():
    return OracleC()


@pytest.fixture(scope="module")
def rc():
    if not reference_available():
        pytest.skip("oracle/_ref not built (needs the reference checkout once)")
    return ReferenceC()


def random_problem(rng, M, K, N, bits, bs, dt, zp_kind, bias=True):
    kb, blob = O.k_blocks(K, bs), O.blob_size(bs, bits)
    a = rng.standard_normal((M, K)).astype(dt)
    b = rng.integers(0, 256, (N, kb, blob), dtype=np.uint8)
    s = rng.uniform(0.005, 0.02, (N, kb)).astype(dt)
    if zp_kind is None:
        zp = None
    elif zp_kind == "packed":
        zp = rng.integers(0, 256, (N, (kb * bits + 7) // 8), dtype=np.uint8)
    else:
        zp = rng.integers(0, 1 << bits, (N, kb)).astype(zp_kind)
    bb = rng.standard_normal(N).astype(dt) if bias else None
    return a, b, s, zp, bb


def test_known_answer_block512_is_128(oc):
    # upstream test.json case q4_block512_schema_legal_cpu_provider_gap_exact: A = 1, code 9
    # (byte 153 = 0x99), default zero point 8, scale 0.25 -> 512 * 1 * 0.25 = 128 exactly.
    a = np.ones((1, 512), np.float32)
    b = np.full((1, 1, 256), 153, np.uint8)
    s = np.full((1, 1), 0.25, np.float32)
    assert O.matmul_nbits(a, b, s, K=512, N=1, block_size=512)[0, 0] == 128.0
    assert oc.matmul(a, b, s, K=512, N=1, block_size=512)[0, 0] == 128.0


@pytest.mark.parametrize("dt", [np.float32, np.float16])
def test_empty_rows(dt, oc):
    a = np.zeros((0, 32), dt)
    b = np.full((4, 1, 16), 17, np.uint8)
    s = np.full((4, 1), 0.05, dt)
    y = O.matmul_nbits(a, b, s, K=32, N=4, block_size=32)
    assert y.shape == (0, 4) and y.dtype == dt
    assert oc.matmul(a, b, s, K=32, N=4, block_size=32).shape == (0, 4)


@pytest.mark.parametrize("M,K", [(1, 8192), (8, 8192), (64, 4096)])
def test_f16_accumulator_cancellation_is_zero(M, K, oc):
    # ORT MatMulNBits.Float16_LargeK_AccumulatorOverflow as frozen upstream: A = 8, every code 15,
    # scales +16 over the first half of K and -16 over the second -> exact result 0 (tol 0.05).
    N, bs = 8, 32
    kb = K // bs
    a = np.full((M, K), 8.0, np.float16)
    b = np.full((N, kb, 16), 255, np.uint8)
    s = np.where(np.arange(kb) < kb // 2, 16.0, -16.0).astype(np.float16)[None, :].repeat(N, 0)
    for y in (O.matmul_nbits(a, b, s, K=K, N=N, block_size=bs),
              O.matmul_nbits(a, b, s, K=K, N=N, block_size=bs, accumulate="float32"),
              oc.matmul(a, b, s, K=K, N=N, block_size=bs)):
        assert np.all(np.abs(y.astype(np.float32)) <= 0.05)


@pytest.mark.parametrize("dt", [np.float32, np.float16])
@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("zp_kind", [None, "float", "packed"])
def test_restatements_agree_with_compiled_reference(dt, bits, zp_kind, oc, rc):
    rng = np.random.default_rng(bits * 31 + (zp_kind is None) + 7 * (dt == np.float16))
    for (M, K, N, bs) in [(3, 77, 19, 16), (2, 64, 5, 32), (1, 300, 9, 128), (4, 33, 6, 32)]:
        zk = dt if zp_kind == "float" else zp_kind
        a, b, s, zp, bias = random_problem(rng, M, K, N, bits, bs, dt, zk)
        y_c = oc.matmul(a, b, s, zp, bias, K=K, N=N, bits=bits, block_size=bs, threads=2)
        y32 = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=bits, block_size=bs, accumulate="float32")
        assert np.array_equal(y_c.view(np.uint8), y32.view(np.uint8))
        if zp_kind != "packed":  # the reference contract takes float zero points only
            y_r = rc.matmul(a, b, s, zp, bias, K=K, N=N, bits=bits, block_size=bs, threads=3)
            assert np.array_equal(y_c.view(np.uint8), y_r.view(np.uint8))
        w_np = O.dequantize(b, s, zp, K=K, bits=bits, block_size=bs)
        w_c = oc.dequantize(b, s, zp, K=K, N=N, bits=bits, block_size=bs)
        assert np.array_equal(w_np.view(np.uint32), w_c.view(np.uint32))
        y64 = O.matmul_nbits(a, b, s, zp, bias, K=K, N=N, bits=bits, block_size=bs)
        ref = y_c.astype(np.float64)
        assert np.abs(y64.astype(np.float64) - ref).max() <= 1e-2 * max(1e-6, np.abs(ref).max())


def test_packed_zero_points_equal_float_form():
    rng = np.random.default_rng(3)
    for bits in (2, 4, 8):
        N, kb = 7, 13
        codes = rng.integers(0, 1 << bits, (N, kb))
        packed = np.zeros((N, (kb * bits + 7) // 8), np.uint8)
        for j in range(kb):
            packed[:, (j * bits) // 8] |= (codes[:, j] << ((j * bits) % 8)).astype(np.uint8)
        assert np.array_equal(O.unpack_packed_zero_points(packed, N, kb, bits), codes.astype(np.float32))


def test_half_decode_all_patterns_match_reference(oc, rc):
    bits = np.arange(65536, dtype=np.uint16)
    mine = oc.f16_bits_to_f32(bits).view(np.uint32)
    ref = np.array([rc.lib.mmnb_ref_half_to_float_bits(int(h)) for h in bits], dtype=np.uint32)
    assert np.array_equal(mine, ref)
    with np.errstate(all="ignore"):
        npv = bits.view(np.float16).astype(np.float32).view(np.uint32)
    finite = ~np.isnan(bits.view(np.float16))
    assert np.array_equal(mine[finite], npv[finite])


def test_half_encode_rounding_boundaries_match_reference(oc, rc):
    # Every half value, its midpoints to both neighbours, one ulp around them, overflow/underflow.
    h = np.arange(0x7c00, dtype=np.uint16).view(np.float16).astype(np.float64)
    nxt = np.append(h[1:], 65520.0)
    mids = (h + nxt) / 2
    cand = np.concatenate([h, mids, np.nextafter(mids.astype(np.float32), np.float32(np.inf)).astype(np.float64),
                           np.nextafter(mids.astype(np.float32), np.float32(-np.inf)).astype(np.float64),
                           [65519.0, 65520.0, 1e6, 1e-9, 2.0 ** -25, 3 * 2.0 ** -26]])
    f = np.concatenate([cand, -cand]).astype(np.float32)
    f = np.concatenate([f, np.array([np.inf, -np.inf, np.nan], np.float32)])
    mine = oc.f32_to_f16_bits(f)
    ref = np.array([rc.lib.mmnb_ref_float_bits_to_half(int(x)) for x in f.view(np.uint32)], dtype=np.uint16)
    assert np.array_equal(mine, ref)
    with np.errstate(all="ignore"):
        npv = f.astype(np.float16).view(np.uint16)
    ok = ~np.isnan(f)
    assert np.array_equal(mine[ok], npv[ok])


def test_golden_fixtures_reproduced_by_c_oracle(oc):
    cases = G.load_cases()
    assert len(cases) == 86
    for case in cases:
        x = case["inputs"]
        at = case["attrs"]
        y = oc.matmul(x["aT"], x["bT"], x["scalesT"], x.get("zeroPointsT"), x.get("biasT"), K=at["K"], N=at["N"],
                      bits=at.get("bits", 4), block_size=at["block_size"], threads=4)
        exp = case["expected"]
        if exp["mode"] == "full":
            assert np.array_equal(y.view(np.uint8), exp["y"].view(np.uint8)), case["name"]
        else:
            assert np.array_equal(y.reshape(-1)[exp["index"]].view(np.uint8), exp["values"].view(np.uint8)), case["name"]
        if "published" in exp:
            assert G.compare(y, exp["published"], case["atol"], case["rtol"])["passed"], case["name"]


def test_golden_fixtures_within_tolerance_of_numpy_oracle():
    for case in G.load_cases():
        x = case["inputs"]
        at = case["attrs"]
        y = O.matmul_nbits(x["aT"], x["bT"], x["scalesT"], x.get("zeroPointsT"), x.get("biasT"), K=at["K"], N=at["N"],
                           bits=at.get("bits", 4), block_size=at["block_size"])
        res = G.check_against(y, case["expected"], max(case["atol"], 1e-5), max(case["rtol"], 1e-3))
        assert res["passed"], (case["name"], res)

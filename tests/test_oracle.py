"""CPU checks of the oracle against the reference's own pins (no GPU).

- decode of every code against the reference's named constants (src/data_types/float8.rs,
  float4.rs, via tests/golden/format_constants.json);
- the soft decode restates minifloat_to_f32 (src/data_types/vector.rs:61-95);
- encode rounding: hand-computed ties and .satfinite boundaries, a second independent (float64)
  formulation of RN, decode->encode round trips;
- the hardware pin: digests of the B200's own `cvt` outputs over all 2^32 f32 patterns
  (tests/golden/cvt_sweep_digests.json, written by tests/golden/make_cvt_digests.py on a B200).
"""

import json
import math
import os

import numpy as np
import pytest

from conftest import GOLDEN

FMT_IDS = {"f8e4m3": 0, "f8e5m2": 1, "f4e2m1": 2, "f6e2m3": 3, "f6e3m2": 4}
NCODES = {0: 256, 1: 256, 2: 16, 3: 64, 4: 64}


def _value(s: str) -> float:
    if s == "nan":
        return math.nan
    if "^" in s:
        b, e = s.split("^")
        return float(b) ** int(e)
    return float(s)


def test_constants_decode(oracle):
    consts = json.load(open(os.path.join(GOLDEN, "format_constants.json")))
    L = oracle.lib()
    n = 0
    for fmt, items in consts.items():
        for c in items:
            want = _value(c["value"])
            if fmt == "f8e8m0":
                got = L.ptxo_ue8m0_to_f32(c["code"])
            else:
                got = L.ptxo_to_f32_via_half(FMT_IDS[fmt], c["code"])
            if math.isnan(want):
                assert math.isnan(got), (fmt, c)
            else:
                assert got == want and math.copysign(1, got) == math.copysign(1, want), (fmt, c)
            n += 1
    assert n == 48


def _minifloat_ref(bits, e, m, bias, specials):
    """A second, independent decode formulation (integer significand times a power of two)."""
    neg = (bits >> (e + m)) & 1
    ex = (bits >> m) & ((1 << e) - 1)
    mn = bits & ((1 << m) - 1)
    if ex == (1 << e) - 1 and (specials == 1 or (specials == 2 and mn == (1 << m) - 1)):
        v = math.inf if (specials == 1 and mn == 0) else math.nan
    elif ex == 0:
        v = mn * 2.0 ** (1 - bias - m)
    else:
        v = ((1 << m) + mn) * 2.0 ** (ex - bias - m)
    return -v if neg else v


@pytest.mark.parametrize("fmt,e,m,bias,sp,n", [(0, 4, 3, 7, 2, 256), (1, 5, 2, 15, 1, 256),
                                               (2, 2, 1, 1, 0, 16), (3, 2, 3, 1, 0, 64),
                                               (4, 3, 2, 3, 0, 64)])
def test_decode_all_codes(oracle, fmt, e, m, bias, sp, n):
    L = oracle.lib()
    for c in range(n):
        got = L.ptxo_minifloat_to_f32(c, e, m, bias, sp)
        want = _minifloat_ref(c, e, m, bias, sp)
        if math.isnan(want):
            assert math.isnan(got)
        else:
            assert got == want and math.copysign(1, got) == math.copysign(1, want), (fmt, c)


def test_ue8m0_decode(oracle):
    L = oracle.lib()
    for c in range(255):
        assert L.ptxo_ue8m0_to_f32(c) == 2.0 ** (c - 127)
    assert math.isnan(L.ptxo_ue8m0_to_f32(255))


def _rn_slow(x: float, e: int, m: int, bias: int, max_mag: float) -> float:
    """RN-even with .satfinite in float64: the quantum of x's binade (or of the subnormal range),
    Python's round() is ties-to-even."""
    if x == 0:
        return 0.0
    a = abs(x)
    emin = 1 - bias
    te = max(math.floor(math.log2(a)), emin)
    # floor(log2) can be off by one at exact powers of two in float; fix it exactly.
    while 2.0 ** te > a and te > emin:
        te -= 1
    while 2.0 ** (te + 1) <= a:
        te += 1
    q = 2.0 ** (te - m)
    r = round(a / q) * q
    r = min(r, max_mag)
    return math.copysign(r, x)


@pytest.mark.parametrize("fmt,e,m,bias,max_mag", [(0, 4, 3, 7, 448.0), (1, 5, 2, 15, 57344.0),
                                                  (2, 2, 1, 1, 6.0), (3, 2, 3, 1, 7.5),
                                                  (4, 3, 2, 3, 28.0)])
def test_encode_matches_float64_formulation(oracle, fmt, e, m, bias, max_mag):
    rng = np.random.default_rng(1234 + fmt)
    x = (rng.standard_normal(20000) * np.exp2(rng.uniform(-20, 20, 20000))).astype(np.float32)
    # exact ties at every binade: midpoints between adjacent representable values
    reps = sorted({abs(oracle.lib().ptxo_to_f32_via_half(fmt, c))
                   for c in range(NCODES[fmt])} - {math.inf})
    reps = [r for r in reps if not math.isnan(r)]
    mids = [(a + b) / 2 for a, b in zip(reps, reps[1:])]
    x = np.concatenate([x, np.array(mids + [-v for v in mids], dtype=np.float32)])
    L = oracle.lib()
    for v in x.tolist():
        code = L.ptxo_f32_to_narrow(fmt, v, 0)
        got = L.ptxo_to_f32_via_half(fmt, code)
        want = _rn_slow(v, e, m, bias, max_mag)
        assert got == want and math.copysign(1, got) == math.copysign(1, want), (fmt, v, code)


def test_encode_boundaries(oracle):
    L = oracle.lib()
    e4 = lambda v, r=0: L.ptxo_f32_to_e4m3(v, r)  # noqa: E731
    e5 = lambda v, r=0: L.ptxo_f32_to_e5m2(v, r)  # noqa: E731
    e2 = lambda v, r=0: L.ptxo_f32_to_e2m1(v, r)  # noqa: E731
    # E4M3: 448 max; 464 is the tie with the would-be 480 (odd mantissa) -> 448; beyond saturates
    assert [e4(v) for v in (448.0, 464.0, 480.0, 1e30, math.inf)] == [0x7E] * 5
    assert e4(-math.inf) == 0xFE and e4(math.nan) == 0x7F
    assert e4(2.0 ** -9) == 0x01 and e4(2.0 ** -10) == 0x00 and e4(1.5 * 2.0 ** -10) == 0x01
    # E5M2: 57344 max, 61440 tie -> 65536 would overflow -> clamps
    assert [e5(v) for v in (57344.0, 61439.0, 61440.0, math.inf)] == [0x7B] * 4
    assert e5(2.0 ** -16) == 0x01 and e5(2.0 ** -17) == 0x00
    # E2M1: ties to even (0.25 -> 0, 0.75 -> 1.0, 2.5 -> 2, 5 -> 4), 6 max, NaN -> +6
    assert [e2(v) for v in (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 7.0, 1e9)] == \
        [0x0, 0x2, 0x2, 0x4, 0x4, 0x6, 0x6, 0x7, 0x7]
    assert e2(math.nan) == 0x7 and e2(-math.inf) == 0xF and e2(-0.0) == 0x8
    # .relu clamps negative results to +0, NaN stays NaN for FP8
    assert e4(-1.0, 1) == 0 and e4(1.0, 1) == 0x38 and e4(math.nan, 1) == 0x7F
    assert e2(-3.0, 1) == 0
    # FP6 (src/data_types/float6.rs): E2M3 max 7.5, E3M2 max 28, sign bit 0x20, no NaN (-> +max)
    f6 = lambda fmt, v, r=0: L.ptxo_f32_to_narrow(fmt, v, r)  # noqa: E731
    assert [f6(3, v) for v in (7.5, 7.75, 8.0, 1e9, math.inf)] == [0x1F] * 5
    assert f6(3, 1.0) == 0x08 and f6(3, 0.125) == 0x01 and f6(3, 0.0625) == 0x00
    assert f6(3, 0.1875) == 0x02 and f6(3, -math.inf) == 0x3F and f6(3, math.nan) == 0x1F
    assert [f6(4, v) for v in (28.0, 30.0, 32.0, math.inf)] == [0x1F] * 4
    assert f6(4, 1.0) == 0x0C and f6(4, 0.0625) == 0x01 and f6(4, 0.25) == 0x04
    assert f6(4, -0.0) == 0x20 and f6(4, -2.0, 1) == 0 and f6(3, -0.5, 1) == 0


def test_ue8m0_encode(oracle):
    L = oracle.lib()
    u = L.ptxo_f32_to_ue8m0
    assert u(1.0, 0, 1) == 127 and u(1.0, 1, 1) == 127
    assert u(1.5, 0, 1) == 127 and u(1.5, 1, 1) == 128
    assert u(3.0e38, 0, 1) == 254 and u(3.0e38, 1, 1) == 254  # 2^128 overflow -> satfinite
    assert u(math.inf, 0, 1) == 254 and u(math.inf, 0, 0) == 255
    assert u(math.nan, 0, 1) == 255
    assert u(0.0, 0, 1) == 0


def test_roundtrip_codes(oracle):
    """decode -> encode is the identity on every finite code (both signs of zero included)."""
    L = oracle.lib()
    for fmt, n in NCODES.items():
        for c in range(n):
            f = L.ptxo_to_f32_via_half(fmt, c)
            if math.isnan(f) or math.isinf(f):
                continue
            assert L.ptxo_f32_to_narrow(fmt, f, 0) == c


def test_bulk_matches_scalar(oracle):
    rng = np.random.default_rng(7)
    x = (rng.standard_normal(1 << 16) * 8).astype(np.float32)
    for fmt in (0, 1, 2, 3, 4):
        codes = oracle.encode(fmt, x)
        L = oracle.lib()
        if fmt == 2:
            lo = np.array([L.ptxo_f32_to_e2m1(v, 0) for v in x[0::2].tolist()], dtype=np.uint8)
            hi = np.array([L.ptxo_f32_to_e2m1(v, 0) for v in x[1::2].tolist()], dtype=np.uint8)
            assert np.array_equal(codes, lo | (hi << 4))
        else:
            ref = np.array([L.ptxo_f32_to_narrow(fmt, v, 0) for v in x.tolist()], dtype=np.uint8)
            assert np.array_equal(codes, ref)


def test_mxfp8_recipe(oracle):
    """The block scale is floor(log2(amax)) - 8 and every element decodes back within half an
    E4M3 ulp of x / scale (or saturates at 448 for the top binade)."""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((64, 256)) * np.exp2(rng.uniform(-8, 8, (64, 1)))).astype(np.float32)
    x[0, 5] *= 100
    xb = oracle.bf16_from_f32(x)
    q, sf = oracle.quantize_mxfp8(xb)
    xf = oracle.bf16_to_f32(xb).reshape(64, 256)
    for r in range(64):
        for b in range(8):
            blk = xf[r, 32 * b:32 * b + 32]
            amax = np.abs(blk).max()
            want = max(int(np.floor(np.log2(amax))) + 127 - 8, 0) if amax > 0 else 0
            assert sf[r, b] == want
            dec = oracle.decode(0, q[r, 32 * b:32 * b + 32]) * 2.0 ** (int(sf[r, b]) - 127)
            err = np.abs(dec - blk)
            ulp = np.maximum(2.0 ** (np.floor(np.log2(np.maximum(np.abs(blk), 1e-38))) - 3),
                             2.0 ** (int(sf[r, b]) - 127 - 9))
            assert np.all((err <= ulp / 2 * 1.0000001) | (np.abs(dec) == 448 * 2.0 ** (int(sf[r, b]) - 127)))


def test_nvfp4_recipe(oracle):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((32, 128)).astype(np.float32)
    xb = oracle.bf16_from_f32(x)
    xf = oracle.bf16_to_f32(xb).reshape(32, 128)
    g = float(np.abs(xf).max() / (448.0 * 6.0))
    q, sf = oracle.quantize_nvfp4(xb, g)
    assert q.shape == (32, 64) and sf.shape == (32, 8)
    for r in range(32):
        for b in range(8):
            blk = xf[r, 16 * b:16 * b + 16]
            s = np.float32(np.float32(np.abs(blk).max()) / np.float32(np.float32(6.0) * np.float32(g)))
            assert sf[r, b] == oracle.lib().ptxo_f32_to_e4m3(float(s), 0)
            sv = oracle.decode(0, sf[r, b:b + 1])[0]
            nib = q[r, 8 * b:8 * b + 8]
            codes = np.stack([nib & 0xF, nib >> 4], 1).reshape(-1)
            dec = oracle.decode(2, (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8)) * sv * g
            # each element within half an E2M1 step (<= 1 at the top binade) of the block scale
            assert np.all(np.abs(dec - blk) <= sv * g * 1.0 + 1e-6)
    with pytest.raises(ValueError):
        oracle.quantize_nvfp4(xb, 0.0)


def test_blocked_layout_indexing():
    """The blocked scale layout is a bijection of each 128 x 4 tile onto 512 bytes."""
    seen = set()
    for r in range(128):
        for s in range(4):
            off = (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
            seen.add(off)
    assert seen == set(range(512))


def test_gemm_refs_small(oracle):
    rng = np.random.default_rng(5)
    M, N, K = 8, 6, 64
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(0, 256, (N, K), dtype=np.uint8)
    A[(A & 0x7F) == 0x7F] = 0  # no NaNs
    B[(B & 0x7F) == 0x7F] = 0
    rows, cols = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    ref, mag = oracle.gemm_fp8_ref(A, B, 0.5, 2.0, rows.ravel(), cols.ravel())
    da = oracle.decode(0, A.ravel()).reshape(M, K).astype(np.float64)
    db = oracle.decode(0, B.ravel()).reshape(N, K).astype(np.float64)
    want = (da @ db.T).ravel()
    assert np.allclose(ref, want, rtol=1e-12, atol=0)
    assert np.allclose(mag, (np.abs(da) @ np.abs(db).T).ravel(), rtol=1e-12)


def test_gemm_mxfp8_ref_small(oracle):
    """MXFP8 reference = E4M3 decode x 2^(UE8M0 - 127) per 32-element block, summed in f64."""
    rng = np.random.default_rng(6)
    M, N, K = 5, 7, 128
    A = rng.integers(0, 256, (M, K), dtype=np.uint8)
    B = rng.integers(0, 256, (N, K), dtype=np.uint8)
    A[(A & 0x7F) == 0x7F] = 0  # no NaNs
    B[(B & 0x7F) == 0x7F] = 0
    sfA = rng.integers(100, 160, (M, K // 32), dtype=np.uint8)
    sfB = rng.integers(100, 160, (N, K // 32), dtype=np.uint8)
    rows, cols = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    ref, mag = oracle.gemm_mxfp8_ref(A, sfA, B, sfB, rows.ravel(), cols.ravel())
    da = oracle.decode(0, A.ravel()).reshape(M, K).astype(np.float64)
    db = oracle.decode(0, B.ravel()).reshape(N, K).astype(np.float64)
    da *= np.exp2(np.repeat(sfA.astype(np.float64) - 127, 32, axis=1))
    db *= np.exp2(np.repeat(sfB.astype(np.float64) - 127, 32, axis=1))
    assert np.allclose(ref, (da @ db.T).ravel(), rtol=1e-12, atol=0)
    assert np.allclose(mag, (np.abs(da) @ np.abs(db).T).ravel(), rtol=1e-12)


DIGESTS = os.path.join(GOLDEN, "cvt_sweep_digests.json")


@pytest.mark.skipif(not os.path.exists(DIGESTS), reason="no hardware digests recorded yet")
@pytest.mark.parametrize("variant", range(12))
def test_oracle_matches_hardware_digests(oracle, variant):
    """The oracle's codes for all 2^32 f32 inputs hash to the digests of the B200's own `cvt`
    outputs (the reference's encoders are those instructions). A few chunks are checked by
    default; PTXSTD_FULL_SWEEP=1 checks all of them."""
    d = json.load(open(DIGESTS))
    chunk = d["chunk"]
    if oracle.VARIANT_NAMES[variant] not in d["variants"]:
        pytest.skip("no hardware digests recorded for this variant yet")
    digs = d["variants"][oracle.VARIANT_NAMES[variant]]
    full = os.environ.get("PTXSTD_FULL_SWEEP") == "1"
    idx = range(len(digs)) if full else sorted({0, 1, len(digs) // 2 - 1, len(digs) // 2,
                                                len(digs) - 2, len(digs) - 1, 100, 200})
    for i in idx:
        got = oracle.sweep_digest(variant, i * chunk, chunk)
        assert f"{got:016x}" == digs[i], (variant, i)

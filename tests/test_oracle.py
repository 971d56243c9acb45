"""CPU checks of the oracle against the reference's own pins (no GPU).

- decode of every code against the reference's named constants (src/data_types/float8.rs,
  float4.rs, via tests/golden/format_constants.json);
- the soft decode restates minifloat_to_f32 (src/data_types/vector.rs:61-95);
- encode rounding: hand-computed ties and .satfinite boundaries, a second independent (float64)
  formulation of RN, decode->encode round trips;
- the hardware pin: digests of the B200's own `cvt` outputs over all 2^32 f32 patterns
  (tests/golden/cvt_sweep_digests.json, written by tests/golden/make_cvt_digests.py on a B200);
- stochastic rounding (cvt.rs): the random-bit assignment the reference documents, the carry
  rule's limits (all-zero bits truncate, all-one bits round up anything inexact), unbiasedness,
  SplitMix64's published outputs, and the B200's own codes for 18 forms
  (tests/golden/cvt_rs_vectors.json, written by tests/golden/make_cvt_rs_vectors.py).
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
@pytest.mark.parametrize("variant", range(34))
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


# ---- stochastic rounding -------------------------------------------------------------------------

RS_FORMATS = {"e4m3": 0, "e5m2": 1, "e2m1": 2, "e2m3": 3, "e3m2": 4}


def test_rs_random_bit_assignment(oracle):
    """Which rbits bits feed which element (float8.rs:59, float6.rs:61, float4.rs:60,
    bfloat16.rs:576-579, float16.rs:742-746). FP8/FP6: a bit of the lower half reaches elements 0
    and 1 (the even one reads the half most significant bit first, the odd one bit-reversed), a
    bit of the upper half elements 2 and 3; E2M1: the low bytes of both halves feed 0 and 1, the
    high bytes 2 and 3; bf16: one element per half."""
    L = oracle.lib()
    for kind, per, owners in [
        (oracle.RS_X4, 4, lambda b: [0, 1] if b < 16 else [2, 3]),
        (oracle.RS_E2M1, 4, lambda b: [0, 1] if (b % 16) < 8 else [2, 3]),
        (oracle.RS_BF16, 2, lambda b: [0] if b < 16 else [1]),
    ]:
        for b in range(32):
            hit = [k for k in range(per) if L.ptxo_rs_random(kind, 1 << b, k) != 0]
            assert hit == owners(b), (kind, b, hit)
    # the even element weights bit 15 (bit 31) most, the odd one bit 0 (bit 16)
    assert L.ptxo_rs_random(oracle.RS_X4, 1 << 15, 0) == 0x8000
    assert L.ptxo_rs_random(oracle.RS_X4, 1, 1) == 0x8000
    assert L.ptxo_rs_random(oracle.RS_X4, 1 << 16, 3) == 0x8000
    # f16 uses only the 13 low bits of each half
    for b in range(32):
        hit = [k for k in range(2) if L.ptxo_rs_random(oracle.RS_F16, 1 << b, k) != 0]
        assert hit == ([0] if b < 13 else [1] if 16 <= b < 29 else []), (b, hit)


# (mantissa bits, minimum normal exponent, largest finite value) of the narrow formats
RS_PARAMS = {"e4m3": (3, -6, 448.0), "e5m2": (2, -14, 57344.0), "e2m1": (1, 0, 6.0),
             "e2m3": (3, 0, 7.5), "e3m2": (2, -2, 28.0)}


def _rs_f64(fmt, x, r):
    """Second, float64 formulation of the stochastic rounding of finite x with w = 16 random
    bits r: quantum 2^(max(e, emin) - M); up when floor(frac * 2^16) + r >= 2^16; .satfinite."""
    M, emin, mx = RS_PARAMS[fmt]
    a = np.abs(x.astype(np.float64))
    _, ex = np.frexp(np.where(a > 0, a, 1.0))
    q = np.ldexp(1.0, np.maximum(ex - 1, emin) - M)
    t = np.floor(a / q)
    up = np.floor((a / q - t) * 65536.0) + r >= 65536
    v = np.minimum((t + up) * q, mx)
    return np.where(np.signbit(x), -v, v)


@pytest.mark.parametrize("fmt", list(RS_FORMATS))
def test_rs_matches_float64_formulation(oracle, fmt):
    """The integer restatement equals an independent float64 one on random finite inputs and
    random bits; with all-zero bits it truncates toward zero."""
    f = RS_FORMATS[fmt]
    rng = np.random.default_rng(5)
    n = 1 << 14
    x = (rng.standard_normal(n) * np.exp2(rng.integers(-12, 8, n))).astype(np.float32)
    rb = rng.integers(0, 1 << 32, n // 4, dtype=np.uint64).astype(np.uint32)
    kind = oracle.RS_E2M1 if f == oracle.E2M1 else oracle.RS_X4
    L = oracle.lib()
    r = np.array([L.ptxo_rs_random(kind, int(rb[i // 4]), i % 4) for i in range(n)])
    got = oracle.decode(f, oracle.encode_rs(f, x, rb)).astype(np.float64)
    assert np.array_equal(got, _rs_f64(fmt, x, r))
    zero = oracle.decode(f, oracle.encode_rs(f, x, np.zeros(n // 4, np.uint32))).astype(np.float64)
    assert np.all(np.abs(zero) <= np.abs(x.astype(np.float64)))
    assert np.array_equal(zero, _rs_f64(fmt, x, np.zeros(n)))


def test_rs_unbiased(oracle):
    """The mean of the stochastic E4M3 and bf16 roundings of one value over random bits is the
    value (the point of .rs), within 5 standard errors."""
    rng = np.random.default_rng(7)
    n = 1 << 16
    rb = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    for v in (1.1, -3.3, 0.0123, 300.7):
        x = np.full(4 * n, v, np.float32)
        q = oracle.decode(0, oracle.encode_rs(0, x, rb)).astype(np.float64)
        assert abs(q.mean() - float(np.float32(v))) < 5 * q.std() / math.sqrt(q.size) + 1e-12, v
        h = oracle.bf16_rs(x[: 2 * n], rb)
        qb = oracle.bf16_to_f32(h).astype(np.float64)
        assert abs(qb.mean() - float(np.float32(v))) < 5 * qb.std() / math.sqrt(qb.size) + 1e-12


def test_splitmix64_published_outputs(oracle):
    """SplitMix64 seeded with 0 (Steele, Lea and Flood 2014; the reference generator's first
    outputs), and the vectorised numpy copy used by the tests."""
    L = oracle.lib()
    assert L.ptxo_splitmix64(0, 0) == 0xE220A8397B1DCDAF
    assert L.ptxo_splitmix64(0, 1) == 0x6E789E6AA1B965F4
    words = oracle.sr_rbits(0x1234, 10)
    for g in range(10):
        assert int(words[g]) == L.ptxo_sr_rbits(0x1234, g)


RS_VECTORS = os.path.join(GOLDEN, "cvt_rs_vectors.json")


@pytest.mark.skipif(not os.path.exists(RS_VECTORS), reason="no hardware vectors recorded yet")
def test_rs_hardware_vectors(oracle):
    """The oracle reproduces the B200's cvt.rs codes for every recorded form."""
    d = json.load(open(RS_VECTORS))["forms"]
    assert len(d) == 18
    for key, rec in d.items():
        x = np.array([int(v, 16) for v in rec["x"]], dtype=np.uint32).view(np.float32)
        rb = np.array([int(v, 16) for v in rec["rbits"]], dtype=np.uint32)
        relu, sat = "_relu" in key, key.endswith("_sat")
        name = key.split("_")[0]
        hw = bytes.fromhex(rec["codes"])
        if name in ("bf16", "f16"):
            got = (oracle.bf16_rs if name == "bf16" else oracle.f16_rs)(x, rb, relu, sat)
            want = np.frombuffer(hw, dtype=np.uint16)
        else:
            got = oracle.encode_rs(RS_FORMATS[name], x, rb, relu)
            want = np.frombuffer(hw, dtype=np.uint8)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (key, bad[:4], got[bad[:4]], want[bad[:4]])


def test_rs_quantize_keeps_scales(oracle):
    """The stochastic quantisers keep the round-to-nearest scales; every element is within one
    code step of the RN element, and one seed always gives the same codes."""
    from ptxstd import workloads
    xb = workloads.normal_bf16(64, 512, std=1.0, seed=3)
    q0, s0 = oracle.quantize_mxfp8(xb)
    q1, s1 = oracle.quantize_mxfp8_rs(xb, 99)
    q2, _ = oracle.quantize_mxfp8_rs(xb, 99)
    q3, _ = oracle.quantize_mxfp8_rs(xb, 100)
    assert np.array_equal(s0, s1) and np.array_equal(q1, q2) and not np.array_equal(q1, q3)
    d0 = oracle.decode(0, q0.ravel()).astype(np.float64)
    d1 = oracle.decode(0, q1.ravel()).astype(np.float64)
    step = np.maximum(np.abs(d0) * 2.0 ** -3, 2.0 ** -9) * 1.0001  # E4M3 spacing
    assert np.all(np.abs(d1 - d0) <= step)
    g = 0.01
    n0, t0 = oracle.quantize_nvfp4(xb, g)
    n1, t1 = oracle.quantize_nvfp4_rs(xb, g, 5)
    assert np.array_equal(t0, t1)


# ---- 2:4 structured sparsity ---------------------------------------------------------------------

def test_prune_24_rules(oracle):
    """The two largest magnitudes of each group of four stay, in index order, ties to the lower
    index; the NaN code sorts highest; metadata nibble = i0 | i1 << 2, even groups low."""
    A = np.array([[0x38, 0x40, 0x30, 0x48,   0x05, 0x05, 0x05, 0x05],
                  [0xC8, 0x01, 0x7F, 0x00,   0x80, 0x00, 0x81, 0x02]], dtype=np.uint8)
    v, m = oracle.prune_24(A)
    assert v.tolist() == [[0x40, 0x48, 0x05, 0x05], [0xC8, 0x7F, 0x81, 0x02]]
    # row 0: group 0 keeps (1, 3) -> 0b1101, group 1 ties keep (0, 1) -> 0b0100
    # row 1: group 0 keeps (0, 2) -> 0b1000, group 1 keeps (2, 3) -> 0b1110
    assert m.tolist() == [[0x4D], [0xE8]]
    d = oracle.decompress_24(v, m)
    assert d.tolist() == [[0, 0x40, 0, 0x48, 0x05, 0x05, 0, 0], [0xC8, 0, 0x7F, 0, 0, 0, 0x81, 0x02]]


def test_sparse_ref_equals_dense_ref(oracle):
    """The sparse reference over (vals, meta) equals the dense MXFP8 reference over the
    decompressed A with each 64-scale repeated for both 32-blocks."""
    rng = np.random.default_rng(8)
    M, N, K = 8, 6, 256
    A = rng.integers(0, 0x7E, (M, K)).astype(np.uint8)
    B = rng.integers(0, 0x7E, (N, K)).astype(np.uint8)
    v, m = oracle.prune_24(A)
    sfA = rng.integers(120, 134, (M, K // 64)).astype(np.uint8)
    sfB = rng.integers(120, 134, (N, K // 64)).astype(np.uint8)
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    r, c = r.ravel(), c.ravel()
    s_ref, s_mag = oracle.gemm_mxfp8_sparse_ref(v, m, sfA, B, sfB, r, c)
    d_ref, d_mag = oracle.gemm_mxfp8_ref(oracle.decompress_24(v, m), np.repeat(sfA, 2, axis=1), B,
                                         np.repeat(sfB, 2, axis=1), r, c)
    assert np.allclose(s_ref, d_ref, rtol=1e-12, atol=0) and np.allclose(s_mag, d_mag, rtol=1e-12)


# ---- scaled up-conversion to bf16 --------------------------------------------------------------

def test_to_bf16_scaled_rules(oracle):
    """Known answers of the exact scaled conversion: an exact power-of-two product, overflow to
    infinity or (with .satfinite) to the largest finite bf16, rounding below 2^-126, .relu, NaN."""
    L = oracle.lib()
    E4 = oracle.E4M3
    assert L.ptxo_to_bf16_scaled(E4, 0x38, 130, 0, 0) == 0x4100          # 1.0 * 2^3
    assert L.ptxo_to_bf16_scaled(E4, 0x7E, 254, 0, 0) == 0x7F80          # 448 * 2^127 -> inf
    assert L.ptxo_to_bf16_scaled(E4, 0xFE, 254, 0, 1) == 0xFF7F          # -> -max finite
    assert L.ptxo_to_bf16_scaled(E4, 0x01, 0, 0, 0) == 0x0000            # 2^-136 -> +0
    assert L.ptxo_to_bf16_scaled(E4, 0x06, 0, 0, 0) == 0x0001            # 0.75 * 2^-133 -> 2^-133
    assert L.ptxo_to_bf16_scaled(E4, 0xB8, 127, 1, 0) == 0x0000          # relu(-1) = +0
    assert L.ptxo_to_bf16_scaled(E4, 0x7F, 127, 0, 0) == 0x7FFF          # NaN code
    assert L.ptxo_to_bf16_scaled(E4, 0x38, 255, 0, 0) == 0x7FFF          # NaN scale
    assert L.ptxo_to_bf16_scaled(oracle.E5M2, 0x7C, 127, 0, 1) == 0x7F7F  # inf, satfinite


def test_to_bf16_scaled_exact_in_range(oracle):
    """Where the product is a normal bf16, the result is exactly code value * 2^(scale - 127)."""
    for fmt, ncodes in [(oracle.E4M3, 256), (oracle.E5M2, 256), (oracle.E2M3, 64)]:
        codes = np.repeat(np.arange(ncodes, dtype=np.uint8), 100)
        scales = np.tile(np.arange(90, 190, dtype=np.uint8), ncodes)
        got = oracle.to_bf16_scaled(fmt, codes, scales, codes.size)
        v = oracle.decode(fmt, codes).astype(np.float64) * np.exp2(scales.astype(np.float64) - 127)
        ok = np.isfinite(v) & ((np.abs(v) >= 2.0 ** -126) | (v == 0)) & (np.abs(v) < 2.0 ** 127)
        want = (v[ok].astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
        assert np.array_equal(got[ok], want)


def test_narrow_to_f16_exact(oracle):
    """The f16 pattern of every code is the exact value (numpy's float16 of the decode)."""
    L = oracle.lib()
    for fmt, n in [(oracle.E4M3, 256), (oracle.E5M2, 256), (oracle.E2M3, 64), (oracle.E3M2, 64),
                   (oracle.E2M1, 16)]:
        for c in range(n):
            v = oracle.decode(fmt, np.array([c if fmt != oracle.E2M1 else c], dtype=np.uint8))
            v = v[0] if fmt != oracle.E2M1 else v[0]
            got = L.ptxo_narrow_to_f16(fmt, c)
            if np.isnan(v):
                assert got == 0x7FFF
            else:
                assert got == int(np.float16(v).view(np.uint16)), (fmt, c)


def test_bf16_mode_rules(oracle):
    L = oracle.lib()
    f = lambda bits, r=0, s=0: L.ptxo_f32_to_bf16_mode(float(np.uint32(bits).view(np.float32)), r, s)  # noqa: E731
    assert f(0x3F800000) == 0x3F80                      # 1.0
    assert f(0x3F808000) == 0x3F80                      # tie to even
    assert f(0x3F818000) == 0x3F82                      # tie to even (up)
    assert f(0x7F7FFFFF) == 0x7F80 and f(0x7F7FFFFF, 0, 1) == 0x7F7F   # rounds past max
    assert f(0xFF800000, 0, 1) == 0xFF7F and f(0xFF800000, 1, 0) == 0
    assert f(0x80000000, 1, 0) == 0 and f(0x7FC00001) == 0x7FFF


# ---- MX formats in the tensor-core operand layout ------------------------------------------

_MX_FORMATS = [("e4m3", 0, 0xFF), ("e5m2", 1, 0xFF), ("e2m3", 3, 0x3F), ("e3m2", 4, 0x3F),
               ("e2m1", 2, 0x0F)]


@pytest.mark.parametrize("name,fmt,mask", _MX_FORMATS)
def test_mx_pack_round_trip(oracle, name, fmt, mask):
    """Packing into the K = 32 operand layout (descriptor.rs:306-315) and back is the identity;
    FP6 groups end in 4 zero bytes, FP4 groups in 8."""
    rng = np.random.default_rng(7 + fmt)
    codes = (rng.integers(0, 256, (8, 128)) & mask).astype(np.uint8)
    packed = oracle.mx_pack(fmt, codes)
    assert packed.shape == codes.shape
    assert np.array_equal(oracle.mx_unpack(fmt, packed), codes)
    pad = {oracle.E2M3: 12, oracle.E3M2: 12, oracle.E2M1: 8}.get(fmt)
    if pad is not None:
        assert not packed.reshape(-1, 16)[:, pad:].any()
    else:
        assert np.array_equal(packed, codes)


def test_mx_pack_known_answers(oracle):
    """Element i of an FP6 group at bits 6i .. 6i+5 of its little-endian 96 bits; FP4 element 2j
    in the low nibble of byte j."""
    one = np.zeros((1, 16), dtype=np.uint8)
    for i in range(16):
        c = one.copy()
        c[0, i] = 0x3F
        bits = int.from_bytes(oracle.mx_pack(oracle.E2M3, c).tobytes()[:12], "little")
        assert bits == 0x3F << (6 * i)
        c[0, i] = 0x9
        p = oracle.mx_pack(oracle.E2M1, c & 0xF).tobytes()
        assert p[i // 2] == (0x9 << (4 * (i % 2))) and sum(p) == p[i // 2]


def test_quantize_mx_e4m3_is_mxfp8(oracle):
    from ptxstd import workloads
    x = workloads.mxfp8_activation(64, 512)
    q, sf = oracle.quantize_mx(x, oracle.E4M3)
    q8, sf8 = oracle.quantize_mxfp8(x)
    assert np.array_equal(q, q8) and np.array_equal(sf, sf8)


@pytest.mark.parametrize("name,fmt,mask", _MX_FORMATS)
def test_quantize_mx_scale_recipe(oracle, name, fmt, mask):
    """Scale = floor(log2 amax) - emax(format) + 127: a block whose amax is the format's largest
    finite value gets 2^0, one whose amax is 2^e gets 2^(e - emax); elements then decode back to
    the input exactly when it is representable."""
    emax = {0: 8, 1: 15, 3: 2, 4: 4, 2: 2}[fmt]
    top = {0: 448.0, 1: 57344.0, 3: 7.5, 4: 28.0, 2: 6.0}[fmt]
    x = np.zeros((2, 32), dtype=np.float32)
    x[0, :] = np.linspace(-top, top, 32).astype(np.float32)
    x[0, 0], x[0, 31] = -top, top
    x[1, :] = 0.0
    x[1, 5] = 2.0 ** 10
    bf = (x.view(np.uint32) >> 16).astype(np.uint16)
    q, sf = oracle.quantize_mx(bf, fmt)
    assert sf[0, 0] == 127 + (int(np.floor(np.log2(top))) - emax)
    assert sf[1, 0] == 127 + 10 - emax
    codes = oracle.mx_unpack(fmt, q)
    dec = oracle.decode(fmt, codes[0] if fmt != oracle.E2M1 else
                        (codes[0, 0::2] | (codes[0, 1::2] << 4)).astype(np.uint8))
    assert dec[0] == -top * 2.0 ** -(int(sf[0, 0]) - 127) and dec[-1] == -dec[0]
    assert codes[1, 5] != 0 and not np.delete(codes[1], 5).any()


def test_cp_unpack_container_rule(oracle):
    """tcgen05.cp decompression, as pinned on the B200: an FP6 code sits in bits 5..0 of its 8-bit
    container, an FP4 code in bits 5..2 (row of codes 0..15 twice -> 00 04 08 .. 3c, twice)."""
    c6 = (np.arange(32) & 0x3F).astype(np.uint8)[None, :]
    assert np.array_equal(oracle.cp_unpack(oracle.E2M3, oracle.mx_pack(oracle.E2M3, c6)), c6)
    c4 = (np.arange(32) & 0xF).astype(np.uint8)[None, :]
    got = oracle.cp_unpack(oracle.E2M1, oracle.mx_pack(oracle.E2M1, c4))
    assert got.tobytes().hex() == "0004080c1014181c2024282c3034383c" * 2


# (format, significand bits after the point, smallest normal exponent, largest finite value)
_MX_FORMAT_GEOMETRY = [(0, 3, -6, 448.0), (1, 2, -14, 57344.0), (3, 3, 0, 7.5),
                       (4, 2, -2, 28.0), (2, 1, 0, 6.0)]


@pytest.mark.parametrize("fmt,mbits,emin,top", _MX_FORMAT_GEOMETRY)
def test_quantize_mx_error_bound(oracle, fmt, mbits, emin, top):
    """Independent float64 check of the MX recipe: each element, decoded and scaled by its block's
    2^(sf - 127), is within half a unit in the last place (of the format, at the element's scaled
    magnitude, subnormal quantum below the normal range) of the input; where the scaled input
    exceeds the format's largest finite value, the element saturates to it."""
    from ptxstd import workloads
    x_bits = workloads.mxfp8_activation(64, 1024, seed=1234 + fmt)
    x = (x_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    q, sf = oracle.quantize_mx(x_bits, fmt)
    codes = oracle.mx_unpack(fmt, q)
    if fmt == oracle.E2M1:
        dec = oracle.decode(fmt, (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8))
    else:
        dec = oracle.decode(fmt, codes)
    dec = dec.reshape(x.shape).astype(np.float64)
    scale = np.exp2(np.repeat(sf.astype(np.float64) - 127.0, 32, axis=1))
    y = x / scale                               # the scaled input the element encodes
    a = np.abs(y)
    e = np.floor(np.log2(np.maximum(a, 2.0 ** emin)))
    half_ulp = np.exp2(e - mbits - 1)
    sat = a > top
    assert np.all(np.abs(dec[sat]) == top) and np.all(np.sign(dec[sat]) == np.sign(y[sat]))
    ok = ~sat
    assert np.all(np.abs(dec[ok] - y[ok]) <= half_ulp[ok]), fmt
    # the recipe keeps every block's largest element at or above half the format's top binade
    amax = np.abs(x).reshape(64, -1, 32).max(axis=2)
    big = amax > 0
    ratio = amax[big] / np.exp2(sf[big].astype(np.float64) - 127.0)
    assert np.all(ratio >= 2.0 ** np.floor(np.log2(top)))


def test_gemm_mx_ref_matches_numpy(oracle):
    """The MX GEMM reference (mixed E3M2 x E2M1 here) equals a float64 numpy product of the
    unpacked, decoded and scaled operands at every output."""
    rng = np.random.default_rng(17)
    M, N, K = 8, 6, 128
    ca = (rng.integers(0, 64, (M, K))).astype(np.uint8)
    cb = (rng.integers(0, 16, (N, K))).astype(np.uint8)
    sfa = rng.integers(120, 135, (M, K // 32), dtype=np.uint8)
    sfb = rng.integers(120, 135, (N, K // 32), dtype=np.uint8)
    A, B = oracle.mx_pack(oracle.E3M2, ca), oracle.mx_pack(oracle.E2M1, cb)
    da = oracle.decode(oracle.E3M2, ca).reshape(M, K).astype(np.float64)
    db = oracle.decode(oracle.E2M1, (cb[:, 0::2] | (cb[:, 1::2] << 4)).astype(np.uint8))
    db = db.reshape(N, K).astype(np.float64)
    da *= np.exp2(np.repeat(sfa.astype(np.float64) - 127, 32, axis=1))
    db *= np.exp2(np.repeat(sfb.astype(np.float64) - 127, 32, axis=1))
    want = da @ db.T
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    ref, mag = oracle.gemm_mx_ref(A, oracle.E3M2, sfa, B, oracle.E2M1, sfb, r.ravel(), c.ravel())
    assert np.allclose(ref, want.ravel(), rtol=1e-12, atol=0)
    assert np.allclose(mag, (np.abs(da) @ np.abs(db).T).ravel(), rtol=1e-12, atol=0)

"""Device conversions vs the oracle, bit-exact (B200).

- every code of every format decoded on the device equals the oracle's decode (bits, NaN too);
- the narrow-float round-trip set (2^24 seeded values with specials) encoded to E4M3, E5M2,
  E2M1x2, E2M3 and E3M2 (RN .satfinite, with and without .relu) and decoded back matches the
  oracle bit for bit;
- all 2^32 f32 bit patterns, through the device's `cvt` for the twelve round-to-nearest variants
  and the eighteen stochastic-rounding forms (cvt.rs with SplitMix64 bits per group), match the
  oracle (the exhaustive pin of the oracle against the instructions the reference wraps);
- the element-wise stochastic entry points (caller-supplied rbits, ragged lengths whose last
  group is zero-padded, .relu, .satfinite) match the oracle bit for bit.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _to_np(t):
    return t.cpu().numpy()


def test_decode_every_code(cuda, oracle):
    import ptxstd.data_types as dt
    torch = cuda
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).cuda()
    for fmt, fid in ((dt.E4M3, 0), (dt.E5M2, 1)):
        got = _to_np(dt.to_f32(fmt, codes)).view(np.uint32)
        want = np.array([oracle.lib().ptxo_to_f32_via_half(fid, c) for c in range(256)],
                        dtype=np.float32).view(np.uint32)
        assert np.array_equal(got, want), (fmt, np.nonzero(got != want)[0][:8])
    got = _to_np(dt.to_f32(dt.E2M1, codes)).view(np.uint32)
    want = oracle.decode(2, np.arange(256, dtype=np.uint8)).view(np.uint32)
    assert np.array_equal(got, want)
    # FP6: the value lives in the low 6 bits (src/data_types/float6.rs:1-8)
    for fmt, fid in ((dt.E2M3, 3), (dt.E3M2, 4)):
        got = _to_np(dt.to_f32(fmt, codes[:64])).view(np.uint32)
        want = np.array([oracle.lib().ptxo_to_f32_via_half(fid, c) for c in range(64)],
                        dtype=np.float32).view(np.uint32)
        assert np.array_equal(got, want), (fmt, np.nonzero(got != want)[0][:8])
    # ue8m0 widens through bf16 with a bit shift (bf16::to_f32, src/data_types/bfloat16.rs:84-86)
    got = _to_np(dt.ue8m0_to_f32(codes)).view(np.uint32)
    want = np.array([oracle.lib().ptxo_ue8m0_to_f32_via_bf16(c) for c in range(256)],
                    dtype=np.float32).view(np.uint32)
    assert np.array_equal(got, want), np.nonzero(got != want)[0][:8]


@pytest.mark.parametrize("relu", [False, True])
def test_roundtrip_set(cuda, oracle, relu):
    import ptxstd.data_types as dt
    from ptxstd import workloads
    torch = cuda
    x = workloads.conversion_inputs(1 << 24)
    xd = torch.from_numpy(x).cuda()
    for fmt, fid in ((dt.E4M3, 0), (dt.E5M2, 1), (dt.E2M1, 2), (dt.E2M3, 3), (dt.E3M2, 4)):
        codes = dt.from_f32(fmt, xd, relu=relu)
        want = oracle.encode(fid, x, relu=relu)
        got = _to_np(codes)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (fmt, relu, [(hex(x[i:i + 1].view(np.uint32)[0]), got[i], want[i])
                                           for i in bad[:8]])
        back = _to_np(dt.to_f32(fmt, codes)).view(np.uint32)
        wback = oracle.decode(fid, want).view(np.uint32)
        assert np.array_equal(back, wback), fmt


def test_ue8m0_set(cuda, oracle):
    import ptxstd.data_types as dt
    from ptxstd import workloads
    torch = cuda
    x = workloads.conversion_inputs(1 << 22)
    xd = torch.from_numpy(x).cuda()
    for up in (False, True):
        for sat in (True, False):
            got = _to_np(dt.ue8m0_from_f32(xd, round_up=up, satfinite=sat))
            want = oracle.ue8m0_encode(x, rnd_up=up, satfinite=sat)
            if not sat:
                # Without .satfinite the ISA leaves overflow undefined: compare the rest only.
                keep = (np.abs(x) < 2.0 ** 127) | np.isnan(x)
                got, want = got[keep], want[keep]
            bad = np.nonzero(got != want)[0]
            assert bad.size == 0, (up, sat, bad[:8])


def test_exhaustive_all_f32(cuda, oracle):
    """All 2^32 inputs, 30 variants, in 2^28 chunks: zero mismatches."""
    import ptxstd.data_types as dt
    torch = cuda
    chunk = 1 << 28
    dev = torch.empty(2 * chunk, dtype=torch.uint8, device="cuda")
    host = torch.empty(2 * chunk, dtype=torch.uint8, pin_memory=True)
    total_bad = {}
    for v in range(len(oracle.VARIANT_NAMES)):
        bad = 0
        report = []
        w = oracle.sweep_width(v)
        for base in range(0, 1 << 32, chunk):
            dt.sweep(v, base, chunk, out=dev)
            host.copy_(dev)
            n, rep = oracle.sweep_compare(v, base, host.numpy()[: w * chunk], max_report=8)
            bad += n
            report += [tuple(int(t) for t in r) for r in rep[:4]]
        total_bad[oracle.VARIANT_NAMES[v]] = (bad, [(hex(a), hex(b), hex(c))
                                                    for a, b, c in report[:8]])
    assert all(b == 0 for b, _ in total_bad.values()), total_bad


# ---- stochastic rounding through the element-wise entry points -----------------------------------

def _rs_inputs(n, seed):
    rng = np.random.default_rng(seed)
    e = rng.integers(-30, 20, n)
    m = rng.integers(0, 1 << 23, n)
    bits = ((rng.integers(0, 2, n) << 31) | ((e + 127) << 23) | m).astype(np.uint32)
    sp = np.array([0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00000, 3], dtype=np.uint32)
    bits[: min(n, sp.size)] = sp[:n]
    rb = rng.integers(0, 1 << 32, (n + 3) // 4, dtype=np.uint64).astype(np.uint32)
    return bits.view(np.float32), rb


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m3", "e3m2", "e2m1"])
@pytest.mark.parametrize("relu", [False, True])
def test_stochastic_vs_oracle(cuda, oracle, fmt, relu):
    import ptxstd.data_types as dt
    torch = cuda
    ofmt = {"e4m3": oracle.E4M3, "e5m2": oracle.E5M2, "e2m3": oracle.E2M3, "e3m2": oracle.E3M2,
            "e2m1": oracle.E2M1}[fmt]
    for n in ((1 << 20), (1 << 20) + 2) + (() if fmt == "e2m1" else ((1 << 20) + 1, 7, 1)):
        x, rb = _rs_inputs(n, n)
        got = _to_np(dt.from_f32_stochastic(fmt, torch.from_numpy(x).cuda(),
                                            torch.from_numpy(rb.view(np.int32)).cuda(), relu))
        want = oracle.encode_rs(ofmt, x, rb, relu)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (n, bad[:4], got[bad[:4]], want[bad[:4]])


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("relu", [False, True])
@pytest.mark.parametrize("sat", [False, True])
def test_stochastic_x2_vs_oracle(cuda, oracle, kind, relu, sat):
    import ptxstd.data_types as dt
    torch = cuda
    dev_fn = dt.bf16_from_f32_stochastic if kind == "bf16" else dt.f16_from_f32_stochastic
    ora_fn = oracle.bf16_rs if kind == "bf16" else oracle.f16_rs
    for n in ((1 << 20), (1 << 20) + 1, 3):
        x, rb = _rs_inputs(n, 7 * n)
        rb = np.concatenate([rb, rb])[: (n + 1) // 2]
        got = _to_np(dev_fn(torch.from_numpy(x).cuda(), torch.from_numpy(rb.view(np.int32)).cuda(),
                            relu, sat)).view(np.uint16)
        want = ora_fn(x, rb, relu, sat)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (n, bad[:4], got[bad[:4]], want[bad[:4]])


def test_stochastic_unbiased_on_device(cuda):
    """Mean of the device's stochastic E4M3 codes of one value over 2^22 random words equals the
    value within 5 standard errors, while RN is biased by its rounding error."""
    import ptxstd.data_types as dt
    torch = cuda
    n = 1 << 24
    v = 1.1  # between the E4M3 codes 1.0 and 1.125
    x = torch.full((n,), v, dtype=torch.float32, device="cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    rb = torch.randint(-(2 ** 31), 2 ** 31 - 1, (n // 4,), dtype=torch.int32, device="cuda",
                       generator=g)
    q = dt.to_f32("e4m3", dt.from_f32_stochastic("e4m3", x, rb)).double()
    mean, se = q.mean().item(), q.std().item() / n ** 0.5
    exact = float(np.float32(v))
    assert abs(mean - exact) < 5 * se
    rn = dt.to_f32("e4m3", dt.from_f32("e4m3", x[:4])).double()[0].item()
    assert abs(rn - exact) > 50 * se


# ---- scaled up-conversion to bf16 ------------------------------------------------------------------

@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m3", "e3m2", "e2m1"])
def test_to_bf16_scaled_exhaustive(cuda, oracle, fmt):
    """Every code times every UE8M0 scale (0x00 .. 0xff), with and without .relu / .satfinite,
    bit for bit against the oracle; then MX dequantisation of random rows with one scale per 32."""
    import ptxstd.data_types as dt
    torch = cuda
    ofmt = {"e4m3": oracle.E4M3, "e5m2": oracle.E5M2, "e2m3": oracle.E2M3, "e3m2": oracle.E3M2,
            "e2m1": oracle.E2M1}[fmt]
    ncodes = {"e4m3": 256, "e5m2": 256, "e2m3": 64, "e3m2": 64, "e2m1": 16}[fmt]
    codes = np.repeat(np.arange(ncodes, dtype=np.uint8), 256)
    scales = np.tile(np.arange(256, dtype=np.uint8), ncodes)
    n = codes.size
    packed = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8) if fmt == "e2m1" else codes
    cd, sd = torch.from_numpy(packed).cuda(), torch.from_numpy(scales).cuda()
    for relu in (False, True):
        for sat in (False, True):
            got = _to_np(dt.to_bf16_scaled(fmt, cd, sd, 1, relu, sat)).view(np.uint16)
            want = oracle.to_bf16_scaled(ofmt, packed, scales, n, 1, relu, sat)
            bad = np.nonzero(got != want)[0]
            assert bad.size == 0, (relu, sat, [(int(codes[i]), int(scales[i]), hex(got[i]),
                                                hex(want[i])) for i in bad[:6]])
    rng = np.random.default_rng(11)
    m = 1 << 16
    rc = rng.integers(0, 256, m // 2 if fmt == "e2m1" else m).astype(np.uint8)
    if fmt in ("e2m3", "e3m2"):
        rc &= 0x3F
    rs = rng.integers(100, 150, m // 32).astype(np.uint8)
    got = _to_np(dt.to_bf16_scaled(fmt, torch.from_numpy(rc).cuda(), torch.from_numpy(rs).cuda(),
                                   32)).view(np.uint16)
    assert np.array_equal(got, oracle.to_bf16_scaled(ofmt, rc, rs, m, 32))


# ---- f16 sources, f16 results, bf16 round-to-nearest modes -----------------------------------------

@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m3", "e3m2", "e2m1"])
def test_from_f16_all_patterns(cuda, oracle, fmt):
    """All 65536 f16 bit patterns, with and without .relu: the device codes equal the oracle's
    encoding of the exactly widened f32 value (FP8 through the hardware f16x2 instruction)."""
    import ptxstd.data_types as dt
    torch = cuda
    ofmt = {"e4m3": oracle.E4M3, "e5m2": oracle.E5M2, "e2m3": oracle.E2M3, "e3m2": oracle.E3M2,
            "e2m1": oracle.E2M1}[fmt]
    h = np.arange(1 << 16, dtype=np.uint16)
    xd = torch.from_numpy(h.view(np.int16)).cuda().view(torch.float16)
    for relu in (False, True):
        got = _to_np(dt.from_f16(fmt, xd, relu))
        want = oracle.encode(ofmt, h.view(np.float16).astype(np.float32), relu)
        bad = np.nonzero(got != want)[0]
        assert bad.size == 0, (relu, [(hex(int(h[i])), hex(got[i]), hex(want[i])) for i in bad[:6]])


@pytest.mark.parametrize("fmt", ["e4m3", "e5m2", "e2m3", "e3m2", "e2m1"])
def test_to_f16_every_code(cuda, oracle, fmt):
    import ptxstd.data_types as dt
    torch = cuda
    ofmt = {"e4m3": oracle.E4M3, "e5m2": oracle.E5M2, "e2m3": oracle.E2M3, "e3m2": oracle.E3M2,
            "e2m1": oracle.E2M1}[fmt]
    ncodes = {"e4m3": 256, "e5m2": 256, "e2m3": 64, "e3m2": 64, "e2m1": 16}[fmt]
    codes = np.arange(ncodes, dtype=np.uint8)
    dev = (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8) if fmt == "e2m1" else codes
    got = _to_np(dt.to_f16(fmt, torch.from_numpy(dev).cuda()).view(torch.int16)).view(np.uint16)
    L = oracle.lib()
    want = np.array([L.ptxo_narrow_to_f16(ofmt, int(c)) for c in codes], dtype=np.uint16)
    assert np.array_equal(got, want), [(int(c), hex(g), hex(w)) for c, g, w in zip(codes, got, want)
                                       if g != w][:6]


def test_bf16_from_f32_modes(cuda, oracle):
    """The element-wise bf16 conversion in its four modes on random bit patterns plus specials
    (the exhaustive pin is the sweep's bf16_rn variants)."""
    import ptxstd.data_types as dt
    torch = cuda
    rng = np.random.default_rng(12)
    bits = rng.integers(0, 1 << 32, 1 << 20, dtype=np.uint64).astype(np.uint32)
    bits[:8] = [0, 0x80000000, 0x7F800000, 0xFF800000, 0x7FC00001, 0x7F7FFFFF, 0xFF7FFFFF, 1]
    x = bits.view(np.float32)
    L = oracle.lib()
    for relu in (False, True):
        for sat in (False, True):
            got = _to_np(dt.bf16_from_f32(torch.from_numpy(x).cuda(), relu, sat)).view(np.uint16)
            want = np.array([L.ptxo_f32_to_bf16_mode(float(v), relu, sat) for v in x[:4096]],
                            dtype=np.uint16)
            assert np.array_equal(got[:4096], want), (relu, sat)

"""MX formats beyond E4M3 on the B200: ptxstd_quantize_mx (E4M3, E5M2, E2M3, E3M2, E2M1 with UE8M0
per 32, payload in the tensor cores' K = 32 operand layout: FP6 / FP4 16-element groups padded
to 16 bytes) and ptxstd_gemm_mx (tcgen05.mma.kind::mxf8f6f4.block_scale.block32 with any pair
of element types).

  - quantise: payload and scales bit-exact against the oracle (ptxo_quantize_mx), both scale
    layouts, inputs with zero blocks, NaN / inf and heavy-tailed rows;
  - GEMM: against the oracle's f64 GEMM over the decoded payloads, with the MXFP8 tolerance
    |C - ref| <= 2^-10 * sum_k |a b| + 2^-8 |ref|. Random codes of every finite value check the
    packing the tensor cores read (a misplaced bit changes the products), over all 25 (A, B)
    type pairs; quantised operands check the quantise -> GEMM chain, mixed types included;
  - the decompressing tcgen05.cp: every FP6 / FP4 code into its 8-bit container.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (name, tcgen05 type code, oracle format, code mask)
TYPES = {"e4m3": (0, 0, 0xFF), "e5m2": (1, 1, 0xFF), "e2m3": (3, 3, 0x3F), "e3m2": (4, 4, 0x3F),
         "e2m1": (5, 2, 0x0F)}


def to_blocked(sf: np.ndarray) -> np.ndarray:
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _activation(rows, cols, seed):
    from ptxstd import workloads
    x = workloads.mxfp8_activation(rows, cols, seed=seed).copy()
    x[1, 0:32] = 0                  # an all-zero block
    x[2, 40] = 0x7FC0               # NaN
    x[3, 70] = 0x7F80               # +inf
    x[4, 100] = 0xFF80              # -inf
    x[5, 130] = 0x0001              # bf16 subnormal
    return x


@pytest.mark.parametrize("name", list(TYPES))
@pytest.mark.parametrize("layout", [0, 1])
def test_quantize_mx_bit_exact(cuda, oracle, name, layout):
    torch = cuda
    import ptxstd
    t, fmt, _ = TYPES[name]
    x = _activation(256, 1024, seed=41 + t)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    q, sf = ptxstd.quantize_mx(xd, name, sf_layout=layout)
    torch.cuda.synchronize()
    qo, sfo = oracle.quantize_mx(x, fmt)
    assert np.array_equal(q.cpu().numpy(), qo)
    want = to_blocked(sfo) if layout == 1 else sfo
    assert np.array_equal(sf.cpu().numpy().ravel(), want.ravel())


def _random_operand(oracle, rng, name, rows, K):
    """Random codes over every finite value of the format, packed; scales 2^-4 .. 2^4."""
    t, fmt, mask = TYPES[name]
    codes = (rng.integers(0, 256, (rows, K)) & mask).astype(np.uint8)
    if name == "e4m3":
        codes[(codes & 0x7F) == 0x7F] = 0x3E
    if name == "e5m2":
        codes[(codes & 0x7C) == 0x7C] = 0x3C
    sf = rng.integers(123, 132, (rows, K // 32), dtype=np.uint8)
    return oracle.mx_pack(fmt, codes), sf


def _gemm_check(torch, oracle, A, ta, sfA, B, tb, sfB, n_samples=2048, seed=0):
    import ptxstd
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    M, N = A.shape[0], B.shape[0]
    C = ptxstd.gemm_mx(dev(A), TYPES[ta][0], dev(to_blocked(sfA)), dev(B), TYPES[tb][0],
                       dev(to_blocked(sfB)))
    torch.cuda.synchronize()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    Cg = C.float().cpu().numpy()
    rng = np.random.default_rng(seed)
    rows = np.concatenate([rng.integers(0, M, n_samples), np.arange(M), np.full(N, M - 1)])
    cols = np.concatenate([rng.integers(0, N, n_samples), np.full(M, N - 1), np.arange(N)])
    ref, mag = oracle.gemm_mx_ref(A, TYPES[ta][1], sfA, B, TYPES[tb][1], sfB, rows, cols)
    got = Cg[rows, cols].astype(np.float64)
    tol = 2.0 ** -10 * mag + 2.0 ** -8 * np.abs(ref)
    bad = np.nonzero(~(np.abs(got - ref) <= tol))[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i]) for i in bad[:6]]


# every (A, B) pair of kind::mxf8f6f4 element types
PAIRS = [(ta, tb) for ta in TYPES for tb in TYPES]


@pytest.mark.parametrize("ta,tb", PAIRS)
def test_gemm_mx_random_codes(cuda, oracle, ta, tb):
    rng = np.random.default_rng(16 * TYPES[ta][0] + TYPES[tb][0])
    M, N, K = 256, 512, 1024
    A, sfA = _random_operand(oracle, rng, ta, M, K)
    B, sfB = _random_operand(oracle, rng, tb, N, K)
    _gemm_check(cuda, oracle, A, ta, sfA, B, tb, sfB)


@pytest.mark.parametrize("ta,tb", [("e2m3", "e2m3"), ("e3m2", "e2m1"), ("e2m1", "e4m3")])
def test_quantize_then_gemm_mx(cuda, oracle, ta, tb):
    """The quantiser's payload and blocked scales feed the GEMM as they are."""
    torch = cuda
    import ptxstd
    from ptxstd import workloads
    M, N, K = 512, 256, 2048
    xa = workloads.normal_bf16(M, K, seed=51)
    xb = workloads.normal_bf16(N, K, seed=52)
    dev = lambda a: torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)  # noqa: E731
    qa, sfa = ptxstd.quantize_mx(dev(xa), ta, sf_layout=1)
    qb, sfb = ptxstd.quantize_mx(dev(xb), tb, sf_layout=1)
    C = ptxstd.gemm_mx(qa, ta, sfa, qb, tb, sfb)
    torch.cuda.synchronize()
    Ao, sfAo = oracle.quantize_mx(xa, TYPES[ta][1])
    Bo, sfBo = oracle.quantize_mx(xb, TYPES[tb][1])
    assert np.array_equal(qa.cpu().numpy(), Ao) and np.array_equal(qb.cpu().numpy(), Bo)
    rng = np.random.default_rng(3)
    rows, cols = rng.integers(0, M, 3000), rng.integers(0, N, 3000)
    ref, mag = oracle.gemm_mx_ref(Ao, TYPES[ta][1], sfAo, Bo, TYPES[tb][1], sfBo, rows, cols)
    got = C.float().cpu().numpy()[rows, cols].astype(np.float64)
    assert (np.abs(got - ref) <= 2.0 ** -10 * mag + 2.0 ** -8 * np.abs(ref)).all()


@pytest.mark.parametrize("name", ["e2m3", "e3m2", "e2m1"])
def test_tcgen05_cp_decompression(cuda, oracle, name):
    """tcgen05.cp .b8x16.b6x16_p32 / .b8x16.b4x16_p64 on every code: each packed element lands in
    its own 8-bit container, in order: an FP6 code in bits 5..0, an FP4 code in bits 5..2 (as an
    E2M3-aligned value), the other bits zero."""
    torch = cuda
    import ptxstd
    t, fmt, mask = TYPES[name]
    rows = 128 * 8
    rng = np.random.default_rng(90 + t)
    codes = (rng.integers(0, 256, (rows, 32)) & mask).astype(np.uint8)
    codes[0, :] = np.arange(32) & mask                      # a known row
    packed = oracle.mx_pack(fmt, codes)
    got = ptxstd.tcgen05_cp_unpack(torch.from_numpy(packed).cuda(), name).cpu().numpy()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    want = oracle.cp_unpack(fmt, packed)
    assert np.array_equal(got, want), (got[0].tobytes().hex(), want[0].tobytes().hex(),
                                       packed[0].tobytes().hex())

"""MXFP8 block-scaled GEMM (tcgen05.mma.kind::mxf8f6f4.block_scale.block32) vs the oracle (B200).

Operands are E4M3 codes with UE8M0 scales per 32 K elements; the scales are rearranged into the
blocked 128x4 layout in numpy (or come straight from ptxstd.quantize_mxfp8 with sf_layout 1), and
the device result is compared with the oracle's f64 GEMM over the decoded values:
  |C - ref| <= 2^-10 * sum_k |a b|  +  half an ulp of bf16 at C,
i.e. the f32 accumulator is within the accumulation bound and C is its bf16 rounding. The
rounding term cannot be dropped here, even at K = 8192 with random signs: the block scales span
2^-5 .. 2^5, so a few 32-element blocks whose two scales are both near the top carry most of
sum |a b|, and |ref| can reach over half of it (0.60 in a 512 x 512 numpy trial of these
operands, where the bf16 rounding of the exact result alone reached 1.8 x the plain bound).
Structured cases isolate the scale layout: per-row A scales, per-K-block A scales (each of the four
MMAs of a stage reads its own scale byte), per-column B scales; random cases cover several tile
counts, a quantise -> GEMM chain and a sampled 8192-cube.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ACC = 2.0 ** -10
ONE = 0x38  # E4M3 1.0


def to_blocked(sf: np.ndarray) -> np.ndarray:
    """Row-major [rows, S] scales -> the blocked 128x4 layout (rows % 128 == 0, S % 4 == 0)."""
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _run(torch, A, sfA, B, sfB):
    import ptxstd
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    c = ptxstd.gemm_mxfp8(dev(A), dev(to_blocked(sfA)), dev(B), dev(to_blocked(sfB)))
    torch.cuda.synchronize()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    return c.float().cpu().numpy()


def _half_ulp_bf16(c: np.ndarray) -> np.ndarray:
    """Half an ulp of bf16 (8 significant bits) at each value of c (2^-134 at zero)."""
    e = np.floor(np.log2(np.maximum(np.abs(c), 2.0 ** -126)))
    return np.exp2(e - 8)


def _check(oracle, A, sfA, B, sfB, Cg, rows, cols):
    """Checks the sampled outputs; prints and returns the largest err / tolerance."""
    ref, mag = oracle.gemm_mxfp8_ref(A, sfA, B, sfB, rows, cols)
    got = Cg[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    tol = TOL_ACC * mag + _half_ulp_bf16(got)
    bad = np.nonzero(~(err <= tol))[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i]) for i in bad[:8]]
    ratio = float((err / np.maximum(tol, 1e-300)).max())
    print(f"max err / (2^-10 sum|ab| + half ulp) = {ratio:.4f} over {rows.size} outputs")
    return ratio


def _bf16(x: float) -> float:
    """x rounded to bf16 (round to nearest even), as a float."""
    u = int(np.array([x], dtype=np.float32).view(np.uint32)[0])
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return float(np.array([u], dtype=np.uint32).view(np.float32)[0])


def _all(M, N):
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    return r.ravel(), c.ravel()


def _operands(M, N, K, seed, lo=122, hi=133):
    from ptxstd import workloads
    rng = np.random.default_rng(seed)
    A = workloads.fp8_operand(M, K, seed)
    B = workloads.fp8_operand(N, K, seed + 1)
    sfA = rng.integers(lo, hi, (M, K // 32), dtype=np.uint8)
    sfB = rng.integers(lo, hi, (N, K // 32), dtype=np.uint8)
    return A, sfA, B, sfB


def test_row_scales(cuda, oracle):
    M, N, K = 256, 256, 256
    A = np.full((M, K), ONE, dtype=np.uint8)
    B = np.full((N, K), ONE, dtype=np.uint8)
    sfA = np.repeat((127 + (np.arange(M) % 9) - 4).astype(np.uint8)[:, None], K // 32, axis=1)
    sfB = np.full((N, K // 32), 127, dtype=np.uint8)
    C = _run(cuda, A, sfA, B, sfB)
    want = K * np.exp2((np.arange(M) % 9) - 4.0)
    assert np.array_equal(C, np.repeat(want[:, None], N, axis=1))


def test_kblock_scales(cuda, oracle):
    """Each 32-element K block of A has its own scale: every MMA must read its own scale byte."""
    M, N, K = 256, 256, 512
    A = np.full((M, K), ONE, dtype=np.uint8)
    B = np.full((N, K), ONE, dtype=np.uint8)
    blocks = K // 32
    e = (np.arange(blocks) % 7) - 3  # exponents -3..3
    sfA = np.repeat((127 + e).astype(np.uint8)[None, :], M, axis=0)
    sfB = np.full((N, blocks), 127, dtype=np.uint8)
    C = _run(cuda, A, sfA, B, sfB)
    assert np.all(C == _bf16(32.0 * np.exp2(e.astype(np.float64)).sum()))
    # a distinct weight per block within one stage (4 blocks x 32 = 128 K): catches byte swaps
    e2 = np.array([0, 1, 2, 3] * (blocks // 4))
    sfA2 = np.repeat((127 + e2).astype(np.uint8)[None, :], M, axis=0)
    A2 = np.zeros((M, K), dtype=np.uint8)
    for st in range(K // 128):
        A2[:, st * 128 + 32:st * 128 + 64] = ONE  # only the second block of every stage
    C2 = _run(cuda, A2, sfA2, B, sfB)
    assert np.all(C2 == 32.0 * 2.0 * (blocks // 4))


def test_col_scales(cuda, oracle):
    M, N, K = 256, 512, 256
    A = np.full((M, K), ONE, dtype=np.uint8)
    B = np.full((N, K), ONE, dtype=np.uint8)
    sfA = np.full((M, K // 32), 127, dtype=np.uint8)
    e = (np.arange(N) % 11) - 5
    sfB = np.repeat((127 + e).astype(np.uint8)[:, None], K // 32, axis=1)
    C = _run(cuda, A, sfA, B, sfB)
    assert np.array_equal(C, np.repeat((K * np.exp2(e.astype(np.float64)))[None, :], M, axis=0))


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (256, 512, 512), (512, 256, 1024),
                                   (768, 512, 384)])
def test_random_all_outputs(cuda, oracle, M, N, K):
    A, sfA, B, sfB = _operands(M, N, K, seed=M + N + K)
    C = _run(cuda, A, sfA, B, sfB)
    _check(oracle, A, sfA, B, sfB, C, *_all(M, N))


def test_nan_scale_propagates(cuda, oracle):
    M, N, K = 256, 256, 256
    A, sfA, B, sfB = _operands(M, N, K, seed=5)
    sfA[3, 2] = 0xFF  # UE8M0 NaN
    C = _run(cuda, A, sfA, B, sfB)
    assert np.isnan(C[3]).all()
    assert np.isfinite(np.delete(C, 3, axis=0)).all()


def test_quantize_then_gemm(cuda, oracle):
    """bf16 -> ptxstd.quantize_mxfp8(sf_layout=1) -> ptxstd.gemm_mxfp8, no relayout in between."""
    import ptxstd
    from ptxstd import workloads
    torch = cuda
    M, N, K = 512, 512, 1024
    xa = workloads.mxfp8_activation(M, K, seed=61)
    xb = workloads.mxfp8_activation(N, K, seed=62)
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda().view(torch.bfloat16)  # noqa: E731,E501
    qa, sa = ptxstd.quantize_mxfp8(dev(xa), sf_layout=1)
    qb, sb = ptxstd.quantize_mxfp8(dev(xb), sf_layout=1)
    C = ptxstd.gemm_mxfp8(qa, sa, qb, sb)
    torch.cuda.synchronize()
    Ao, sAo = oracle.quantize_mxfp8(xa)
    Bo, sBo = oracle.quantize_mxfp8(xb)
    assert np.array_equal(qa.cpu().numpy(), Ao) and np.array_equal(qb.cpu().numpy(), Bo)
    _check(oracle, Ao, sAo, Bo, sBo, C.float().cpu().numpy(), *_all(M, N))


def test_cube_8192_sampled(cuda, oracle):
    M = N = K = 8192
    A, sfA, B, sfB = _operands(M, N, K, seed=77)
    C = _run(cuda, A, sfA, B, sfB)
    rng = np.random.default_rng(78)
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, 4321), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.full(M, 8000)])
    _check(oracle, A, sfA, B, sfB, C, rows, cols)


def test_rejects_bad_shapes(cuda):
    import ptxstd
    torch = cuda
    L = ptxstd.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    for M, N, K in [(128, 256, 128), (256, 128, 128), (256, 256, 64), (0, 256, 128)]:
        assert L.ptxstd_gemm_mxfp8(p, p, p, p, p, M, N, K, None) == 1  # PTXSTD_EINVAL
    assert L.ptxstd_gemm_mxfp8(p + 8, p, p, p, p, 256, 256, 128, None) == 1

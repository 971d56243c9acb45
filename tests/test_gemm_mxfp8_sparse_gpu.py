"""2:4-sparse MXFP8 GEMM (tcgen05.mma.sp kind::mxf8f6f4 .block_scale) and 2:4 pruning vs the oracle
(B200).

A is pruned to 2:4 (the two largest magnitudes of every group of four) by ptxstd.prune_24 and
compared bit for bit with the oracle's pruning; the GEMM takes the compressed values, the metadata
nibbles and one UE8M0 scale per 64 logical K for each operand (blocked 128x4 layout) and is
compared with the oracle's f64 GEMM over the decompressed operands:
  |C - ref| <= 2^-10 * sum_k |a b|  +  2^-8 * |ref|   (the second term: bf16 output rounding).
Structured scale cases isolate the scale slots (per-row, per-64-K-block, per-column); the sparse
GEMM also agrees with the dense MXFP8 GEMM run on the decompressed A.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ACC = 2.0 ** -10
TOL_OUT = 2.0 ** -8


def to_blocked(sf: np.ndarray) -> np.ndarray:
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _codes(rng, rows, cols):
    """Random finite E4M3 codes (no NaN), random signs."""
    mag = rng.integers(0, 0x7F, (rows, cols))
    return (mag | (rng.integers(0, 2, (rows, cols)) << 7)).astype(np.uint8)


def _dev(torch, x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def _run(torch, vals, meta, sfA, B, sfB):
    import ptxstd
    c = ptxstd.gemm_mxfp8_sparse(_dev(torch, vals), _dev(torch, meta), _dev(torch, to_blocked(sfA)),
                                 _dev(torch, B), _dev(torch, to_blocked(sfB)))
    torch.cuda.synchronize()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    return c.float().cpu().numpy()


def _check(oracle, vals, meta, sfA, B, sfB, C, rows, cols):
    ref, mag = oracle.gemm_mxfp8_sparse_ref(vals, meta, sfA, B, sfB, rows, cols)
    got = C[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    bad = np.nonzero(err > TOL_ACC * mag + TOL_OUT * np.abs(ref))[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i], mag[i]) for i in bad[:8]]


def _case(oracle, rng, M, N, K, sf_lo=122, sf_hi=132):
    A = _codes(rng, M, K)
    vals, meta = oracle.prune_24(A)
    B = _codes(rng, N, K)
    sfA = rng.integers(sf_lo, sf_hi, (M, K // 64)).astype(np.uint8)
    sfB = rng.integers(sf_lo, sf_hi, (N, K // 64)).astype(np.uint8)
    return vals, meta, sfA, B, sfB


def test_prune_matches_oracle(cuda, oracle):
    import ptxstd
    torch = cuda
    rng = np.random.default_rng(1)
    for rows, cols in [(256, 1024), (3, 8), (17, 40)]:
        A = rng.integers(0, 256, (rows, cols)).astype(np.uint8)   # NaN codes included
        A[0, :8] = [5, 5, 5, 5, 0x80, 0x00, 0x7F, 0xFF]           # ties, -0/+0, both NaNs
        v, m = ptxstd.prune_24(_dev(torch, A))
        wv, wm = oracle.prune_24(A)
        assert np.array_equal(v.cpu().numpy(), wv) and np.array_equal(m.cpu().numpy(), wm)


def test_sparse_gemm_all_outputs(cuda, oracle):
    rng = np.random.default_rng(2)
    vals, meta, sfA, B, sfB = _case(oracle, rng, 256, 256, 256)
    C = _run(cuda, vals, meta, sfA, B, sfB)
    r, c = np.meshgrid(np.arange(256), np.arange(256), indexing="ij")
    _check(oracle, vals, meta, sfA, B, sfB, C, r.ravel(), c.ravel())


@pytest.mark.parametrize("M,N,K", [(512, 768, 1024), (256, 512, 2048), (768, 256, 512)])
def test_sparse_gemm_shapes(cuda, oracle, M, N, K):
    rng = np.random.default_rng(M + N + K)
    vals, meta, sfA, B, sfB = _case(oracle, rng, M, N, K)
    C = _run(cuda, vals, meta, sfA, B, sfB)
    rows = np.concatenate([rng.integers(0, M, 2048), np.full(N, M - 1), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 2048), np.arange(N), np.full(M, N - 1)])
    _check(oracle, vals, meta, sfA, B, sfB, C, rows, cols)


@pytest.mark.parametrize("which", ["a_rows", "a_kblocks", "b_cols", "b_kblocks"])
def test_scale_slots(cuda, oracle, which):
    """Powers of two that differ along one axis only: each of the four MMAs of a stage must read
    its own scale byte, each row / column its own lane."""
    rng = np.random.default_rng(3)
    M = N = 256
    K = 1024
    vals, meta, _, B, _ = _case(oracle, rng, M, N, K)
    sfA = np.full((M, K // 64), 127, np.uint8)
    sfB = np.full((N, K // 64), 127, np.uint8)
    if which == "a_rows":
        sfA[:] = (120 + np.arange(M) % 16)[:, None]
    elif which == "a_kblocks":
        sfA[:] = (120 + np.arange(K // 64) % 16)[None, :]
    elif which == "b_cols":
        sfB[:] = (120 + np.arange(N) % 16)[:, None]
    else:
        sfB[:] = (120 + (np.arange(K // 64) * 5) % 16)[None, :]
    C = _run(cuda, vals, meta, sfA, B, sfB)
    r, c = np.meshgrid(np.arange(0, M, 3), np.arange(0, N, 5), indexing="ij")
    _check(oracle, vals, meta, sfA, B, sfB, C, r.ravel(), c.ravel())


def test_agrees_with_dense_gemm(cuda, oracle):
    """The dense MXFP8 GEMM over the decompressed A (each 64-scale repeated for both 32-blocks)
    gives the same products; the two results differ at most by accumulation order."""
    import ptxstd
    torch = cuda
    rng = np.random.default_rng(4)
    M, N, K = 256, 512, 1024
    vals, meta, sfA, B, sfB = _case(oracle, rng, M, N, K)
    Cs = _run(torch, vals, meta, sfA, B, sfB)
    Ad = oracle.decompress_24(vals, meta)
    Cd = ptxstd.gemm_mxfp8(_dev(torch, Ad), _dev(torch, to_blocked(np.repeat(sfA, 2, axis=1))),
                           _dev(torch, B), _dev(torch, to_blocked(np.repeat(sfB, 2, axis=1))))
    Cd = Cd.float().cpu().numpy()
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    ref, mag = oracle.gemm_mxfp8_sparse_ref(vals, meta, sfA, B, sfB, r.ravel(), c.ravel())
    tol = 2 * (TOL_ACC * mag + TOL_OUT * np.abs(ref))
    assert np.all(np.abs(Cs.ravel().astype(np.float64) - Cd.ravel()) <= tol)


def test_full_size_sampled(cuda, oracle):
    """8192^3 (logical K), sampled outputs plus a whole row and column."""
    rng = np.random.default_rng(5)
    M = N = K = 8192
    vals, meta, sfA, B, sfB = _case(oracle, rng, M, N, K)
    C = _run(cuda, vals, meta, sfA, B, sfB)
    rows = np.concatenate([rng.integers(0, M, 2048), np.full(N, 4097), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 2048), np.arange(N), np.full(M, 8191)])
    _check(oracle, vals, meta, sfA, B, sfB, C, rows, cols)


def test_bad_shapes(cuda):
    import ptxstd
    torch = cuda
    L = ptxstd.lib()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    assert L.ptxstd_gemm_mxfp8_sparse(p, p, p, p, p, p, 256, 256, 128, None) == ptxstd.EINVAL
    assert L.ptxstd_gemm_mxfp8_sparse(p, p, p, p, p, p, 128, 256, 256, None) == ptxstd.EINVAL
    assert L.ptxstd_gemm_mxfp8_sparse(p + 8, p, p, p, p, p, 256, 256, 256, None) == ptxstd.EINVAL
    assert L.ptxstd_prune_24_e4m3(p, 4, 12, p, p, None) == ptxstd.EINVAL

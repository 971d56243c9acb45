"""FP8 E4M3 GEMM (tcgen05.mma.kind::f8f6f4) vs the oracle's f64 GEMM over decoded values (B200).

Tolerance, per output: |C - ref| <= 2^-10 * sa*sb*sum_k |a_ik b_jk|  +  2^-8 * |ref|.
The first term is the stated accumulation bound; the second is the bf16 rounding of the output
(half an ulp of bf16 is at most 2^-8 relative), which the stated bound does not include.
Small shapes are checked at every output; the 8192^3 workload at 4096 random outputs plus two
full rows and two full columns.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ACC = 2.0 ** -10
TOL_OUT = 2.0 ** -8


def _run(torch, A, B, sa, sb):
    import ptxstd
    a = torch.from_numpy(A).cuda()
    b = torch.from_numpy(B).cuda()
    c = ptxstd.gemm_fp8(a, b, sa, sb)
    torch.cuda.synchronize()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    return c.float().cpu().numpy()


def _check(oracle, A, B, sa, sb, Cg, rows, cols):
    ref, mag = oracle.gemm_fp8_ref(A, B, sa, sb, rows, cols)
    got = Cg[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    tol = TOL_ACC * mag + TOL_OUT * np.abs(ref)
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i], mag[i]) for i in bad[:8]]
    return float((err / np.maximum(mag, 1e-30)).max())


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (128, 256, 1024), (256, 512, 256),
                                   (384, 768, 640), (1024, 1024, 2048)])
def test_small_all_outputs(cuda, oracle, M, N, K):
    from ptxstd import workloads
    A = workloads.fp8_operand(M, K, seed=M + K)
    B = workloads.fp8_operand(N, K, seed=N + 7 * K)
    Cg = _run(cuda, A, B, 0.75, 1.25)
    rows, cols = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    _check(oracle, A, B, 0.75, 1.25, Cg, rows.ravel(), cols.ravel())


def test_identity_structure(cuda, oracle):
    """A = identity blocks (1.0 = 0x38), B random: C must reproduce B^T exactly (one term)."""
    from ptxstd import workloads
    M = N = K = 256
    A = np.zeros((M, K), dtype=np.uint8)
    A[np.arange(M), np.arange(K)] = 0x38
    B = workloads.fp8_operand(N, K, seed=99)
    Cg = _run(cuda, A, B, 1.0, 1.0)
    want = oracle.decode(0, B.ravel()).reshape(N, K).T
    assert np.array_equal(Cg, want.astype(np.float32))


def test_full_size_sampled(cuda, oracle):
    from ptxstd import workloads
    M = N = K = 8192
    A = workloads.fp8_operand(M, K, seed=31)
    B = workloads.fp8_operand(N, K, seed=32)
    Cg = _run(cuda, A, B, 0.75, 1.25)
    rng = np.random.default_rng(5)
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, 17), np.full(N, M - 1),
                           np.arange(M), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.arange(N),
                           np.full(M, 0), np.full(M, N - 129)])
    _check(oracle, A, B, 0.75, 1.25, Cg, rows, cols)


def test_rejects_bad_shapes(cuda):
    import ptxstd
    torch = cuda
    a = torch.zeros((100, 128), dtype=torch.uint8, device="cuda")
    b = torch.zeros((256, 128), dtype=torch.uint8, device="cuda")
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.gemm_fp8(a, b)

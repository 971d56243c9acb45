"""FP8 E4M3 GEMM (tcgen05.mma.kind::f8f6f4) vs the oracle's f64 GEMM over decoded values (B200).

The 8192^3 workload (random signs) is held to the plain accumulation bound, per output
  |C - ref| <= 2^-10 * sa*sb*sum_k |a_ik b_jk|,
at 4096 random outputs plus two full rows and two full columns; with random signs at K = 8192,
|ref| stays a small fraction of sum |a b| (under 0.18 in a 512 x 512 numpy trial of these
operands), so the bound also covers the bf16 rounding of the output. Small shapes (K down to 128)
are checked at every output with the bf16 rounding added, 2^-8 * |ref| (half an ulp of bf16,
relative): there a few large products can make |ref| close to sum |a b|, and the rounding of a
correct result alone can then exceed the plain bound.
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


def _check(oracle, A, B, sa, sb, Cg, rows, cols, plain=False):
    """Checks the sampled outputs; plain=True drops the output-rounding term. Prints and returns
    the largest err / (2^-10 * sum |a b|)."""
    ref, mag = oracle.gemm_fp8_ref(A, B, sa, sb, rows, cols)
    got = Cg[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    tol = TOL_ACC * mag + (0.0 if plain else TOL_OUT * np.abs(ref))
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i], mag[i]) for i in bad[:8]]
    ratio = float((err / np.maximum(TOL_ACC * mag, 1e-300)).max())
    print(f"max err / (2^-10 sum|ab|) = {ratio:.4f} over {rows.size} outputs")
    return ratio


@pytest.mark.parametrize("M,N,K", [(128, 256, 128), (128, 256, 1024), (256, 512, 256),
                                   (384, 768, 640), (512, 256, 128), (1536, 768, 384),
                                   (1024, 1024, 2048)])
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
    _check(oracle, A, B, 0.75, 1.25, Cg, rows, cols, plain=True)


def test_rejects_bad_shapes(cuda):
    import ptxstd
    torch = cuda
    a = torch.zeros((100, 128), dtype=torch.uint8, device="cuda")
    b = torch.zeros((256, 128), dtype=torch.uint8, device="cuda")
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.gemm_fp8(a, b)

"""NVFP4 block-scaled GEMM (tcgen05.mma.kind::mxf4nvf4.block_scale.block16) vs the oracle (B200).

Operands are built on the CPU (the oracle's NVFP4 quantiser, row-major scales), the scales are
rearranged into the blocked 128x4 layout in numpy, and the device result is compared with the
oracle's f64 GEMM over the decoded values. The MLP up-projection shape (M = 8192, N = 28672,
K = 8192, random signs) is held to the plain accumulation bound
  |C - ref| <= 2^-10 * ga*gb*sum_k |a b|,
which also covers the bf16 rounding of the output there: with random signs |ref| is a small
fraction of sum |a b| at K = 8192. The small random shapes (K down to 256) add the bf16 rounding
of the output, 2^-8 * |ref| (half an ulp of bf16, relative): at small K a few large products can
make |ref| close to sum |a b|, and then the rounding of a correct result alone can exceed the
plain bound. Structured cases isolate the scale layout (per-row A scales, per-K-block A scales,
per-column B scales) and are checked exactly.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ACC = 2.0 ** -10
TOL_OUT = 2.0 ** -8


@pytest.fixture(autouse=True, params=[0, 1], ids=["persistent", "dynamic"])
def schedule(request, ptxstd_lib):
    """Every case runs under both tile schedules of the CTA-pair kernel: the persistent raster
    and the cluster-launch-control schedule (one cluster per tile, tiles taken over)."""
    ptxstd_lib.set_gemm_schedule(request.param)
    yield request.param
    ptxstd_lib.set_gemm_schedule(0)


def to_blocked(sf: np.ndarray) -> np.ndarray:
    """Row-major [rows, S] scales -> the blocked 128x4 layout (rows % 128 == 0, S % 4 == 0)."""
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _run(torch, A, sfA, ga, B, sfB, gb):
    import ptxstd
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).cuda()  # noqa: E731
    c = ptxstd.gemm_nvfp4(dev(A), dev(to_blocked(sfA)), ga, dev(B), dev(to_blocked(sfB)), gb)
    torch.cuda.synchronize()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    return c.float().cpu().numpy()


def _check(oracle, A, sfA, ga, B, sfB, gb, Cg, rows, cols, plain=False):
    """Checks the sampled outputs; plain=True drops the output-rounding term. Prints and returns
    the largest err / (2^-10 * sum |a b|)."""
    ref, mag = oracle.gemm_nvfp4_ref(A, sfA, ga, B, sfB, gb, rows, cols)
    got = Cg[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    tol = TOL_ACC * mag + (0.0 if plain else TOL_OUT * np.abs(ref))
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i]) for i in bad[:8]]
    ratio = float((err / np.maximum(TOL_ACC * mag, 1e-300)).max())
    print(f"max err / (2^-10 sum|ab|) = {ratio:.4f} over {rows.size} outputs")
    return ratio


def _all(M, N):
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    return r.ravel(), c.ravel()


def _ones(rows, K):
    return np.full((rows, K // 2), 0x22, dtype=np.uint8)  # E2M1 1.0 in both nibbles


@pytest.mark.parametrize("M", [128, 256])
def test_row_scales(cuda, oracle, M):
    """A = B = 1, sfA[m, :] = 2^(m % 8 - 4), sfB = 1: C[m, n] = K * sfA(m).
    M = 256 runs the CTA-pair kernel (rows 128..255 come from the second CTA)."""
    N, K = 256, 256
    A, B = _ones(M, K), _ones(N, K)
    e = (np.arange(M) % 8) - 4 + (np.arange(M) >= 128)
    sfA = np.repeat((0x38 + 8 * e).astype(np.uint8)[:, None], K // 16, axis=1)
    sfB = np.full((N, K // 16), 0x38, dtype=np.uint8)
    Cg = _run(cuda, A, sfA, 1.0, B, sfB, 1.0)
    want = K * 2.0 ** e[:, None] * np.ones((1, N))
    assert np.array_equal(Cg, want.astype(np.float32)), np.argwhere(Cg != want)[:8]


@pytest.mark.parametrize("M", [128, 256])
def test_k_block_scales(cuda, oracle, M):
    """sfA[m, s] = 2^(s % 4), sfB[n, s] = 2^((s // 4) % 4): each K block weighs differently."""
    N, K = 256, 1024
    A, B = _ones(M, K), _ones(N, K)
    s = np.arange(K // 16)
    sfA = np.repeat((0x38 + 8 * (s % 4)).astype(np.uint8)[None, :], M, axis=0)
    sfB = np.repeat((0x38 + 8 * ((s // 4) % 4)).astype(np.uint8)[None, :], N, axis=0)
    Cg = _run(cuda, A, sfA, 1.0, B, sfB, 1.0)
    want = float(np.sum(16 * 2.0 ** (s % 4) * 2.0 ** ((s // 4) % 4)))
    assert np.all(Cg == want), (Cg[0, :4], want)


@pytest.mark.parametrize("M", [128, 256])
def test_col_scales(cuda, oracle, M):
    """sfB[n, :] = 2^(n % 14 - 6) (normal E4M3 powers of two): C[m, n] = K * sfB(n)."""
    N, K = 512, 256
    A, B = _ones(M, K), _ones(N, K)
    e = (np.arange(N) % 14) - 6
    sfA = np.full((M, K // 16), 0x38, dtype=np.uint8)
    sfB = np.repeat((0x38 + 8 * e).astype(np.uint8)[:, None], K // 16, axis=1)
    Cg = _run(cuda, A, sfA, 1.0, B, sfB, 1.0)
    want = K * 2.0 ** e[None, :] * np.ones((M, 1))
    assert np.array_equal(Cg, want.astype(np.float32)), np.argwhere(Cg != want)[:8]


def _operands(oracle, rows, K, seed, std=1.0):
    from ptxstd import workloads
    xb = workloads.normal_bf16(rows, K, std=std, seed=seed)
    xf = (xb.astype(np.uint32) << 16).view(np.float32)
    g = float(np.abs(xf).max() / (448.0 * 6.0))
    q, sf = oracle.quantize_nvfp4(xb, g)
    return q, sf, g


@pytest.mark.parametrize("M,N,K", [(128, 256, 256), (256, 512, 512), (384, 768, 1280),
                                   (1024, 1024, 2048)])
def test_random_all_outputs(cuda, oracle, M, N, K):
    A, sfA, ga = _operands(oracle, M, K, seed=M + K)
    B, sfB, gb = _operands(oracle, N, K, seed=N + 3 * K)
    Cg = _run(cuda, A, sfA, ga, B, sfB, gb)
    _check(oracle, A, sfA, ga, B, sfB, gb, Cg, *_all(M, N))


def test_mlp_up_projection_sampled(cuda, oracle):
    M, N, K = 8192, 28672, 8192
    A, sfA, ga = _operands(oracle, M, K, seed=41)
    B, sfB, gb = _operands(oracle, N, K, seed=42)
    Cg = _run(cuda, A, sfA, ga, B, sfB, gb)
    rng = np.random.default_rng(6)
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, 5), np.arange(M)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.full(M, N - 1)])
    _check(oracle, A, sfA, ga, B, sfB, gb, Cg, rows, cols, plain=True)

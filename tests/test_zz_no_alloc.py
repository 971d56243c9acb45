"""The allocation-free decode entry point against the regular one (B200).

ptxstd_gemm_decode_noalloc serves callers that cannot allocate device memory at call time (a
serving loop with a fixed memory plan, or a thin binding that owns no allocator); it keeps its
scratch in a fixed device array inside the library instead of a caller workspace. This test calls
it through the C ABI twice in a row (the array keeps the previous call's contents, so the second
call checks that each call re-initialises what it needs) and requires each result to equal
ptxstd_gemm_decode's on the same inputs bit for bit: both run the same kernels with the same
split of the work, and a weight block shared between CTAs is summed from their partials in a
fixed order, so the scratch's location and previous contents must not change a single bit. The
first result is also held to the GEMM tests' tolerance against the oracle. It also checks that a
shape whose scratch exceeds the array is rejected. The file sorts last so that a run stopping at
the first failure has already run every other test.
"""

import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ACC = 2.0 ** -10
TOL_OUT = 2.0 ** -8


def _blocked(sf):
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _noalloc_fn(ptxstd):
    fn = ptxstd.lib().ptxstd_gemm_decode_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_int64,
                   C.c_int64, C.c_int64, C.c_void_p]
    return fn


@pytest.mark.parametrize("M,N,K", [(16, 1024, 2048), (5, 57344, 8192)])
def test_noalloc_matches_regular_entry_point(cuda, oracle, M, N, K):
    import ptxstd
    from ptxstd import workloads
    torch = cuda
    x = workloads.normal_bf16(M, K, seed=101 + M)
    wb = workloads.normal_bf16(N, K, std=0.02, seed=202 + N)
    wf = (wb.astype(np.uint32) << 16).view(np.float32)
    gw = float(np.abs(wf).max() / (448.0 * 6.0))
    W, sfW = oracle.quantize_nvfp4(wb, gw)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    xd = dev(x.view(np.int16)).view(torch.bfloat16)
    Wd, sfd = dev(W), dev(_blocked(sfW))
    stream = torch.cuda.current_stream().cuda_stream

    want = ptxstd.gemm_decode(xd, Wd, sfd, gw).float().cpu().numpy()
    fn = _noalloc_fn(ptxstd)
    # sum_k |x w| per output, from the oracle, for the tolerance
    rng = np.random.default_rng(3)
    n_s = min(M * N, 8192)
    rows = rng.integers(0, M, n_s)
    cols = rng.integers(0, N, n_s)
    ref, mag = oracle.gemm_decode_ref(x, W, sfW, gw, rows, cols)
    a = want[rows, cols].astype(np.float64)
    assert (np.abs(a - ref) <= TOL_ACC * mag + TOL_OUT * np.abs(ref)).all()
    for call in range(2):
        y = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        st = fn(xd.data_ptr(), Wd.data_ptr(), sfd.data_ptr(), gw, y.data_ptr(), M, N, K, stream)
        assert st == 0, ptxstd.status_string(st)
        torch.cuda.synchronize()
        code, detail = ptxstd.last_device_error()
        assert code == 0, (code, hex(detail))
        got = y.float().cpu().numpy()
        assert np.isfinite(got).all(), call
        diff = np.argwhere(got != want)
        assert diff.size == 0, (call, diff[:8].tolist())


def test_noalloc_rejects_oversized_shape(cuda):
    import ptxstd
    torch = cuda
    M, N, K = 16, 128, 131072  # the 4 MiB x image alone fills the fixed array
    assert ptxstd.lib().ptxstd_gemm_decode_workspace_bytes(M, N, K) > (4 << 20)
    x = torch.zeros((M, K), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, K // 2), dtype=torch.uint8, device="cuda")
    y = torch.zeros((M, 128), dtype=torch.bfloat16, device="cuda")
    fn = _noalloc_fn(ptxstd)
    st = fn(x.data_ptr(), w.data_ptr(), w.data_ptr(), 1.0, y.data_ptr(), M, N, K,
            torch.cuda.current_stream().cuda_stream)
    assert st == ptxstd.EINVAL

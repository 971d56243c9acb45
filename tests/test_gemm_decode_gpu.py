"""Decode-shape GEMM (x bf16 -> MXFP8 in the call; NVFP4 weights) vs the oracle (B200).

The oracle quantises x with the MXFP8 recipe and takes an f64 dot product over the decoded
operands; tolerance per output: |y - ref| <= 2^-10 * sum_k |x w| + 2^-8 * |ref| (the second term:
bf16 rounding of the output). Covers M = 1, 5, 16 tokens, single and multiple 128-row weight
blocks, stage counts that split unevenly across CTAs, two calls in a row on one workspace, and
the N = 57344, K = 8192 decode workload at sampled outputs plus whole rows.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL_ACC = 2.0 ** -10
TOL_OUT = 2.0 ** -8


def to_blocked(sf):
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _weights(oracle, N, K, seed):
    from ptxstd import workloads
    wb = workloads.normal_bf16(N, K, std=0.02, seed=seed)
    wf = (wb.astype(np.uint32) << 16).view(np.float32)
    gw = float(np.abs(wf).max() / (448.0 * 6.0))
    W, sfW = oracle.quantize_nvfp4(wb, gw)
    return W, sfW, gw


def _run(torch, x, W, sfW, gw, calls=1):
    import ptxstd
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    xd = dev(x.view(np.int16)).view(torch.bfloat16)
    Wd, sfd = dev(W), dev(to_blocked(sfW))
    ys = []
    for _ in range(calls):
        ys.append(ptxstd.gemm_decode(xd, Wd, sfd, gw))
    torch.cuda.synchronize()
    code, detail = ptxstd.last_device_error()
    assert code == 0, (code, hex(detail))
    return [y.float().cpu().numpy() for y in ys]


def _check(oracle, x, W, sfW, gw, yg, rows, cols):
    ref, mag = oracle.gemm_decode_ref(x, W, sfW, gw, rows, cols)
    got = yg[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    tol = TOL_ACC * mag + TOL_OUT * np.abs(ref)
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i], mag[i]) for i in bad[:8]]


@pytest.mark.parametrize("M,N,K", [(16, 128, 256), (16, 256, 512), (5, 384, 1024),
                                   (1, 1024, 2048), (16, 2048, 4096), (16, 1152, 8192)])
def test_small_all_outputs(cuda, oracle, M, N, K):
    from ptxstd import workloads
    x = workloads.normal_bf16(M, K, seed=M + K)
    W, sfW, gw = _weights(oracle, N, K, seed=N + K)
    y1, y2 = _run(cuda, x, W, sfW, gw, calls=2)
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    _check(oracle, x, W, sfW, gw, y1, r.ravel(), c.ravel())
    # the second call on the same (re-initialised) workspace gives the same result
    assert np.allclose(y1, y2, rtol=2.0 ** -7, atol=0)


def test_scaled_rows(cuda, oracle):
    """Token rows with very different magnitudes (per-row 2^U(-8, 8), one x100 outlier)."""
    from ptxstd import workloads
    M, N, K = 16, 512, 2048
    x = workloads.mxfp8_activation(M, K, seed=77)
    W, sfW, gw = _weights(oracle, N, K, seed=78)
    (y,) = _run(cuda, x, W, sfW, gw)
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    _check(oracle, x, W, sfW, gw, y, r.ravel(), c.ravel())


def test_decode_workload_sampled(cuda, oracle):
    from ptxstd import workloads
    M, N, K = 16, 57344, 8192
    x = workloads.normal_bf16(M, K, seed=91)
    W, sfW, gw = _weights(oracle, N, K, seed=92)
    (y,) = _run(cuda, x, W, sfW, gw)
    rng = np.random.default_rng(9)
    rows = np.concatenate([rng.integers(0, M, 4096), np.full(N, 0), np.full(N, 15)])
    cols = np.concatenate([rng.integers(0, N, 4096), np.arange(N), np.arange(N)])
    _check(oracle, x, W, sfW, gw, y, rows, cols)


def test_rejects_bad_shapes(cuda):
    import ptxstd
    torch = cuda
    x = torch.zeros((17, 256), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, 128), dtype=torch.uint8, device="cuda")
    sf = torch.zeros((128 * 16,), dtype=torch.uint8, device="cuda")
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.gemm_decode(x, w, sf, 1.0)   # M > 16

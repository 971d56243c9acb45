"""Decode-shape GEMM (x bf16 -> MXFP8 in the call; NVFP4 weights) vs the oracle (B200).

The oracle quantises x with the MXFP8 recipe and takes an f64 dot product over the decoded
operands. The N = 57344, K = 8192 decode workload (N(0, 1) activations, N(0, 0.02) weights) is
held to the plain accumulation bound |y - ref| <= 2^-10 * sum_k |x w| at sampled outputs plus
whole rows: with random signs and K = 8192, |ref| is a small fraction of sum |x w|, so the bound
also covers the bf16 rounding of the output. The small shapes (K down to 256, and rows scaled by
up to 2^8 with a x100 outlier) add the bf16 rounding, 2^-8 * |ref| (half an ulp, relative): at
small K, or with one outlier product, |ref| can come close to sum |x w|, and the rounding of a
correct result alone can then exceed the plain bound. Covers M = 1, 5, 16 tokens, single and
multiple 128-row weight blocks, stage counts that split unevenly across CTAs, and two calls in a
row on one workspace.
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


def _check(oracle, x, W, sfW, gw, yg, rows, cols, plain=False):
    """Checks the sampled outputs; plain=True drops the output-rounding term. Prints and returns
    the largest err / (2^-10 * sum |x w|)."""
    ref, mag = oracle.gemm_decode_ref(x, W, sfW, gw, rows, cols)
    got = yg[rows, cols].astype(np.float64)
    err = np.abs(got - ref)
    tol = TOL_ACC * mag + (0.0 if plain else TOL_OUT * np.abs(ref))
    bad = np.nonzero(err > tol)[0]
    assert bad.size == 0, [(int(rows[i]), int(cols[i]), got[i], ref[i], mag[i]) for i in bad[:8]]
    ratio = float((err / np.maximum(TOL_ACC * mag, 1e-300)).max())
    print(f"max err / (2^-10 sum|xw|) = {ratio:.4f} over {rows.size} outputs")
    return ratio


@pytest.mark.parametrize("M,N,K", [(16, 128, 256), (16, 256, 512), (5, 384, 1024),
                                   (1, 1024, 2048), (16, 2048, 4096), (16, 1152, 8192)])
def test_small_all_outputs(cuda, oracle, M, N, K):
    from ptxstd import workloads
    x = workloads.normal_bf16(M, K, seed=M + K)
    W, sfW, gw = _weights(oracle, N, K, seed=N + K)
    y1, y2 = _run(cuda, x, W, sfW, gw, calls=2)
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    _check(oracle, x, W, sfW, gw, y1, r.ravel(), c.ravel())
    # the second call on the same workspace gives the same bits: a block shared between CTAs is
    # summed from their partials in a fixed order, whichever CTA finishes last
    assert np.array_equal(y1, y2)


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
    _check(oracle, x, W, sfW, gw, y, rows, cols, plain=True)


def test_rejects_bad_shapes(cuda):
    import ptxstd
    torch = cuda
    x = torch.zeros((17, 256), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((128, 128), dtype=torch.uint8, device="cuda")
    sf = torch.zeros((128 * 16,), dtype=torch.uint8, device="cuda")
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.gemm_decode(x, w, sf, 1.0)   # M > 16

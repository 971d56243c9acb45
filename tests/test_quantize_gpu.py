"""Quantise kernels vs the oracle, bit-exact (B200): payload bytes and scale bytes.

Covers the MXFP8 activation workload at full size (8192 x 8192 bf16, N(0,1) * 2^U(-8,8) per row,
every 64th row with a x100 outlier), both scale layouts, and the edge cases: all-zero blocks,
NaN / infinity inside a block, bf16 subnormals, values at the E4M3 saturation boundary, a single
row, the smallest legal width, and ragged row counts that leave a partial warp step.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _blocked_to_rowmajor(sf_blocked: np.ndarray, rows: int, sf_cols: int) -> np.ndarray:
    out = np.empty((rows, sf_cols), dtype=np.uint8)
    r = np.arange(rows)[:, None]
    s = np.arange(sf_cols)[None, :]
    off = ((r // 128) * (sf_cols // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out[:, :] = sf_blocked.reshape(-1)[off]
    return out


def _edge_matrix(rows, cols, seed):
    from ptxstd import workloads
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((rows, cols)) * np.exp2(rng.uniform(-8, 8, (rows, 1)))).astype(
        np.float32)
    xb = workloads._bf16(x)
    if rows >= 8 and cols >= 64:
        xb[0, :32] = 0                                      # all-zero block
        xb[1, 0] = 0x7FC0                                   # NaN in a block
        xb[2, 3] = 0x7F80                                   # +inf
        xb[3, 5] = 0xFF80                                   # -inf
        xb[4, :32] = rng.integers(1, 0x80, 32)              # bf16 subnormals only
        xb[5, :32] = workloads._bf16(np.full(32, 448.0 * 2 ** -3, np.float32))
        xb[5, 7] = workloads._bf16(np.array([479.0 * 2 ** -3], np.float32))[0]
        xb[6, 32:64] = workloads._bf16(np.float32(2.0 ** np.arange(-16, 16, dtype=np.float32)))
        xb[7, :16] = 0x8000                                 # -0
    return xb


def _check_mxfp8(torch, oracle, xb, layout):
    import ptxstd
    rows, cols = xb.shape
    q, sf = ptxstd.quantize_mxfp8(torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16),
                                  sf_layout=layout)
    wq, wsf = oracle.quantize_mxfp8(xb)
    gq = q.cpu().numpy()
    gsf = sf.cpu().numpy()
    if layout == 1:
        gsf = _blocked_to_rowmajor(gsf, rows, cols // 32)
    bad = np.argwhere(gq != wq)
    assert bad.shape[0] == 0, bad[:8]
    bad = np.argwhere(gsf != wsf)
    assert bad.shape[0] == 0, (bad[:8], gsf[tuple(bad[0])], wsf[tuple(bad[0])])


def _check_nvfp4(torch, oracle, xb, g, layout):
    import ptxstd
    rows, cols = xb.shape
    q, sf = ptxstd.quantize_nvfp4(torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16),
                                  g, sf_layout=layout)
    wq, wsf = oracle.quantize_nvfp4(xb, g)
    gq = q.cpu().numpy()
    gsf = sf.cpu().numpy()
    if layout == 1:
        gsf = _blocked_to_rowmajor(gsf, rows, cols // 16)
    bad = np.argwhere(gq != wq)
    assert bad.shape[0] == 0, bad[:8]
    bad = np.argwhere(gsf != wsf)
    assert bad.shape[0] == 0, bad[:8]


@pytest.mark.parametrize("layout", [0, 1])
def test_mxfp8_full_size(cuda, oracle, layout):
    from ptxstd import workloads
    xb = workloads.mxfp8_activation(8192, 8192)
    _check_mxfp8(cuda, oracle, xb, layout)


@pytest.mark.parametrize("shape", [(1, 32), (3, 96), (37, 160), (128, 128), (1000, 4096 + 32)])
def test_mxfp8_edges(cuda, oracle, shape):
    xb = _edge_matrix(*shape, seed=sum(shape))
    _check_mxfp8(cuda, oracle, xb, 0)


def test_mxfp8_blocked_edges(cuda, oracle):
    xb = _edge_matrix(256, 512, seed=11)
    _check_mxfp8(cuda, oracle, xb, 1)


@pytest.mark.parametrize("layout", [0, 1])
def test_nvfp4_operand(cuda, oracle, layout):
    from ptxstd import workloads
    xb = workloads.normal_bf16(2048, 8192, seed=21)
    xf = (xb.astype(np.uint32) << 16).view(np.float32)
    g = float(np.abs(xf).max() / (448.0 * 6.0))
    _check_nvfp4(cuda, oracle, xb, g, layout)


@pytest.mark.parametrize("shape", [(1, 16), (5, 48), (37, 160), (128, 128), (999, 1024 + 16)])
def test_nvfp4_edges(cuda, oracle, shape):
    xb = _edge_matrix(*shape, seed=7 + sum(shape))
    for g in (1.0, 1e-3, 2.0 ** -20, 37.5):
        _check_nvfp4(cuda, oracle, xb, g, 0)


def _check_rs(torch, oracle, xb, layout, seed, fmt, g=None):
    import ptxstd
    rows, cols = xb.shape
    xt = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    if fmt == "mxfp8":
        q, sf = ptxstd.quantize_mxfp8(xt, sf_layout=layout, seed=seed)
        wq, wsf = oracle.quantize_mxfp8_rs(xb, seed)
        per = 32
    else:
        q, sf = ptxstd.quantize_nvfp4(xt, g, sf_layout=layout, seed=seed)
        wq, wsf = oracle.quantize_nvfp4_rs(xb, g, seed)
        per = 16
    gq, gsf = q.cpu().numpy(), sf.cpu().numpy()
    if layout == 1:
        gsf = _blocked_to_rowmajor(gsf, rows, cols // per)
    bad = np.argwhere(gq != wq)
    assert bad.shape[0] == 0, (seed, bad[:8])
    assert np.array_equal(gsf, wsf)
    return gq


@pytest.mark.parametrize("layout", [0, 1])
def test_stochastic_quantize_vs_oracle(cuda, oracle, layout):
    """Seeded stochastic rounding (SplitMix64 bits per group of four): payload and scales
    bit-exact against the oracle, for edge-case matrices and several seeds; the scales equal the
    round-to-nearest scales; another seed changes the codes."""
    torch = cuda
    xb = _edge_matrix(256, 1024, 21)
    a = _check_rs(torch, oracle, xb, layout, 0, "mxfp8")
    b = _check_rs(torch, oracle, xb, layout, 2 ** 64 - 1, "mxfp8")
    assert not np.array_equal(a, b)
    _check_rs(torch, oracle, xb, layout, 12345, "nvfp4", g=0.05)
    _check_rs(torch, oracle, xb, layout, 7, "nvfp4", g=3.0e-4)


def test_stochastic_quantize_full_size(cuda, oracle):
    """The MXFP8 workload (8192 x 8192) with stochastic rounding, bit-exact."""
    from ptxstd import workloads
    xb = workloads.mxfp8_activation(8192, 8192)
    _check_rs(cuda, oracle, xb, 1, 0xC0FFEE, "mxfp8")


def test_invalid_arguments(cuda):
    import ptxstd
    torch = cuda
    x = torch.zeros((4, 40), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.quantize_mxfp8(x)           # cols % 32 != 0
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.quantize_nvfp4(x[:, :32].contiguous(), float("inf"))
    with pytest.raises(ptxstd.PtxStdError):
        ptxstd.quantize_mxfp8(torch.zeros((4, 128), dtype=torch.bfloat16, device="cuda"),
                              sf_layout=1)  # rows % 128 != 0


def test_back_to_back_calls_keep_stream_order(cuda, oracle):
    """The quantisers launch with programmatic dependent launch: a call may start on the SMs that
    the previous kernel of the stream frees, and waits (griddepcontrol.wait) before it reads x or
    writes q and sf. In one stream, with no synchronisation between the launches:
      - a call reads the x that the torch kernel just before it wrote (read after write);
      - the torch kernel just after a call overwrites that call's x (write after read);
      - two calls into the same outputs leave the second call's bytes (write after write).
    """
    torch = cuda
    import ptxstd
    rows, cols = 2048, 4096
    xb = [_edge_matrix(rows, cols, seed=71), _edge_matrix(rows, cols, seed=72)]
    xs = [torch.from_numpy(v.view(np.int16)).cuda().view(torch.bfloat16) for v in xb]
    want = [oracle.quantize_mxfp8(v) for v in xb]
    x = torch.empty_like(xs[0])
    n = 6
    qs = [torch.empty((rows, cols), dtype=torch.uint8, device="cuda") for _ in range(n)]
    sfs = [torch.empty((rows, cols // 32), dtype=torch.uint8, device="cuda") for _ in range(n)]
    qw = torch.empty((rows, cols), dtype=torch.uint8, device="cuda")
    sfw = torch.empty((rows, cols // 32), dtype=torch.uint8, device="cuda")
    for i in range(n):
        ptxstd.quantize_mxfp8(xs[(i + 1) % 2], out=(qw, sfw))
        x.copy_(xs[i % 2])
        ptxstd.quantize_mxfp8(x, out=(qs[i], sfs[i]))
        x.fill_(float("nan"))
        ptxstd.quantize_mxfp8(xs[i % 2], out=(qw, sfw))
    torch.cuda.synchronize()
    for i in range(n):
        assert np.array_equal(qs[i].cpu().numpy(), want[i % 2][0]), i
        assert np.array_equal(sfs[i].cpu().numpy(), want[i % 2][1]), i
    assert np.array_equal(qw.cpu().numpy(), want[(n - 1) % 2][0])
    assert np.array_equal(sfw.cpu().numpy(), want[(n - 1) % 2][1])

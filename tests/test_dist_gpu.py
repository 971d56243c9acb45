"""N-sharded GEMMs on two GPUs through libptxstd's NCCL layer (needs >= 2 B200s; skips otherwise).

Two spawned ranks (one per GPU) build the same seeded weights, keep their N shard, and run
  - ptxstd_gemm_decode_sharded: every rank must end with the full [M, N] output, equal to the
    single-GPU decode of the unsharded weights within the GEMM test tolerance;
  - ptxstd_gemm_nvfp4_sharded: each rank's C columns must equal, bit for bit, the same columns of
    the unsharded GEMM (the computation of a column does not depend on the sharding);
  - ptxstd_gemm_decode_sharded_p2p (the gather fused into the GEMM over NVLink peer memory): over
    consecutive steps, with M = 16 and M = 5, into the library-owned output and into a copy, and as
    replays of a captured CUDA graph fed new tokens, every rank's y must match the NCCL path of the
    same tokens within the GEMM test tolerance (the two differ only in the order of the fp32
    split-K additions);
  - failure detection of the peer-to-peer protocol: rank 0 runs a step that rank 1 never starts
    (a READY flag that nothing raises); its bounded waits must give up and report PTXSTD_ETIMEOUT
    naming the epilogue's READY wait, with the CUDA context still usable afterwards.
torch.distributed (gloo) only carries the NCCL unique id.
"""

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _blocked(sf):
    rows, S = sf.shape
    r = np.arange(rows)[:, None]
    s = np.arange(S)[None, :]
    off = ((r // 128) * (S // 4) + s // 4) * 512 + (r % 32) * 16 + ((r // 32) % 4) * 4 + s % 4
    out = np.empty(rows * S, dtype=np.uint8)
    out[off.ravel()] = sf.ravel()
    return out


def _worker(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "ptx-std_b200"), os.path.join(root, "oracle")]
    import torch
    import torch.distributed as td

    import oracle as O
    import ptxstd
    from ptxstd import workloads
    from ptxstd.dist import Dist, shard_range

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world)
    dist = Dist.from_torch()
    msgs = []
    M, N, K = 16, 512 * world, 2048  # 512 columns per rank
    x = workloads.normal_bf16(M, K, seed=21)
    wb = workloads.normal_bf16(N, K, std=0.02, seed=22)
    gw = float(np.abs((wb.astype(np.uint32) << 16).view(np.float32)).max() / (448.0 * 6.0))
    W, sfW = O.quantize_nvfp4(wb, gw)
    lo, hi = shard_range(N, world, rank)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    xd = dev(x.view(np.int16)).view(torch.bfloat16)
    y = dist.gemm_decode(xd, dev(W[lo:hi]), dev(_blocked(sfW[lo:hi])), gw, N)
    yfull = ptxstd.gemm_decode(xd, dev(W), dev(_blocked(sfW)), gw)
    torch.cuda.synchronize()
    a, b = y.float().cpu().numpy(), yfull.float().cpu().numpy()
    r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
    _, mag = O.gemm_decode_ref(x, W, sfW, gw, r.ravel(), c.ravel())
    tol = 2.0 ** -10 * mag.reshape(M, N) + 2.0 ** -8 * np.maximum(np.abs(a), np.abs(b))
    if not (np.abs(a - b) <= tol).all():
        msgs.append(f"rank {rank}: sharded decode differs")

    # peer-to-peer decode against the NCCL path of the same tokens
    wsh, sfsh = dev(W[lo:hi]), dev(_blocked(sfW[lo:hi]))

    xn = [workloads.normal_bf16(M, K, seed=30 + i) for i in range(4)]
    mags = [O.gemm_decode_ref(v, W, sfW, gw, r.ravel(), c.ravel())[1].reshape(M, N) for v in xn]
    xs = [dev(v.view(np.int16)).view(torch.bfloat16) for v in xn]

    def close(got, want, i, what, m=M):
        g, w_ = got.float().cpu().numpy(), want.float().cpu().numpy()
        t = 2.0 ** -10 * mags[i][:m] + 2.0 ** -8 * np.maximum(np.abs(g), np.abs(w_))
        if g.shape != w_.shape or not (np.abs(g - w_) <= t).all():
            msgs.append(f"rank {rank}: p2p decode differs ({what})")

    for i in range(2):
        yp = dist.gemm_decode_p2p(xs[i], wsh, sfsh, gw, N)
        yn = dist.gemm_decode(xs[i], wsh, sfsh, gw, N)
        torch.cuda.synchronize()
        close(yp, yn, i, f"step {i}")
    yc = torch.empty((5, N), dtype=torch.bfloat16, device="cuda")
    dist.gemm_decode_p2p(xs[2][:5].contiguous(), wsh, sfsh, gw, N, out=yc)
    yn = dist.gemm_decode(xs[2][:5].contiguous(), wsh, sfsh, gw, N)
    torch.cuda.synchronize()
    close(yc, yn, 2, "M = 5 copy", m=5)
    xg = xs[0].clone()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        yg = dist.gemm_decode_p2p(xg, wsh, sfsh, gw, N)
    for i in (3, 1):
        xg.copy_(xs[i])
        g.replay()
        yn = dist.gemm_decode(xs[i], wsh, sfsh, gw, N)
        torch.cuda.synchronize()
        close(yg, yn, i, f"graph replay {i}")
    del g

    Ma = 256
    A, sfA = O.quantize_nvfp4(workloads.normal_bf16(Ma, K, seed=23), 0.01)
    cs = dist.gemm_nvfp4(dev(A), dev(_blocked(sfA)), 0.01, dev(W[lo:hi]),
                         dev(_blocked(sfW[lo:hi])), gw, N)
    cf = ptxstd.gemm_nvfp4(dev(A), dev(_blocked(sfA)), 0.01, dev(W), dev(_blocked(sfW)), gw)
    torch.cuda.synchronize()
    if not torch.equal(cs, cf[:, lo:hi]):
        msgs.append(f"rank {rank}: sharded nvfp4 columns differ")
    code, _ = ptxstd.last_device_error()
    if code:
        msgs.append(f"rank {rank}: device error {code}")
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write("\n".join(msgs) if msgs else "ok")
    dist.close()
    td.barrier()
    td.destroy_process_group()


def _timeout_worker(rank, world, port, out_dir):
    import sys
    # a failure-detection test: no NVLink multicast (NVLS) objects in NCCL while a step is left
    # unfinished on purpose
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "ptx-std_b200"), os.path.join(root, "oracle")]
    import torch
    import torch.distributed as td

    import oracle as O
    import ptxstd
    from ptxstd import workloads
    from ptxstd.dist import Dist, shard_range

    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world)
    dist = Dist.from_torch()
    M, N, K = 16, 1024, 2048
    x = workloads.normal_bf16(M, K, seed=21)
    wb = workloads.normal_bf16(N, K, std=0.02, seed=22)
    W, sfW = O.quantize_nvfp4(wb, 1e-3)
    lo, hi = shard_range(N, world, rank)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    xd = dev(x.view(np.int16)).view(torch.bfloat16)
    wsh, sfsh = dev(W[lo:hi]), dev(_blocked(sfW[lo:hi]))
    dist.decode_p2p_output(N)
    ptxstd.last_device_error()
    msg = "ok"
    if rank == 0:
        dist.gemm_decode_p2p(xd, wsh, sfsh, 1e-3, N)  # rank 1 never starts this step
        torch.cuda.synchronize()
        code, detail = ptxstd.last_device_error()
        if code != ptxstd.ETIMEOUT or detail != 0x3540:
            msg = f"expected ETIMEOUT / 0x3540, got {code} / {detail:#x}"
        # the context is still usable
        y = ptxstd.gemm_decode(xd, dev(W), dev(_blocked(sfW)), 1e-3)
        torch.cuda.synchronize()
        if ptxstd.last_device_error()[0] != 0 or not torch.isfinite(y.float()).all():
            msg = "single-GPU decode after the timeout failed"
    with open(os.path.join(out_dir, f"rank{rank}"), "w") as f:
        f.write(msg)
    td.barrier()
    dist.close()
    td.barrier()
    td.destroy_process_group()


def test_p2p_decode_timeout_two_gpus(cuda, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_timeout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       join=True, start_method="spawn")
    for r in range(2):
        assert open(tmp_path / f"rank{r}").read() == "ok"


def test_sharded_two_gpus(cuda, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for r in range(2):
        assert open(tmp_path / f"rank{r}").read() == "ok"


def test_sharded_all_gpus(cuda, tmp_path):
    """The same checks with one rank on every visible GPU (4 or 8 on one box)."""
    torch = cuda
    n = torch.cuda.device_count()
    if n <= 2:
        pytest.skip("needs more than two GPUs")
    import torch.multiprocessing as mp
    mp.start_processes(_worker, args=(n, _free_port(), str(tmp_path)), nprocs=n, join=True,
                       start_method="spawn")
    for r in range(n):
        assert open(tmp_path / f"rank{r}").read() == "ok"

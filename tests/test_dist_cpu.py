"""The N-sharded path's host logic with two gloo ranks on the CPU (no GPU).

Each rank takes its shard of the weight rows (ptxstd.dist.shard_range), computes its block of the
decode output with the oracle, all-gathers the rank-major blocks over gloo, and reassembles them
with ptxstd.dist.unshard_columns — the same permutation the device kernel applies after the NCCL
all-gather. Rank 0 checks the result equals the unsharded computation exactly, and the NVFP4 GEMM's
column shards likewise.
"""

import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_path):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "ptx-std_b200"), os.path.join(root, "oracle")]
    import torch
    import torch.distributed as td

    import oracle as O
    from ptxstd import workloads
    from ptxstd.dist import shard_range, unshard_columns

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world)
    M, N, K = 5, 512, 256
    x = workloads.normal_bf16(M, K, seed=11)
    wb = workloads.normal_bf16(N, K, std=0.02, seed=12)
    gw = float(np.abs((wb.astype(np.uint32) << 16).view(np.float32)).max() / (448.0 * 6.0))
    W, sfW = O.quantize_nvfp4(wb, gw)
    lo, hi = shard_range(N, world, rank)
    ns = hi - lo
    # this rank's output block [M, ns] from its weight rows only
    r, c = np.meshgrid(np.arange(M), np.arange(ns), indexing="ij")
    ref, _ = O.gemm_decode_ref(x, W[lo:hi], sfW[lo:hi], gw, r.ravel(), c.ravel())
    mine = torch.from_numpy(ref.astype(np.float32))
    blocks = [torch.empty_like(mine) for _ in range(world)]
    td.all_gather(blocks, mine)
    y = unshard_columns(torch.cat(blocks).numpy(), world, M)

    # NVFP4 GEMM column shards: C[:, lo:hi] from B rows lo:hi
    A, sfA = O.quantize_nvfp4(workloads.normal_bf16(8, K, seed=13), 0.01)
    rc, cc = np.meshgrid(np.arange(8), np.arange(ns), indexing="ij")
    cref, _ = O.gemm_nvfp4_ref(A, sfA, 0.01, W[lo:hi], sfW[lo:hi], gw, rc.ravel(), cc.ravel())
    cm = torch.from_numpy(cref.astype(np.float32))
    cblocks = [torch.empty_like(cm) for _ in range(world)]
    td.all_gather(cblocks, cm)
    cfull = unshard_columns(torch.cat(cblocks).numpy(), world, 8)
    if rank == 0:
        r, c = np.meshgrid(np.arange(M), np.arange(N), indexing="ij")
        want, _ = O.gemm_decode_ref(x, W, sfW, gw, r.ravel(), c.ravel())
        r2, c2 = np.meshgrid(np.arange(8), np.arange(N), indexing="ij")
        cwant, _ = O.gemm_nvfp4_ref(A, sfA, 0.01, W, sfW, gw, r2.ravel(), c2.ravel())
        ok = (np.array_equal(y, want.astype(np.float32).reshape(M, N)) and
              np.array_equal(cfull, cwant.astype(np.float32).reshape(8, N)))
        with open(out_path, "w") as f:
            f.write("ok" if ok else "mismatch")
    td.barrier()
    td.destroy_process_group()


def test_sharded_decode_gather_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    out = str(tmp_path / "result")
    mp.start_processes(_worker, args=(2, _free_port(), out), nprocs=2, join=True,
                       start_method="spawn")
    assert open(out).read() == "ok"


def test_shard_range():
    from ptxstd.dist import shard_range
    assert [shard_range(57344, 8, r) for r in (0, 7)] == [(0, 7168), (50176, 57344)]
    assert shard_range(28672, 4, 2) == (14336, 21504)
    with pytest.raises(ValueError):
        shard_range(100, 8, 0)


def test_unshard_columns_matches_layout():
    from ptxstd.dist import unshard_columns
    world, M, ns = 4, 3, 5
    full = np.arange(M * world * ns).reshape(M, world * ns)
    gathered = np.concatenate([full[:, r * ns:(r + 1) * ns].ravel() for r in range(world)])
    assert np.array_equal(unshard_columns(gathered, world, M), full)

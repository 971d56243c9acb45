"""Multi-GPU layer over the C ABI: N-sharded NVFP4 GEMM and decode GEMM with an NCCL all-gather,
or with the gather fused into the decode GEMM over NVLink peer memory.

One process per GPU. torch.distributed only carries the NCCL unique id from rank 0 to the others
(plumbing); the communicator and the all-gather live in libptxstd (ptxstd_dist_*).

Sharding: a weight of N rows is split into `world` contiguous blocks of N / world rows; rank r owns
rows [r * N / world, (r + 1) * N / world). The decode output is gathered rank-major,
[world][M][N / world], and permuted on the device into row-major [M, N] (`unshard_columns` is the
same permutation in numpy, used by the CPU tests). The peer-to-peer decode
(`Dist.gemm_decode_p2p`) needs no permutation: each rank's epilogue stores its columns straight
into every rank's row-major y.
"""

from __future__ import annotations

import ctypes as C

import numpy as np

from . import _dev, _stream, _torch, check, lib

_SIGS = {
    "ptxstd_dist_unique_id": (C.c_int, [C.c_void_p]),
    "ptxstd_dist_init": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "ptxstd_dist_free": (C.c_int, [C.c_void_p]),
    "ptxstd_dist_size": (C.c_int, [C.c_void_p, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "ptxstd_gemm_nvfp4_sharded": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float,
                                            C.c_void_p, C.c_void_p, C.c_float, C.c_void_p,
                                            C.c_int64, C.c_int64, C.c_int64, C.c_void_p]),
    "ptxstd_gemm_decode_sharded_workspace_bytes": (C.c_size_t, [C.c_void_p, C.c_int64,
                                                                C.c_int64, C.c_int64]),
    "ptxstd_gemm_decode_sharded": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                             C.c_float, C.c_void_p, C.c_int64, C.c_int64,
                                             C.c_int64, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_dist_decode_p2p_init": (C.c_int, [C.c_void_p, C.c_int64, C.POINTER(C.c_void_p)]),
    "ptxstd_gemm_decode_sharded_p2p": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                                 C.c_float, C.c_void_p, C.c_int64, C.c_int64,
                                                 C.c_int64, C.c_void_p, C.c_size_t, C.c_void_p]),
}

P2P_ROWS = 16  # rows of the library-owned peer-to-peer decode output


class _DeviceRows:
    """__cuda_array_interface__ of library-owned bf16 [rows, n] memory, viewed by torch."""

    def __init__(self, ptr: int, rows: int, n: int):
        self.__cuda_array_interface__ = {"shape": (rows, n), "typestr": "<i2",
                                         "data": (ptr, False), "version": 3, "strides": None}


def _lib():
    L = lib()
    for name, (res, args) in _SIGS.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of an N-row weight owned by `rank` (N must divide evenly)."""
    if n % world:
        raise ValueError(f"N = {n} does not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def unshard_columns(gathered: np.ndarray, world: int, m: int) -> np.ndarray:
    """[world * M * ns] rank-major blocks -> row-major [M, world * ns]."""
    g = np.asarray(gathered).reshape(world, m, -1)
    return np.ascontiguousarray(g.transpose(1, 0, 2).reshape(m, -1))


class Dist:
    """An NCCL communicator for this rank on the current CUDA device."""

    def __init__(self, world: int, rank: int, unique_id: bytes):
        if len(unique_id) != 128:
            raise ValueError("NCCL unique id is 128 bytes")
        self.world, self.rank = world, rank
        buf = (C.c_uint8 * 128).from_buffer_copy(unique_id)
        h = C.c_void_p()
        check(_lib().ptxstd_dist_init(buf, world, rank, C.byref(h)), "dist_init")
        self.handle = h
        self._ws = {}
        self._p2p = None  # (n_total, bf16 [16, n_total] view of the library-owned y)

    @staticmethod
    def new_unique_id() -> bytes:
        buf = (C.c_uint8 * 128)()
        check(_lib().ptxstd_dist_unique_id(buf), "dist_unique_id")
        return bytes(buf)

    @classmethod
    def from_torch(cls):
        """Creates the communicator of every rank of the default torch.distributed group."""
        import torch.distributed as td
        world, rank = td.get_world_size(), td.get_rank()
        obj = [cls.new_unique_id() if rank == 0 else None]
        td.broadcast_object_list(obj, src=0)
        return cls(world, rank, obj[0])

    def close(self):
        self._p2p = None
        if self.handle:
            check(_lib().ptxstd_dist_free(self.handle), "dist_free")
            self.handle = None

    def gemm_nvfp4(self, a, sfa, ga, b_shard, sfb_shard, gb, n_total, out=None, stream=None):
        torch = _torch()
        M, Kh = a.shape
        ns = n_total // self.world
        c = out if out is not None else torch.empty((M, ns), dtype=torch.bfloat16,
                                                    device=a.device)
        check(_lib().ptxstd_gemm_nvfp4_sharded(self.handle, _dev(a), _dev(sfa), float(ga),
                                               _dev(b_shard), _dev(sfb_shard), float(gb),
                                               _dev(c), M, n_total, 2 * Kh, _stream(stream)),
              "gemm_nvfp4_sharded")
        return c

    def gemm_decode(self, x, w_shard, sfw_shard, gw, n_total, out=None, stream=None):
        """y [M, n_total] (every rank) = MXFP8(x) * NVFP4(W)^T * gw, W split along N."""
        torch = _torch()
        M, K = x.shape
        nbytes = int(_lib().ptxstd_gemm_decode_sharded_workspace_bytes(self.handle, M, n_total,
                                                                        K))
        if nbytes == 0:
            raise ValueError("bad decode shape for this communicator")
        ptr = self._workspace(nbytes, x.device)
        y = out if out is not None else torch.empty((M, n_total), dtype=torch.bfloat16,
                                                    device=x.device)
        check(_lib().ptxstd_gemm_decode_sharded(self.handle, _dev(x), _dev(w_shard),
                                                _dev(sfw_shard), float(gw), _dev(y), M, n_total,
                                                K, ptr, nbytes, _stream(stream)),
              "gemm_decode_sharded")
        return y

    def _workspace(self, nbytes, device):
        torch = _torch()
        ws = self._ws.get(nbytes)
        if ws is None:
            ws = torch.empty(nbytes + 1024, dtype=torch.uint8, device=device)
            self._ws[nbytes] = ws
        return ws.data_ptr() + (-ws.data_ptr()) % 1024

    def decode_p2p_output(self, n_total):
        """The library-owned y [16, n_total] bf16 of the peer-to-peer decode (set up on first use,
        collectively: every rank calls it with the same n_total)."""
        torch = _torch()
        if self._p2p is None:
            ptr = C.c_void_p()
            check(_lib().ptxstd_dist_decode_p2p_init(self.handle, n_total, C.byref(ptr)),
                  "dist_decode_p2p_init")
            y = torch.as_tensor(_DeviceRows(ptr.value, P2P_ROWS, n_total),
                                device=torch.device("cuda", torch.cuda.current_device()))
            self._p2p = (n_total, y.view(torch.bfloat16))
        elif self._p2p[0] != n_total:
            raise ValueError("the peer-to-peer decode output is set up for another N")
        return self._p2p[1]

    def gemm_decode_p2p(self, x, w_shard, sfw_shard, gw, n_total, out=None, stream=None):
        """y [M, n_total] (every rank) = MXFP8(x) * NVFP4(W)^T * gw, W split along N, the gather
        fused into the GEMM. Returns rows [:M] of the library-owned output (valid until the next
        call), or `out` filled with a copy of them."""
        M, K = x.shape
        y = self.decode_p2p_output(n_total)
        ns = n_total // self.world
        nbytes = int(lib().ptxstd_gemm_decode_workspace_bytes(M, ns, K))
        if nbytes == 0:
            raise ValueError("bad decode shape for this communicator")
        ptr = self._workspace(nbytes, x.device)
        check(_lib().ptxstd_gemm_decode_sharded_p2p(self.handle, _dev(x), _dev(w_shard),
                                                    _dev(sfw_shard), float(gw),
                                                    _dev(out) if out is not None else None, M,
                                                    n_total, K, ptr, nbytes, _stream(stream)),
              "gemm_decode_sharded_p2p")
        return out if out is not None else y[:M]

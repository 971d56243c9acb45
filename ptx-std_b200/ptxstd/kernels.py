"""Quantise and GEMM kernels of libptxstd over CUDA tensors (torch supplies memory/streams)."""

from __future__ import annotations

from . import _dev, _stream, _torch, check, lib

SF_ROWMAJOR, SF_BLOCKED = 0, 1


def quantize_mxfp8(x, sf_layout: int = SF_ROWMAJOR, out=None, stream=None, seed=None):
    """bf16 [rows, cols] -> (E4M3 [rows, cols] uint8, UE8M0 scales uint8).

    Scales are [rows, cols/32] row-major (sf_layout 0) or the blocked 128x4 GEMM layout (1).
    With a `seed`, the elements are rounded stochastically (ptxstd_quantize_mxfp8_rs: random bits
    from SplitMix64 started at the seed, group of four elements i // 4).
    """
    torch = _torch()
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("expected a 2-D bfloat16 tensor")
    rows, cols = x.shape
    if out is None:
        q = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
        sf = torch.empty((rows, cols // 32), dtype=torch.uint8, device=x.device)
    else:
        q, sf = out
    if seed is None:
        check(lib().ptxstd_quantize_mxfp8_layout(_dev(x), rows, cols, _dev(q), _dev(sf),
                                                 sf_layout, _stream(stream)), "quantize_mxfp8")
    else:
        check(lib().ptxstd_quantize_mxfp8_rs(_dev(x), rows, cols, _dev(q), _dev(sf), sf_layout,
                                             int(seed) & (2**64 - 1), _stream(stream)),
              "quantize_mxfp8(seed)")
    return q, sf


def gemm_fp8(a, b, sa: float = 1.0, sb: float = 1.0, out=None, stream=None):
    """E4M3 codes a [M, K], b [N, K] (uint8, K contiguous) -> bf16 C [M, N] = sa*sb * a @ b^T."""
    torch = _torch()
    if a.dtype != torch.uint8 or b.dtype != torch.uint8 or a.dim() != 2 or b.dim() != 2:
        raise TypeError("expected 2-D uint8 E4M3 code tensors")
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError("K mismatch")
    c = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    check(lib().ptxstd_gemm_fp8(_dev(a), _dev(b), float(sa), float(sb), _dev(c), M, N, K,
                                _stream(stream)), "gemm_fp8")
    return c


def gemm_mxfp8(a, sfa, b, sfb, out=None, stream=None):
    """MXFP8 a [M, K], b [N, K] (uint8, E4M3) with blocked UE8M0 scales per 32 -> bf16 [M, N]."""
    torch = _torch()
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError("K mismatch")
    if sfa.numel() != M * K // 32 or sfb.numel() != N * K // 32:
        raise ValueError("scale tensors must hold one UE8M0 per 32 elements")
    c = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    check(lib().ptxstd_gemm_mxfp8(_dev(a), _dev(sfa), _dev(b), _dev(sfb), _dev(c), M, N, K,
                                  _stream(stream)), "gemm_mxfp8")
    return c


# MX element types (the tcgen05 F8f6f4ElementType codes)
MX_E4M3, MX_E5M2, MX_E2M3, MX_E3M2, MX_E2M1 = 0, 1, 3, 4, 5
MX_TYPES = {"e4m3": MX_E4M3, "e5m2": MX_E5M2, "e2m3": MX_E2M3, "e3m2": MX_E3M2, "e2m1": MX_E2M1}


def _mx_type(t) -> int:
    """An MX element type by name or tcgen05 code; ValueError for anything else."""
    code = MX_TYPES.get(t) if isinstance(t, str) else int(t)
    if code not in MX_TYPES.values():
        raise ValueError(f"unknown MX element type {t!r} (one of {sorted(MX_TYPES)})")
    return code


def quantize_mx(x, elem_type, sf_layout: int = 1, out=None, stream=None):
    """bf16 [rows, cols] -> (payload [rows, cols] uint8 in the tensor-core operand layout,
    UE8M0 scales per 32) for any MX element type ("e4m3", "e5m2", "e2m3", "e3m2", "e2m1" or the
    MX_* code). FP6 / FP4 payloads are 16-element groups padded to 16 bytes."""
    torch = _torch()
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("expected a 2-D bfloat16 tensor")
    t = _mx_type(elem_type)
    rows, cols = x.shape
    if out is None:
        q = torch.empty((rows, cols), dtype=torch.uint8, device=x.device)
        sf = torch.empty((rows, cols // 32), dtype=torch.uint8, device=x.device)
    else:
        q, sf = out
    check(lib().ptxstd_quantize_mx(_dev(x), rows, cols, t, _dev(q), _dev(sf), sf_layout,
                                   _stream(stream)), "quantize_mx")
    return q, sf


def gemm_mx(a, a_type, sfa, b, b_type, sfb, out=None, stream=None):
    """MX GEMM with any pair of element types: a [M, K], b [N, K] payloads in the operand layout
    of quantize_mx, blocked UE8M0 scales per 32 -> bf16 [M, N]."""
    torch = _torch()
    ta, tb = _mx_type(a_type), _mx_type(b_type)
    M, K = a.shape
    N = b.shape[0]
    if b.shape[1] != K:
        raise ValueError("K mismatch")
    if sfa.numel() != M * K // 32 or sfb.numel() != N * K // 32:
        raise ValueError("scale tensors must hold one UE8M0 per 32 elements")
    c = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    check(lib().ptxstd_gemm_mx(_dev(a), ta, _dev(sfa), _dev(b), tb, _dev(sfb), _dev(c), M, N, K,
                               _stream(stream)), "gemm_mx")
    return c


def tcgen05_cp_unpack(packed, elem_type, stream=None):
    """Packed FP6 / FP4 rows [n * 128, 32] (uint8, the quantize_mx layout) through the
    decompressing tcgen05.cp into TMEM and back: one 8-bit container per element, same shape."""
    torch = _torch()
    t = _mx_type(elem_type)
    if t not in (MX_E2M3, MX_E3M2, MX_E2M1):
        raise ValueError("the decompressing copy takes FP6 (e2m3, e3m2) or FP4 (e2m1) payloads")
    if packed.dtype != torch.uint8 or packed.dim() != 2 or packed.shape[1] != 32 or \
            packed.shape[0] % 128:
        raise ValueError("expected uint8 [n * 128, 32]")
    out = torch.empty_like(packed)
    check(lib().ptxstd_tcgen05_cp_unpack(_dev(packed), _dev(out), packed.shape[0] // 128, t,
                                         _stream(stream)), "tcgen05_cp_unpack")
    return out


def prune_24(codes, stream=None):
    """2:4 pruning of E4M3 codes [rows, cols] (uint8) -> (vals [rows, cols/2], meta [rows, cols/8])
    (ptxstd_prune_24_e4m3: the two largest magnitudes of each group of four are kept)."""
    torch = _torch()
    if codes.dtype != torch.uint8 or codes.dim() != 2:
        raise TypeError("expected 2-D uint8 E4M3 codes")
    rows, cols = codes.shape
    codes = codes.contiguous()
    vals = torch.empty((rows, cols // 2), dtype=torch.uint8, device=codes.device)
    meta = torch.empty((rows, cols // 8), dtype=torch.uint8, device=codes.device)
    check(lib().ptxstd_prune_24_e4m3(_dev(codes), rows, cols, _dev(vals), _dev(meta),
                                     _stream(stream)), "prune_24")
    return vals, meta


def gemm_mxfp8_sparse(vals, meta, sfa, b, sfb, out=None, stream=None):
    """2:4-sparse MXFP8: A as (vals [M, K/2], meta [M, K/8]) from prune_24, b [N, K] E4M3, blocked
    UE8M0 scales per 64 logical K for both operands -> bf16 [M, N]."""
    torch = _torch()
    M, Kh = vals.shape
    K = 2 * Kh
    N = b.shape[0]
    if b.shape[1] != K or meta.shape != (M, K // 8):
        raise ValueError("shape mismatch")
    if sfa.numel() != M * K // 64 or sfb.numel() != N * K // 64:
        raise ValueError("scale tensors must hold one UE8M0 per 64 logical elements")
    c = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=vals.device)
    check(lib().ptxstd_gemm_mxfp8_sparse(_dev(vals), _dev(meta), _dev(sfa), _dev(b), _dev(sfb),
                                         _dev(c), M, N, K, _stream(stream)), "gemm_mxfp8_sparse")
    return c


SCHEDULE_PERSISTENT, SCHEDULE_DYNAMIC = 0, 1


def set_gemm_schedule(schedule: int) -> None:
    """Tile schedule of the CTA-pair NVFP4 GEMM for later calls, process-wide:
    SCHEDULE_PERSISTENT (default, a fixed raster over resident pairs) or SCHEDULE_DYNAMIC
    (one cluster per tile; running pairs take over tiles of clusters not yet started)."""
    check(lib().ptxstd_set_gemm_schedule(int(schedule)), "set_gemm_schedule")


def get_gemm_schedule() -> int:
    return int(lib().ptxstd_get_gemm_schedule())


def gemm_nvfp4(a, sfa, ga: float, b, sfb, gb: float, out=None, stream=None):
    """NVFP4 a [M, K/2], b [N, K/2] (uint8, E2M1x2) with blocked E4M3 scales -> bf16 [M, N]."""
    torch = _torch()
    M, Kh = a.shape
    N = b.shape[0]
    if b.shape[1] != Kh:
        raise ValueError("K mismatch")
    K = 2 * Kh
    if sfa.numel() != M * K // 16 or sfb.numel() != N * K // 16:
        raise ValueError("scale tensors must hold one E4M3 per 16 elements")
    c = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=a.device)
    check(lib().ptxstd_gemm_nvfp4(_dev(a), _dev(sfa), float(ga), _dev(b), _dev(sfb), float(gb),
                                  _dev(c), M, N, K, _stream(stream)), "gemm_nvfp4")
    return c


_workspaces: dict = {}


def decode_workspace(M: int, N: int, K: int, device=None):
    """A cached device workspace for gemm_decode (one per device and size)."""
    torch = _torch()
    dev = torch.device(device) if device is not None else torch.device(
        "cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    nbytes = int(lib().ptxstd_gemm_decode_workspace_bytes(M, N, K))
    key = (dev.index, nbytes)
    ws = _workspaces.get(key)
    if ws is None:
        ws = torch.empty(nbytes + 1024, dtype=torch.uint8, device=dev)
        _workspaces[key] = ws
    off = (-ws.data_ptr()) % 1024
    return ws, ws.data_ptr() + off, nbytes


def gemm_decode(x, w, sfw, gw: float, out=None, workspace=None, stream=None):
    """bf16 x [M <= 16, K] (quantised to MXFP8 in the call) times NVFP4 w [N, K/2] with blocked
    E4M3 scales and global scale gw -> bf16 [M, N]."""
    torch = _torch()
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("expected a 2-D bfloat16 activation tensor")
    M, K = x.shape
    N = w.shape[0]
    if w.shape[1] * 2 != K or sfw.numel() != N * K // 16:
        raise ValueError("shape mismatch")
    y = out if out is not None else torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        _, ptr, nbytes = decode_workspace(M, N, K, x.device)
    else:
        ptr, nbytes = workspace
    check(lib().ptxstd_gemm_decode(_dev(x), _dev(w), _dev(sfw), float(gw), _dev(y), M, N, K,
                                   ptr, nbytes, _stream(stream)), "gemm_decode")
    return y


def quantize_nvfp4(x, global_scale: float, sf_layout: int = SF_ROWMAJOR, out=None,
                   stream=None, seed=None):
    """bf16 [rows, cols] -> (E2M1x2 [rows, cols/2] uint8, E4M3 scales per 16 uint8).

    With a `seed`, the elements are rounded stochastically (ptxstd_quantize_nvfp4_rs)."""
    torch = _torch()
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("expected a 2-D bfloat16 tensor")
    rows, cols = x.shape
    if out is None:
        q = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
        sf = torch.empty((rows, cols // 16), dtype=torch.uint8, device=x.device)
    else:
        q, sf = out
    if seed is None:
        check(lib().ptxstd_quantize_nvfp4_layout(_dev(x), rows, cols, float(global_scale),
                                                 _dev(q), _dev(sf), sf_layout, _stream(stream)),
              "quantize_nvfp4")
    else:
        check(lib().ptxstd_quantize_nvfp4_rs(_dev(x), rows, cols, float(global_scale), _dev(q),
                                             _dev(sf), sf_layout, int(seed) & (2**64 - 1),
                                             _stream(stream)), "quantize_nvfp4(seed)")
    return q, sf

"""Quantise and GEMM kernels of libptxstd over CUDA tensors (torch supplies memory/streams)."""

from __future__ import annotations

from . import _dev, _stream, _torch, check, lib

SF_ROWMAJOR, SF_BLOCKED = 0, 1


def quantize_mxfp8(x, sf_layout: int = SF_ROWMAJOR, out=None, stream=None):
    """bf16 [rows, cols] -> (E4M3 [rows, cols] uint8, UE8M0 scales uint8).

    Scales are [rows, cols/32] row-major (sf_layout 0) or the blocked 128x4 GEMM layout (1).
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
    check(lib().ptxstd_quantize_mxfp8_layout(_dev(x), rows, cols, _dev(q), _dev(sf), sf_layout,
                                             _stream(stream)), "quantize_mxfp8")
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


def quantize_nvfp4(x, global_scale: float, sf_layout: int = SF_ROWMAJOR, out=None,
                   stream=None):
    """bf16 [rows, cols] -> (E2M1x2 [rows, cols/2] uint8, E4M3 scales per 16 uint8)."""
    torch = _torch()
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise TypeError("expected a 2-D bfloat16 tensor")
    rows, cols = x.shape
    if out is None:
        q = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
        sf = torch.empty((rows, cols // 16), dtype=torch.uint8, device=x.device)
    else:
        q, sf = out
    check(lib().ptxstd_quantize_nvfp4_layout(_dev(x), rows, cols, float(global_scale), _dev(q),
                                             _dev(sf), sf_layout, _stream(stream)),
          "quantize_nvfp4")
    return q, sf

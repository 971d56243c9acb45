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

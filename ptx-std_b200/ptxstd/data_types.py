"""Narrow-float conversions over CUDA tensors (ptx-std src/data_types/).

Each function mirrors a reference conversion applied element-wise, computed by libptxstd's
kernels with the same `cvt` instructions the reference's pair methods wrap:

- ``from_f32(fmt, x, relu)``: Vector<fmt, N>::from_f32::<RELU> (src/data_types/narrow.rs:354-361),
  RN .satfinite; one code per byte for FP8 and FP6 (src/data_types/float6.rs: the value in the
  low 6 bits), two per byte (element 0 low nibble) for E2M1.
- ``to_f32(fmt, codes)``: exact decode through f16 (narrow.rs:292-299).
- ``ue8m0_from_f32(x, round_up, satfinite)``: f8e8m0::from_f32::<RND, OVERFLOW>
  (narrow.rs:600-617); ``ue8m0_to_f32``: through bf16 (narrow.rs:683-690).
- ``from_f32_stochastic(fmt, x, rbits, relu)``: Vector<fmt, N>::from_f32_stochastic::<RELU>
  (narrow.rs:494-505), one rbits word per group of four elements; ``bf16_from_f32_stochastic``
  and ``f16_from_f32_stochastic``: bf16xN / f16xN::from_f32_stochastic::<R, O>
  (bfloat16.rs:572-598, float16.rs:740-766), one word per pair.
"""

from __future__ import annotations

from . import _dev, _stream, _torch, check, lib

E4M3, E5M2, E2M1, E2M3, E3M2 = "e4m3", "e5m2", "e2m1", "e2m3", "e3m2"

_ENC = {E4M3: "ptxstd_cvt_f32_to_e4m3", E5M2: "ptxstd_cvt_f32_to_e5m2",
        E2M1: "ptxstd_cvt_f32_to_e2m1x2", E2M3: "ptxstd_cvt_f32_to_e2m3",
        E3M2: "ptxstd_cvt_f32_to_e3m2"}
_DEC = {E4M3: "ptxstd_cvt_e4m3_to_f32", E5M2: "ptxstd_cvt_e5m2_to_f32",
        E2M1: "ptxstd_cvt_e2m1x2_to_f32", E2M3: "ptxstd_cvt_e2m3_to_f32",
        E3M2: "ptxstd_cvt_e3m2_to_f32"}


def from_f32(fmt: str, x, relu: bool = False, stream=None):
    torch = _torch()
    if x.dtype != torch.float32:
        raise TypeError("expected float32")
    x = x.contiguous()
    n = x.numel()
    out = torch.empty(n // 2 if fmt == E2M1 else n, dtype=torch.uint8, device=x.device)
    check(getattr(lib(), _ENC[fmt])(_dev(x), _dev(out), n, int(relu), _stream(stream)),
          f"from_f32({fmt})")
    return out


_F16 = {E4M3: "e4m3", E5M2: "e5m2", E2M1: "e2m1x2", E2M3: "e2m3", E3M2: "e3m2"}


def from_f16(fmt: str, x, relu: bool = False, stream=None):
    """Vector<fmt, N>::from_f16 (narrow.rs:164-172): float16 tensor -> codes (RN .satfinite)."""
    torch = _torch()
    if x.dtype != torch.float16:
        raise TypeError("expected float16")
    x = x.contiguous()
    n = x.numel()
    out = torch.empty(n // 2 if fmt == E2M1 else n, dtype=torch.uint8, device=x.device)
    check(getattr(lib(), f"ptxstd_cvt_f16_to_{_F16[fmt]}")(_dev(x), _dev(out), n, int(relu),
                                                            _stream(stream)), f"from_f16({fmt})")
    return out


def to_f16(fmt: str, codes, stream=None):
    """Vector<fmt, N>::to_f16 (narrow.rs:275-291): exact float16 values of the codes."""
    torch = _torch()
    codes = codes.contiguous()
    n = codes.numel()
    out = torch.empty(2 * n if fmt == E2M1 else n, dtype=torch.float16, device=codes.device)
    check(getattr(lib(), f"ptxstd_cvt_{_F16[fmt]}_to_f16")(_dev(codes), _dev(out), n,
                                                            _stream(stream)), f"to_f16({fmt})")
    return out


def bf16_from_f32(x, relu: bool = False, satfinite: bool = False, stream=None):
    """bf16xN::from_f32::<R, O> (bfloat16.rs:104-118): bf16 bit patterns (int16), RN."""
    torch = _torch()
    if x.dtype != torch.float32:
        raise TypeError("expected float32")
    x = x.contiguous()
    out = torch.empty(x.numel(), dtype=torch.int16, device=x.device)
    check(lib().ptxstd_cvt_f32_to_bf16(_dev(x), _dev(out), x.numel(), int(relu), int(satfinite),
                                       _stream(stream)), "bf16_from_f32")
    return out


def from_bf16(fmt: str, x, relu: bool = False, stream=None):
    """Vector<fmt, N>::from_bf16 (narrow.rs:363-395): bf16 widens to f32 exactly, so the RN
    conversion of the widened value is the same rounding of the same real number."""
    torch = _torch()
    return from_f32(fmt, x.to(torch.float32), relu, stream)


def to_f32(fmt: str, codes, stream=None):
    torch = _torch()
    codes = codes.contiguous()
    n = codes.numel()
    out = torch.empty(2 * n if fmt == E2M1 else n, dtype=torch.float32, device=codes.device)
    check(getattr(lib(), _DEC[fmt])(_dev(codes), _dev(out), n, _stream(stream)),
          f"to_f32({fmt})")
    return out


_ENC_RS = {E4M3: "ptxstd_cvt_f32_to_e4m3_rs", E5M2: "ptxstd_cvt_f32_to_e5m2_rs",
           E2M1: "ptxstd_cvt_f32_to_e2m1x2_rs", E2M3: "ptxstd_cvt_f32_to_e2m3_rs",
           E3M2: "ptxstd_cvt_f32_to_e3m2_rs"}


def _rbits(rbits, need: int):
    torch = _torch()
    if rbits.dtype not in (torch.int32, torch.uint32) or rbits.numel() < need:
        raise ValueError(f"rbits must be 32-bit words, at least {need} of them")
    return rbits.contiguous()


def from_f32_stochastic(fmt: str, x, rbits, relu: bool = False, stream=None):
    """Stochastic rounding: elements 4g .. 4g+3 of x with rbits[g] (32-bit words)."""
    torch = _torch()
    if x.dtype != torch.float32:
        raise TypeError("expected float32")
    x = x.contiguous()
    n = x.numel()
    rb = _rbits(rbits, (n + 3) // 4)
    out = torch.empty(n // 2 if fmt == E2M1 else n, dtype=torch.uint8, device=x.device)
    check(getattr(lib(), _ENC_RS[fmt])(_dev(x), _dev(rb), _dev(out), n, int(relu),
                                       _stream(stream)), f"from_f32_stochastic({fmt})")
    return out


def _x2_stochastic(name, x, rbits, relu, satfinite, stream):
    torch = _torch()
    if x.dtype != torch.float32:
        raise TypeError("expected float32")
    x = x.contiguous()
    n = x.numel()
    rb = _rbits(rbits, (n + 1) // 2)
    out = torch.empty(n, dtype=torch.int16, device=x.device)
    check(getattr(lib(), name)(_dev(x), _dev(rb), _dev(out), n, int(relu), int(satfinite),
                               _stream(stream)), name)
    return out


def bf16_from_f32_stochastic(x, rbits, relu: bool = False, satfinite: bool = False,
                             stream=None):
    """bf16 bit patterns (int16) of x rounded stochastically, elements 2p, 2p+1 with rbits[p]."""
    return _x2_stochastic("ptxstd_cvt_f32_to_bf16_rs", x, rbits, relu, satfinite, stream)


def f16_from_f32_stochastic(x, rbits, relu: bool = False, satfinite: bool = False, stream=None):
    """f16 bit patterns (int16) of x rounded stochastically, elements 2p, 2p+1 with rbits[p]."""
    return _x2_stochastic("ptxstd_cvt_f32_to_f16_rs", x, rbits, relu, satfinite, stream)


_SCALED = {E4M3: "ptxstd_cvt_e4m3_to_bf16_scaled", E5M2: "ptxstd_cvt_e5m2_to_bf16_scaled",
           E2M1: "ptxstd_cvt_e2m1x2_to_bf16_scaled", E2M3: "ptxstd_cvt_e2m3_to_bf16_scaled",
           E3M2: "ptxstd_cvt_e3m2_to_bf16_scaled"}


def to_bf16_scaled(fmt: str, codes, scales, block: int = 1, relu: bool = False,
                   satfinite: bool = False, stream=None):
    """Vector<fmt, N>::to_bf16_scaled (narrow.rs:444-465): bf16 bit patterns (int16) of each code
    times its UE8M0 scale scales[i // block]. E2M1 codes are packed two per byte."""
    torch = _torch()
    codes = codes.contiguous()
    scales = scales.contiguous()
    n = 2 * codes.numel() if fmt == E2M1 else codes.numel()
    if scales.numel() < (n + block - 1) // block:
        raise ValueError("too few scales")
    out = torch.empty(n, dtype=torch.int16, device=codes.device)
    check(getattr(lib(), _SCALED[fmt])(_dev(codes), _dev(scales), _dev(out), n, block, int(relu),
                                       int(satfinite), _stream(stream)), f"to_bf16_scaled({fmt})")
    return out


def ue8m0_from_f32(x, round_up: bool = False, satfinite: bool = True, stream=None):
    torch = _torch()
    x = x.contiguous()
    out = torch.empty(x.numel(), dtype=torch.uint8, device=x.device)
    check(lib().ptxstd_cvt_f32_to_ue8m0(_dev(x), _dev(out), x.numel(), int(round_up),
                                        int(satfinite), _stream(stream)), "ue8m0_from_f32")
    return out


def ue8m0_to_f32(codes, stream=None):
    torch = _torch()
    codes = codes.contiguous()
    out = torch.empty(codes.numel(), dtype=torch.float32, device=codes.device)
    check(lib().ptxstd_cvt_ue8m0_to_f32(_dev(codes), _dev(out), codes.numel(), _stream(stream)),
          "ue8m0_to_f32")
    return out


def sweep_width(variant: int) -> int:
    """Bytes per input of a sweep variant: 2 for the bf16/f16 forms (22..33)."""
    return 2 if variant >= 22 else 1


def sweep(variant: int, base: int, n: int, out=None, stream=None):
    """Codes of the f32 bit patterns base .. base+n-1 (see ptxstd_cvt_sweep)."""
    torch = _torch()
    if out is None:
        out = torch.empty(n * sweep_width(variant), dtype=torch.uint8, device="cuda")
    elif out.numel() < n * sweep_width(variant):
        raise ValueError("sweep output too small")
    check(lib().ptxstd_cvt_sweep(variant, base, n, _dev(out), _stream(stream)), "sweep")
    return out

"""Python host side of libptxstd: ctypes bindings of include/ptxstd.h plus torch conveniences.

Module layout mirrors caelunshun/ptx-std's modules: ``ptxstd.data_types`` (narrow-float
conversions, src/data_types/), ``ptxstd.tcgen05`` (descriptor builders, src/tcgen05/descriptor.rs),
and the kernels built on them (quantise, GEMM). torch supplies device memory and streams only;
every computation runs in libptxstd.so's CUDA kernels. There is no fallback: if the library or a
CUDA device is missing, calls raise.
"""

from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG, "libptxstd.so")

OK, EINVAL, ECUDA, ENCCL, ETIMEOUT, EUNSUPPORTED = range(6)


class PtxStdError(RuntimeError):
    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {status_string(status)} ({status})")


_lib: C.CDLL | None = None

_u8p = C.c_void_p
_SIGS = {
    "ptxstd_status_string": (C.c_char_p, [C.c_int]),
    "ptxstd_version": (C.c_int, []),
    "ptxstd_device_supported": (C.c_int, [C.c_int]),
    "ptxstd_last_device_error": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_int),
                                           C.POINTER(C.c_uint32)]),
    "ptxstd_cvt_f32_to_e4m3": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                         C.c_void_p]),
    "ptxstd_cvt_f32_to_e5m2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                         C.c_void_p]),
    "ptxstd_cvt_f32_to_e2m1x2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                           C.c_void_p]),
    "ptxstd_cvt_f32_to_ue8m0": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_int,
                                          C.c_void_p]),
    "ptxstd_cvt_e4m3_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_e5m2_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_e2m1x2_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_ue8m0_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_f32_to_e2m3": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                         C.c_void_p]),
    "ptxstd_cvt_f32_to_e3m2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                         C.c_void_p]),
    "ptxstd_cvt_e2m3_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_e3m2_to_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_sweep": (C.c_int, [C.c_int, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p]),
    "ptxstd_cvt_e4m3_to_bf16_scaled": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                 C.c_size_t, C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_cvt_e5m2_to_bf16_scaled": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                 C.c_size_t, C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_cvt_e2m1x2_to_bf16_scaled": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                 C.c_size_t, C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_cvt_e2m3_to_bf16_scaled": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                 C.c_size_t, C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_cvt_e3m2_to_bf16_scaled": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                                 C.c_size_t, C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_cvt_f16_to_e4m3": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                          C.c_void_p]),
    "ptxstd_cvt_e4m3_to_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_f16_to_e5m2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                          C.c_void_p]),
    "ptxstd_cvt_e5m2_to_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_f16_to_e2m1x2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                          C.c_void_p]),
    "ptxstd_cvt_e2m1x2_to_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_f16_to_e2m3": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                          C.c_void_p]),
    "ptxstd_cvt_e2m3_to_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_f16_to_e3m2": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int,
                                          C.c_void_p]),
    "ptxstd_cvt_e3m2_to_f16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ptxstd_cvt_f32_to_bf16": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_int,
                                         C.c_void_p]),
    "ptxstd_cvt_f32_to_e4m3_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.c_int, C.c_void_p]),
    "ptxstd_cvt_f32_to_e5m2_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.c_int, C.c_void_p]),
    "ptxstd_cvt_f32_to_e2m3_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.c_int, C.c_void_p]),
    "ptxstd_cvt_f32_to_e3m2_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.c_int, C.c_void_p]),
    "ptxstd_cvt_f32_to_e2m1x2_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                              C.c_int, C.c_void_p]),
    "ptxstd_cvt_f32_to_bf16_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                            C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_cvt_f32_to_f16_rs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t,
                                           C.c_int, C.c_int, C.c_void_p]),
    "ptxstd_quantize_mxfp8": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                        C.c_void_p, C.c_void_p]),
    "ptxstd_quantize_nvfp4": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_float, C.c_void_p,
                                        C.c_void_p, C.c_void_p]),
    "ptxstd_quantize_mxfp8_layout": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                               C.c_void_p, C.c_int, C.c_void_p]),
    "ptxstd_quantize_nvfp4_layout": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_float,
                                               C.c_void_p, C.c_void_p, C.c_int, C.c_void_p]),
    "ptxstd_quantize_mxfp8_rs": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                           C.c_void_p, C.c_int, C.c_uint64, C.c_void_p]),
    "ptxstd_quantize_nvfp4_rs": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_float,
                                           C.c_void_p, C.c_void_p, C.c_int, C.c_uint64,
                                           C.c_void_p]),
    "ptxstd_gemm_fp8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_float, C.c_float, C.c_void_p,
                                  C.c_int64, C.c_int64, C.c_int64, C.c_void_p]),
    "ptxstd_set_gemm_schedule": (C.c_int, [C.c_int]),
    "ptxstd_get_gemm_schedule": (C.c_int, []),
    "ptxstd_gemm_nvfp4": (C.c_int, [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p,
                                    C.c_float, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                    C.c_void_p]),
    "ptxstd_quantize_mx": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p,
                                     C.c_void_p, C.c_int, C.c_void_p]),
    "ptxstd_tcgen05_cp_unpack": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.c_int,
                                           C.c_void_p]),
    "ptxstd_gemm_mx": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                 C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int64,
                                 C.c_void_p]),
    "ptxstd_gemm_mxfp8": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_int64, C.c_int64, C.c_int64, C.c_void_p]),
    "ptxstd_prune_24_e4m3": (C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                                       C.c_void_p]),
    "ptxstd_gemm_mxfp8_sparse": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                           C.c_int64, C.c_void_p]),
    "ptxstd_gemm_decode_workspace_bytes": (C.c_size_t, [C.c_int64, C.c_int64, C.c_int64]),
    "ptxstd_gemm_decode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p,
                                     C.c_int64, C.c_int64, C.c_int64, C.c_void_p, C.c_size_t,
                                     C.c_void_p]),
    "ptxstd_idesc_f16": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_uint32, C.c_uint32,
                                   C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_tf32": (C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_f8f6f4": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_uint32, C.c_uint32,
                                      C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_i8": (C.c_int, [C.c_int, C.c_int, C.c_uint32, C.c_uint32,
                                  C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_mxf8f6f4": (C.c_int, [C.c_int, C.c_int, C.c_uint32, C.c_uint32,
                                        C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_mxf4": (C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_mxf4nvf4": (C.c_int, [C.c_int, C.c_uint32, C.c_uint32,
                                        C.POINTER(C.c_uint32)]),
    "ptxstd_idesc_set": (C.c_int, [C.c_uint32, C.c_int, C.c_int, C.c_uint32,
                                   C.POINTER(C.c_uint32)]),
    "ptxstd_smem_desc": (C.c_int, [C.c_uint32, C.c_uint32, C.c_uint32, C.c_int,
                                   C.POINTER(C.c_uint64)]),
    "ptxstd_smem_desc_with_base_offset": (C.c_int, [C.c_uint64, C.c_uint32,
                                                    C.POINTER(C.c_uint64)]),
    "ptxstd_smem_desc_add_start_bytes": (C.c_int, [C.c_uint64, C.c_uint32,
                                                   C.POINTER(C.c_uint64)]),
    "ptxstd_zero_mask_new": (C.c_int, [C.c_uint32, C.c_uint32, C.POINTER(C.c_uint64)]),
    "ptxstd_zero_mask_with_sub_mask_start": (C.c_int, [C.c_uint64, C.c_uint32, C.c_int,
                                                       C.c_uint32, C.POINTER(C.c_uint64)]),
    "ptxstd_zero_mask_with_column_shift": (C.c_int, [C.c_uint64, C.c_uint32,
                                                     C.POINTER(C.c_uint64)]),
}


def lib() -> C.CDLL:
    """Loads ptx-std_b200/libptxstd.so (built by ptx-std_b200/build.py); raises if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run `python ptx-std_b200/build.py` first")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().ptxstd_status_string(status).decode()


def check(status: int, what: str = "ptxstd") -> None:
    if status != OK:
        raise PtxStdError(status, what)


def _torch():
    import torch
    return torch


def _stream(stream=None) -> int:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def _dev(t) -> int:
    torch = _torch()
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return t.data_ptr()


def last_device_error(clear: bool = True, stream=None) -> tuple[int, int]:
    code, detail = C.c_int(0), C.c_uint32(0)
    check(lib().ptxstd_last_device_error(_stream(stream), int(clear), C.byref(code),
                                         C.byref(detail)), "last_device_error")
    return code.value, detail.value


from . import data_types, tcgen05  # noqa: E402
from .kernels import (MX_E2M1, MX_E2M3, MX_E3M2, MX_E4M3, MX_E5M2,  # noqa: E402
                      SCHEDULE_DYNAMIC, SCHEDULE_PERSISTENT, get_gemm_schedule, set_gemm_schedule,
                      gemm_decode, gemm_fp8, gemm_mx, gemm_mxfp8, gemm_mxfp8_sparse, gemm_nvfp4,
                      prune_24, quantize_mx, quantize_mxfp8, quantize_nvfp4,
                      tcgen05_cp_unpack)

__all__ = ["lib", "check", "PtxStdError", "status_string", "last_device_error", "data_types",
           "tcgen05", "quantize_mxfp8", "quantize_nvfp4", "quantize_mx", "gemm_fp8",
           "gemm_mxfp8", "gemm_mx", "gemm_nvfp4", "gemm_decode", "gemm_mxfp8_sparse", "prune_24",
           "tcgen05_cp_unpack", "set_gemm_schedule", "get_gemm_schedule", "SCHEDULE_PERSISTENT",
           "SCHEDULE_DYNAMIC",
           "MX_E4M3", "MX_E5M2", "MX_E2M3", "MX_E3M2", "MX_E2M1"]

"""The C ABI library loads without a GPU and exports every function include/*.h declares."""

import ctypes as C
import glob
import os
import re
import subprocess

from conftest import ROOT


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = open(h).read()
        names |= set(re.findall(r"PTXSTD_API\s+[\w\s\*]*?\b(ptxstd_\w+)\s*\(", src))
    return names


def test_exports_every_declared_symbol(ptxstd_lib):
    lib_path = ptxstd_lib.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (ptxstd_\w+)", out))
    declared = _declared()
    assert len(declared) >= 30
    missing = declared - exported
    assert not missing, sorted(missing)
    L = C.CDLL(lib_path)
    for name in declared:
        assert getattr(L, name) is not None


def test_no_undeclared_exports(ptxstd_lib):
    out = subprocess.run(["nm", "-D", "--defined-only", ptxstd_lib.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (\w+)", out))
    assert exported - _declared() == set() or all(not n.startswith("ptxstd_")
                                                  for n in exported - _declared())


def test_status_strings_and_version(ptxstd_lib):
    L = ptxstd_lib.lib()
    assert ptxstd_lib.status_string(0) == "ok"
    assert ptxstd_lib.status_string(ptxstd_lib.ETIMEOUT) == "device-side wait timed out"
    assert L.ptxstd_version() >= 100


def test_host_validation_without_gpu(ptxstd_lib):
    """Argument checks happen before any CUDA call, so they answer EINVAL on a CPU-only host."""
    L = ptxstd_lib.lib()
    EINVAL = ptxstd_lib.EINVAL
    assert L.ptxstd_quantize_mxfp8(None, 128, 96 + 1, None, None, None) == EINVAL
    assert L.ptxstd_quantize_mxfp8(None, 0, 64, None, None, None) == EINVAL
    assert L.ptxstd_quantize_nvfp4(None, 128, 64, 0.0, None, None, None) == EINVAL
    assert L.ptxstd_quantize_nvfp4_layout(16, 128, 64, 1.0, 16, 16, 2, None) == EINVAL
    assert L.ptxstd_cvt_f32_to_e2m1x2(16, 16, 3, 0, None) == EINVAL
    assert L.ptxstd_cvt_sweep(34, 0, 16, 16, None) == EINVAL
    assert L.ptxstd_cvt_sweep(12, 2, 16, 16, None) == EINVAL      # stochastic: base % 4
    assert L.ptxstd_cvt_f32_to_e2m1x2_rs(16, 16, 16, 3, 0, None) == EINVAL   # odd n
    assert L.ptxstd_cvt_f32_to_e4m3_rs(8, 16, 16, 4, 0, None) == EINVAL      # x not 16-aligned
    assert L.ptxstd_cvt_f32_to_bf16_rs(16, 2, 16, 4, 0, 0, None) == EINVAL   # rbits misaligned
    assert L.ptxstd_quantize_mxfp8_rs(16, 128, 96 + 1, 16, 16, 0, 1, None) == EINVAL
    assert L.ptxstd_quantize_nvfp4_rs(16, 128, 64, 0.0, 16, 16, 0, 1, None) == EINVAL
    assert L.ptxstd_cvt_sweep(0, (1 << 32) - 8, 16, 16, None) == EINVAL
    # MX element types are the tcgen05 codes 0, 1, 3, 4, 5 (2 is not one)
    assert L.ptxstd_quantize_mx(16, 128, 128, 2, 16, 16, 0, None) == EINVAL
    assert L.ptxstd_quantize_mx(16, 128, 96 + 1, 0, 16, 16, 0, None) == EINVAL
    assert L.ptxstd_gemm_mx(16, 2, 16, 16, 0, 16, 16, 256, 256, 128, None) == EINVAL
    assert L.ptxstd_gemm_mx(16, 0, 16, 16, 6, 16, 16, 256, 256, 128, None) == EINVAL
    assert L.ptxstd_gemm_mx(16, 3, 16, 16, 5, 16, 16, 256, 256, 100, None) == EINVAL


def test_dist_validation_without_gpu(ptxstd_lib):
    """The multi-GPU entry points reject a missing communicator or bad arguments before any CUDA
    or NCCL call."""
    from ptxstd import dist as D
    L = D._lib()
    EINVAL = ptxstd_lib.EINVAL
    out = C.c_void_p()
    assert L.ptxstd_dist_unique_id(None) == EINVAL
    assert L.ptxstd_dist_init(None, 2, 0, C.byref(out)) == EINVAL
    assert L.ptxstd_dist_init((C.c_uint8 * 128)(), 2, 2, C.byref(out)) == EINVAL  # rank >= nranks
    assert L.ptxstd_dist_free(None) == ptxstd_lib.OK
    assert L.ptxstd_gemm_nvfp4_sharded(None, 16, 16, 1.0, 16, 16, 1.0, 16, 256, 512, 256,
                                       None) == EINVAL
    assert L.ptxstd_gemm_decode_sharded_workspace_bytes(None, 16, 1024, 2048) == 0
    assert L.ptxstd_gemm_decode_sharded(None, 16, 16, 16, 1.0, 16, 16, 1024, 2048, 1024,
                                        1 << 20, None) == EINVAL
    y = C.c_void_p()
    assert L.ptxstd_dist_decode_p2p_init(None, 1024, C.byref(y)) == EINVAL
    assert L.ptxstd_gemm_decode_sharded_p2p(None, 16, 16, 16, 1.0, None, 16, 1024, 2048, 1024,
                                            1 << 20, None) == EINVAL


def test_integration_binding_names_exist():
    """Every function the Rust `extern "C"` block of INTEGRATION.md binds is declared in
    include/ptxstd.h (the documented binding cannot drift from the header)."""
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    bound = set(re.findall(r"pub fn (ptxstd_\w+)\s*\(", doc))
    assert bound, "no bindings found"
    missing = bound - _declared()
    assert not missing, sorted(missing)

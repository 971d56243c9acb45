"""ctypes loader for the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import this module, and
only to check results or to time the CPU baseline. It builds ``oracle/_build/liboracle.so`` from
``oracle/oracle.c`` with ``make`` when the library is missing.
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

E4M3, E5M2, E2M1, E2M3, E3M2 = 0, 1, 2, 3, 4
# the tcgen05 element-type codes of kind::f8f6f4 / mxf8f6f4 (F8f6f4ElementType,
# src/tcgen05/descriptor.rs:316-327) -> these formats
MMA_TYPE_TO_FORMAT = {0: E4M3, 1: E5M2, 3: E2M3, 4: E3M2, 5: E2M1}
(V_E4M3, V_E5M2, V_E2M1, V_E4M3_RELU, V_E5M2_RELU, V_E2M1_RELU, V_UE8M0_RZ,
 V_UE8M0_RP) = range(8)
VARIANT_NAMES = ["e4m3", "e5m2", "e2m1", "e4m3_relu", "e5m2_relu", "e2m1_relu", "ue8m0_rz",
                 "ue8m0_rp", "e2m3", "e3m2", "e2m3_relu", "e3m2_relu",
                 "e4m3_rs", "e5m2_rs", "e2m3_rs", "e3m2_rs", "e2m1_rs",
                 "e4m3_rs_relu", "e5m2_rs_relu", "e2m3_rs_relu", "e3m2_rs_relu", "e2m1_rs_relu",
                 "bf16_rs", "bf16_rs_relu", "bf16_rs_sat", "bf16_rs_relu_sat",
                 "f16_rs", "f16_rs_relu", "f16_rs_sat", "f16_rs_relu_sat",
                 "bf16_rn", "bf16_rn_relu", "bf16_rn_sat", "bf16_rn_relu_sat"]
# stochastic-rounding random-value kinds (ptxo_rs_random)
RS_X4, RS_E2M1, RS_BF16, RS_F16 = 0, 1, 2, 3
SWEEP_SEED = 0x2545F4914F6CDD1D

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: C.CDLL) -> None:
    u8, u16, u32, u64, i32, i64, f32 = (C.c_uint8, C.c_uint16, C.c_uint32, C.c_uint64, C.c_int,
                                        C.c_int64, C.c_float)
    p = C.c_void_p
    sigs = {
        "ptxo_minifloat_to_f32": (f32, [u8, u32, u32, C.c_int32, i32]),
        "ptxo_e4m3_to_f32": (f32, [u8]),
        "ptxo_e5m2_to_f32": (f32, [u8]),
        "ptxo_e2m1_to_f32": (f32, [u8]),
        "ptxo_ue8m0_to_f32": (f32, [u8]),
        "ptxo_to_f32_via_half": (f32, [i32, u8]),
        "ptxo_ue8m0_to_f32_via_bf16": (f32, [u8]),
        "ptxo_f32_to_e4m3": (u8, [f32, i32]),
        "ptxo_f32_to_e5m2": (u8, [f32, i32]),
        "ptxo_f32_to_e2m1": (u8, [f32, i32]),
        "ptxo_f32_to_narrow": (u8, [i32, f32, i32]),
        "ptxo_f32_to_ue8m0": (u8, [f32, i32, i32]),
        "ptxo_f32_to_bf16": (u16, [f32]),
        "ptxo_bf16_to_f32": (f32, [u16]),
        "ptxo_encode_array": (None, [i32, p, p, C.c_size_t, i32, i32]),
        "ptxo_decode_array": (None, [i32, p, p, C.c_size_t, i32]),
        "ptxo_ue8m0_encode_array": (None, [p, p, C.c_size_t, i32, i32, i32]),
        "ptxo_encode_variant": (u8, [i32, f32]),
        "ptxo_sweep_compare": (u64, [i32, u64, u64, p, p, u64, i32]),
        "ptxo_sweep_digest": (u64, [i32, u64, u64, i32]),
        "ptxo_fnv1a64": (u64, [p, C.c_size_t, u64]),
        "ptxo_digest_bytes": (u64, [p, u64, i32]),
        "ptxo_quantize_mxfp8": (None, [p, i64, i64, p, p, i32]),
        "ptxo_quantize_nvfp4": (i32, [p, i64, i64, f32, p, p, i32]),
        "ptxo_gemm_fp8_ref": (None, [p, p, i64, i64, i64, f32, f32, p, p, i64, p, p, i32]),
        "ptxo_gemm_nvfp4_ref": (None, [p, p, f32, p, p, f32, i64, i64, i64, p, p, i64, p, p,
                                       i32]),
        "ptxo_gemm_decode_ref": (None, [p, p, p, f32, i64, i64, i64, p, p, i64, p, p, i32]),
        "ptxo_gemm_mxfp8_ref": (None, [p, p, p, p, i64, i64, i64, p, p, i64, p, p, i32]),
        "ptxo_mx_pack": (None, [i32, p, p, C.c_size_t]),
        "ptxo_mx_unpack": (None, [i32, p, p, C.c_size_t]),
        "ptxo_cp_unpack": (None, [i32, p, p, C.c_size_t]),
        "ptxo_quantize_mx": (None, [p, i64, i64, i32, p, p, i32]),
        "ptxo_gemm_mx_ref": (None, [p, i32, p, p, i32, p, i64, i64, i64, p, p, i64, p, p, i32]),
        "ptxo_sgemm_nt": (None, [p, p, p, i64, i64, i64, i32]),
        "ptxo_idesc_f16": (i32, [i32, i32, i32, u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_tf32": (i32, [u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_f8f6f4": (i32, [i32, i32, i32, u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_i8": (i32, [i32, i32, u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_mxf8f6f4": (i32, [i32, i32, u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_mxf4": (i32, [u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_mxf4nvf4": (i32, [i32, u32, u32, C.POINTER(u32)]),
        "ptxo_idesc_with_field": (i32, [u32, u32, u32, u32, C.POINTER(u32)]),
        "ptxo_smem_desc": (i32, [u32, u32, u32, i32, C.POINTER(u64)]),
        "ptxo_smem_desc_with_base_offset": (i32, [u64, u32, C.POINTER(u64)]),
        "ptxo_smem_desc_add_start_bytes": (i32, [u64, u32, C.POINTER(u64)]),
        "ptxo_zero_mask_new": (i32, [u32, u32, C.POINTER(u64)]),
        "ptxo_zero_mask_with_sub_mask_start": (i32, [u64, u32, i32, u32, C.POINTER(u64)]),
        "ptxo_zero_mask_with_column_shift": (i32, [u64, u32, C.POINTER(u64)]),
        "ptxo_hardware_threads": (i32, []),
        "ptxo_rs_random": (u32, [i32, u32, i32]),
        "ptxo_f32_to_narrow_rs": (u8, [i32, f32, u32, i32]),
        "ptxo_f32_to_bf16_rs": (u16, [f32, u32, i32, i32]),
        "ptxo_f32_to_f16_rs": (u16, [f32, u32, i32, i32]),
        "ptxo_encode_rs_array": (None, [i32, p, p, p, C.c_size_t, i32, i32]),
        "ptxo_bf16_rs_array": (None, [p, p, p, C.c_size_t, i32, i32, i32]),
        "ptxo_f16_rs_array": (None, [p, p, p, C.c_size_t, i32, i32, i32]),
        "ptxo_splitmix64": (u64, [u64, u64]),
        "ptxo_sr_rbits": (u32, [u64, u64]),
        "ptxo_sweep_code": (u32, [i32, u64]),
        "ptxo_sweep_width": (i32, [i32]),
        "ptxo_quantize_mxfp8_rs": (None, [p, i64, i64, u64, p, p, i32]),
        "ptxo_prune_24": (None, [p, i64, i64, p, p, i32]),
        "ptxo_to_bf16_scaled": (u16, [i32, u8, u8, i32, i32]),
        "ptxo_f32_to_bf16_mode": (u16, [f32, i32, i32]),
        "ptxo_narrow_to_f16": (u16, [i32, u8]),
        "ptxo_to_bf16_scaled_array": (None, [i32, p, p, p, C.c_size_t, C.c_size_t, i32, i32, i32]),
        "ptxo_decompress_24": (None, [p, p, i64, i64, p, i32]),
        "ptxo_gemm_mxfp8_sparse_ref": (None, [p, p, p, p, p, i64, i64, i64, p, p, i64, p, p,
                                              i32]),
        "ptxo_quantize_nvfp4_rs": (i32, [p, i64, i64, f32, u64, p, p, i32]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ---- numpy conveniences ------------------------------------------------------------------------

def encode(fmt: int, x: np.ndarray, relu: bool = False, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    out = np.empty(n // 2 if fmt == E2M1 else n, dtype=np.uint8)
    lib().ptxo_encode_array(fmt, _ptr(x), _ptr(out), n, int(relu), threads)
    return out


def decode(fmt: int, codes: np.ndarray, threads: int = 0) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    n = codes.size * 2 if fmt == E2M1 else codes.size
    out = np.empty(n, dtype=np.float32)
    lib().ptxo_decode_array(fmt, _ptr(codes), _ptr(out), n, threads)
    return out


def ue8m0_encode(x: np.ndarray, rnd_up: bool = False, satfinite: bool = True,
                 threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.uint8)
    lib().ptxo_ue8m0_encode_array(_ptr(x), _ptr(out), x.size, int(rnd_up), int(satfinite),
                                  threads)
    return out


def quantize_mxfp8(x_bf16: np.ndarray, threads: int = 0):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    q = np.empty((rows, cols), dtype=np.uint8)
    sf = np.empty((rows, cols // 32), dtype=np.uint8)
    lib().ptxo_quantize_mxfp8(_ptr(x), rows, cols, _ptr(q), _ptr(sf), threads)
    return q, sf


def quantize_nvfp4(x_bf16: np.ndarray, g: float, threads: int = 0):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    q = np.empty((rows, cols // 2), dtype=np.uint8)
    sf = np.empty((rows, cols // 16), dtype=np.uint8)
    rc = lib().ptxo_quantize_nvfp4(_ptr(x), rows, cols, float(g), _ptr(q), _ptr(sf), threads)
    if rc != 0:
        raise ValueError("bad global scale")
    return q, sf


def _samples(rows, cols):
    r = np.ascontiguousarray(rows, dtype=np.int64)
    c = np.ascontiguousarray(cols, dtype=np.int64)
    return r, c, np.empty(r.size), np.empty(r.size)


def gemm_fp8_ref(A, B, sa, sb, rows, cols, threads=0):
    A = np.ascontiguousarray(A, dtype=np.uint8)
    B = np.ascontiguousarray(B, dtype=np.uint8)
    (M, K), N = A.shape, B.shape[0]
    r, c, ref, mag = _samples(rows, cols)
    lib().ptxo_gemm_fp8_ref(_ptr(A), _ptr(B), M, N, K, sa, sb, _ptr(r), _ptr(c), r.size,
                            _ptr(ref), _ptr(mag), threads)
    return ref, mag


def gemm_nvfp4_ref(A, sfA, ga, B, sfB, gb, rows, cols, threads=0):
    A, sfA, B, sfB = (np.ascontiguousarray(t, dtype=np.uint8) for t in (A, sfA, B, sfB))
    M, K = A.shape[0], A.shape[1] * 2
    N = B.shape[0]
    r, c, ref, mag = _samples(rows, cols)
    lib().ptxo_gemm_nvfp4_ref(_ptr(A), _ptr(sfA), ga, _ptr(B), _ptr(sfB), gb, M, N, K, _ptr(r),
                              _ptr(c), r.size, _ptr(ref), _ptr(mag), threads)
    return ref, mag


def gemm_mxfp8_ref(A, sfA, B, sfB, rows, cols, threads=0):
    """MXFP8 GEMM reference at sampled outputs; scales row-major [rows, K/32]."""
    A, sfA, B, sfB = (np.ascontiguousarray(t, dtype=np.uint8) for t in (A, sfA, B, sfB))
    (M, K), N = A.shape, B.shape[0]
    r, c, ref, mag = _samples(rows, cols)
    lib().ptxo_gemm_mxfp8_ref(_ptr(A), _ptr(sfA), _ptr(B), _ptr(sfB), M, N, K, _ptr(r), _ptr(c),
                              r.size, _ptr(ref), _ptr(mag), threads)
    return ref, mag


def mx_pack(fmt: int, codes: np.ndarray) -> np.ndarray:
    """One code per byte -> the tcgen05 operand layout (FP6/FP4 groups of 16 padded to 16 bytes);
    the last axis is the K axis (a multiple of 16)."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    out = np.empty_like(c)
    lib().ptxo_mx_pack(fmt, _ptr(c), _ptr(out), c.size)
    return out


def mx_unpack(fmt: int, packed: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.empty_like(p)
    lib().ptxo_mx_unpack(fmt, _ptr(p), _ptr(out), p.size)
    return out


def cp_unpack(fmt: int, packed: np.ndarray) -> np.ndarray:
    """The 8-bit containers of tcgen05.cp's FP6 / FP4 decompression, one per element."""
    p_ = np.ascontiguousarray(packed, dtype=np.uint8)
    out = np.empty_like(p_)
    lib().ptxo_cp_unpack(fmt, _ptr(p_), _ptr(out), p_.size)
    return out


def quantize_mx(x_bf16: np.ndarray, fmt: int, threads: int = 0):
    """OCP MX quantisation to `fmt` (E4M3 .. E3M2): (q [rows, cols] packed, sf [rows, cols/32])."""
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    q = np.empty((rows, cols), dtype=np.uint8)
    sf = np.empty((rows, cols // 32), dtype=np.uint8)
    lib().ptxo_quantize_mx(_ptr(x), rows, cols, fmt, _ptr(q), _ptr(sf), threads)
    return q, sf


def gemm_mx_ref(A, fa, sfA, B, fb, sfB, rows, cols, threads=0):
    """MX GEMM reference at sampled outputs: packed operands of formats fa / fb, row-major
    UE8M0 scales [rows, K/32]."""
    A, sfA, B, sfB = (np.ascontiguousarray(t, dtype=np.uint8) for t in (A, sfA, B, sfB))
    (M, K), N = A.shape, B.shape[0]
    r, c, ref, mag = _samples(rows, cols)
    lib().ptxo_gemm_mx_ref(_ptr(A), fa, _ptr(sfA), _ptr(B), fb, _ptr(sfB), M, N, K, _ptr(r),
                           _ptr(c), r.size, _ptr(ref), _ptr(mag), threads)
    return ref, mag


def to_bf16_scaled(fmt: int, codes: np.ndarray, scales: np.ndarray, n: int, block: int = 1,
                   relu: bool = False, satfinite: bool = False, threads: int = 0) -> np.ndarray:
    """bf16 bit patterns of n narrow codes times their UE8M0 scales (scales[i // block])."""
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    sc = np.ascontiguousarray(scales, dtype=np.uint8)
    out = np.empty(n, dtype=np.uint16)
    lib().ptxo_to_bf16_scaled_array(fmt, _ptr(c), _ptr(sc), _ptr(out), n, block, int(relu),
                                    int(satfinite), threads)
    return out


def prune_24(codes: np.ndarray, threads: int = 0):
    """2:4 magnitude pruning of E4M3 codes [rows, cols] -> (vals [rows, cols/2], meta [rows, cols/8])."""
    x = np.ascontiguousarray(codes, dtype=np.uint8)
    rows, cols = x.shape
    vals = np.empty((rows, cols // 2), dtype=np.uint8)
    meta = np.empty((rows, cols // 8), dtype=np.uint8)
    lib().ptxo_prune_24(_ptr(x), rows, cols, _ptr(vals), _ptr(meta), threads)
    return vals, meta


def decompress_24(vals: np.ndarray, meta: np.ndarray, threads: int = 0) -> np.ndarray:
    v = np.ascontiguousarray(vals, dtype=np.uint8)
    m = np.ascontiguousarray(meta, dtype=np.uint8)
    rows, cols = v.shape[0], v.shape[1] * 2
    out = np.empty((rows, cols), dtype=np.uint8)
    lib().ptxo_decompress_24(_ptr(v), _ptr(m), rows, cols, _ptr(out), threads)
    return out


def gemm_mxfp8_sparse_ref(vals, meta, sfA, B, sfB, rows, cols, threads=0):
    """2:4-sparse MXFP8 GEMM reference at sampled outputs; scales row-major [rows, K/64]."""
    vals, meta, sfA, B, sfB = (np.ascontiguousarray(t, dtype=np.uint8)
                               for t in (vals, meta, sfA, B, sfB))
    M, K = vals.shape[0], vals.shape[1] * 2
    N = B.shape[0]
    r, c, ref, mag = _samples(rows, cols)
    lib().ptxo_gemm_mxfp8_sparse_ref(_ptr(vals), _ptr(meta), _ptr(sfA), _ptr(B), _ptr(sfB), M, N,
                                     K, _ptr(r), _ptr(c), r.size, _ptr(ref), _ptr(mag), threads)
    return ref, mag


def gemm_decode_ref(x_bf16, W, sfW, gw, rows, cols, threads=0):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    W, sfW = (np.ascontiguousarray(t, dtype=np.uint8) for t in (W, sfW))
    M, K = x.shape
    N = W.shape[0]
    r, c, ref, mag = _samples(rows, cols)
    lib().ptxo_gemm_decode_ref(_ptr(x), _ptr(W), _ptr(sfW), gw, M, N, K, _ptr(r), _ptr(c),
                               r.size, _ptr(ref), _ptr(mag), threads)
    return ref, mag


def sgemm_nt(A, B, threads=0):
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    N = B.shape[0]
    Cm = np.empty((M, N), dtype=np.float32)
    lib().ptxo_sgemm_nt(_ptr(A), _ptr(B), _ptr(Cm), M, N, K, threads)
    return Cm


def sweep_width(variant: int) -> int:
    """Bytes per input of a sweep variant (2 for the bf16/f16 stochastic forms)."""
    return int(lib().ptxo_sweep_width(variant))


def sweep_compare(variant: int, base: int, dev_codes: np.ndarray, max_report: int = 64,
                  threads: int = 0):
    dev = np.ascontiguousarray(dev_codes, dtype=np.uint8)
    rep = np.zeros((max_report, 3), dtype=np.uint32)
    n = lib().ptxo_sweep_compare(variant, base, dev.size // sweep_width(variant), _ptr(dev),
                                 _ptr(rep), max_report, threads)
    return int(n), rep[: min(int(n), max_report)]


def encode_rs(fmt: int, x: np.ndarray, rbits: np.ndarray, relu: bool = False,
              threads: int = 0) -> np.ndarray:
    """Stochastic rounding of x (f32) with rbits[i // 4] (E2M1 packed two per byte)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rb = np.ascontiguousarray(rbits, dtype=np.uint32)
    assert rb.size >= (x.size + 3) // 4
    out = np.empty(x.size // 2 if fmt == E2M1 else x.size, dtype=np.uint8)
    lib().ptxo_encode_rs_array(fmt, _ptr(x), _ptr(rb), _ptr(out), x.size, int(relu), threads)
    return out


def bf16_rs(x: np.ndarray, rbits: np.ndarray, relu=False, satfinite=False, threads=0):
    """Stochastic rounding f32 -> bf16 bit patterns with rbits[i // 2]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rb = np.ascontiguousarray(rbits, dtype=np.uint32)
    assert rb.size >= (x.size + 1) // 2
    out = np.empty(x.size, dtype=np.uint16)
    lib().ptxo_bf16_rs_array(_ptr(x), _ptr(rb), _ptr(out), x.size, int(relu), int(satfinite),
                             threads)
    return out


def f16_rs(x: np.ndarray, rbits: np.ndarray, relu=False, satfinite=False, threads=0):
    """Stochastic rounding f32 -> f16 bit patterns with rbits[i // 2]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    rb = np.ascontiguousarray(rbits, dtype=np.uint32)
    assert rb.size >= (x.size + 1) // 2
    out = np.empty(x.size, dtype=np.uint16)
    lib().ptxo_f16_rs_array(_ptr(x), _ptr(rb), _ptr(out), x.size, int(relu), int(satfinite),
                            threads)
    return out


def sr_rbits(seed: int, groups: int) -> np.ndarray:
    """rbits of groups 0 .. groups-1 of the seeded quantisers (vectorised SplitMix64)."""
    g = np.arange((groups + 1) // 2, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = np.uint64(seed) + (g + np.uint64(1)) * np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z.view(np.uint32)[:groups].copy()


def quantize_mxfp8_rs(x_bf16: np.ndarray, seed: int, threads: int = 0):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    q = np.empty((rows, cols), dtype=np.uint8)
    sf = np.empty((rows, cols // 32), dtype=np.uint8)
    lib().ptxo_quantize_mxfp8_rs(_ptr(x), rows, cols, seed, _ptr(q), _ptr(sf), threads)
    return q, sf


def quantize_nvfp4_rs(x_bf16: np.ndarray, g: float, seed: int, threads: int = 0):
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    rows, cols = x.shape
    q = np.empty((rows, cols // 2), dtype=np.uint8)
    sf = np.empty((rows, cols // 16), dtype=np.uint8)
    if lib().ptxo_quantize_nvfp4_rs(_ptr(x), rows, cols, float(g), seed, _ptr(q), _ptr(sf),
                                    threads) != 0:
        raise ValueError("bad global scale")
    return q, sf


def sweep_digest(variant: int, base: int, n: int, threads: int = 0) -> int:
    return int(lib().ptxo_sweep_digest(variant, base, n, threads))


def digest_bytes(data: np.ndarray, threads: int = 0) -> int:
    d = np.ascontiguousarray(data, dtype=np.uint8)
    return int(lib().ptxo_digest_bytes(_ptr(d), d.size, threads))


def fnv1a64(data: np.ndarray, seed: int = 0) -> int:
    d = np.ascontiguousarray(data, dtype=np.uint8)
    return int(lib().ptxo_fnv1a64(_ptr(d), d.size, seed))


def bf16_from_f32(x: np.ndarray) -> np.ndarray:
    """RNE f32 -> bf16 bit patterns (vectorised numpy restatement of ptxo_f32_to_bf16)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r = np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)

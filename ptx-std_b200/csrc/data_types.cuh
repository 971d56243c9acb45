// Device conversions of the narrow formats: the B200 form of ptx-std's data_types module
// (src/data_types/narrow.rs, float8.rs, float4.rs). Each pair function is the one `cvt`
// instruction the reference's pair_* method wraps; element 0 of a pair always lands in the least
// significant bits, so the PTX operands are swapped (`cvt` puts operand a in the upper half,
// src/data_types/narrow.rs:18-21).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace ptxstd::data_types {

// ---- f32 -> narrow, RN .satfinite [.relu] ---------------------------------------------------
// f8e4m3x2::pair_from_f32 (narrow.rs:156-162): cvt.rn.satfinite{.relu}.e4m3x2.f32.
template <bool RELU = false>
__device__ __forceinline__ uint16_t e4m3x2_from_f32(float x0, float x1) {
    uint16_t r;
    if constexpr (RELU)
        asm("cvt.rn.satfinite.relu.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else
        asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    return r;
}
// f8e5m2x2::pair_from_f32: cvt.rn.satfinite{.relu}.e5m2x2.f32.
template <bool RELU = false>
__device__ __forceinline__ uint16_t e5m2x2_from_f32(float x0, float x1) {
    uint16_t r;
    if constexpr (RELU)
        asm("cvt.rn.satfinite.relu.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else
        asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    return r;
}
// f6e2m3x2 / f6e3m2x2::pair_from_f32 (src/data_types/float6.rs, narrow_cvt! core from_f32):
// cvt.rn.satfinite{.relu}.e2m3x2.f32 / .e3m2x2.f32, one value in the low 6 bits of each byte,
// x0 in the low byte.
template <bool RELU = false>
__device__ __forceinline__ uint16_t e2m3x2_from_f32(float x0, float x1) {
    uint16_t r;
    if constexpr (RELU)
        asm("cvt.rn.satfinite.relu.e2m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else
        asm("cvt.rn.satfinite.e2m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    return r;
}
template <bool RELU = false>
__device__ __forceinline__ uint16_t e3m2x2_from_f32(float x0, float x1) {
    uint16_t r;
    if constexpr (RELU)
        asm("cvt.rn.satfinite.relu.e3m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else
        asm("cvt.rn.satfinite.e3m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    return r;
}
// f4e2m1x2::pair_from_f32: cvt.rn.satfinite{.relu}.e2m1x2.f32 (one byte, x0 in the low nibble).
template <bool RELU = false>
__device__ __forceinline__ uint32_t e2m1x2_from_f32(float x0, float x1) {
    uint32_t r;
    if constexpr (RELU)
        asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.relu.e2m1x2.f32 t, %1, %2;\n\t"
            "cvt.u32.u8 %0, t;\n\t}"
            : "=r"(r)
            : "f"(x1), "f"(x0));
    else
        asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
            "cvt.u32.u8 %0, t;\n\t}"
            : "=r"(r)
            : "f"(x1), "f"(x0));
    return r;
}
// Four E2M1 values packed in 16 bits (element 0 in bits 0..3).
__device__ __forceinline__ uint32_t e2m1x4_from_f32(float x0, float x1, float x2, float x3) {
    return e2m1x2_from_f32(x0, x1) | (e2m1x2_from_f32(x2, x3) << 8);
}

// ---- f32 -> narrow, stochastic rounding (.rs, sm_100a) -----------------------------------------
// quad_from_f32_stochastic (narrow.rs:217-229): cvt.rs.satfinite{.relu}.<fmt>x4.f32 d,
// {x3, x2, x1, x0}, rbits -- element 0 in the least significant bits of d. Each element is
// truncated toward zero unless its random value plus the discarded mantissa bits carries; the
// random bits of the four elements come from rbits as the reference documents per format
// (float8.rs:59, float6.rs:61, float4.rs:60).
#define PTXSTD_RS_X4(NAME, TY, RES, CONS)                                                        \
    template <bool RELU = false>                                                                 \
    __device__ __forceinline__ uint32_t NAME(float x0, float x1, float x2, float x3,             \
                                             uint32_t rbits) {                                   \
        RES r;                                                                                   \
        if constexpr (RELU)                                                                      \
            asm("cvt.rs.relu.satfinite." TY ".f32 %0, {%1, %2, %3, %4}, %5;"                     \
                : "=" CONS(r)                                                                    \
                : "f"(x3), "f"(x2), "f"(x1), "f"(x0), "r"(rbits));                               \
        else                                                                                     \
            asm("cvt.rs.satfinite." TY ".f32 %0, {%1, %2, %3, %4}, %5;"                          \
                : "=" CONS(r)                                                                    \
                : "f"(x3), "f"(x2), "f"(x1), "f"(x0), "r"(rbits));                               \
        return static_cast<uint32_t>(r);                                                         \
    }
PTXSTD_RS_X4(e4m3x4_from_f32_rs, "e4m3x4", uint32_t, "r")
PTXSTD_RS_X4(e5m2x4_from_f32_rs, "e5m2x4", uint32_t, "r")
PTXSTD_RS_X4(e2m3x4_from_f32_rs, "e2m3x4", uint32_t, "r")
PTXSTD_RS_X4(e3m2x4_from_f32_rs, "e3m2x4", uint32_t, "r")
PTXSTD_RS_X4(e2m1x4_from_f32_rs, "e2m1x4", uint16_t, "h")  // 16 bits, element 0 in bits 0..3
#undef PTXSTD_RS_X4

// bf16x2 / f16x2::pair_from_f32_stochastic::<R, O> (bfloat16.rs:456-462, float16.rs:589-595):
// cvt.rs{.relu}{.satfinite}.{bf16x2,f16x2}.f32 d, x1, x0, rbits; the low half of rbits serves
// element 0.
#define PTXSTD_RS_X2(NAME, TY)                                                                   \
    template <bool RELU, bool SAT>                                                               \
    __device__ __forceinline__ uint32_t NAME(float x0, float x1, uint32_t rbits) {               \
        uint32_t r;                                                                              \
        if constexpr (RELU && SAT)                                                               \
            asm("cvt.rs.relu.satfinite." TY ".f32 %0, %1, %2, %3;"                               \
                : "=r"(r) : "f"(x1), "f"(x0), "r"(rbits));                                       \
        else if constexpr (RELU)                                                                 \
            asm("cvt.rs.relu." TY ".f32 %0, %1, %2, %3;" : "=r"(r) : "f"(x1), "f"(x0), "r"(rbits)); \
        else if constexpr (SAT)                                                                  \
            asm("cvt.rs.satfinite." TY ".f32 %0, %1, %2, %3;"                                    \
                : "=r"(r) : "f"(x1), "f"(x0), "r"(rbits));                                       \
        else                                                                                     \
            asm("cvt.rs." TY ".f32 %0, %1, %2, %3;" : "=r"(r) : "f"(x1), "f"(x0), "r"(rbits));    \
        return r;                                                                                \
    }
PTXSTD_RS_X2(bf16x2_from_f32_rs, "bf16x2")
PTXSTD_RS_X2(f16x2_from_f32_rs, "f16x2")
#undef PTXSTD_RS_X2

// Counter-based random bits for the seeded stochastic-rounding quantisers: output i of SplitMix64
// (Steele, Lea and Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014) started
// at `seed`. Group g of four consecutive elements takes the low (g even) or high (g odd) word of
// output g / 2, so an 8-element vector takes both words of one output.
__device__ __forceinline__ uint64_t splitmix64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// ---- f16 -> narrow ------------------------------------------------------------------------------
// f8e4m3x2 / f8e5m2x2::pair_from_f16 (narrow.rs:164-172): cvt.rn.satfinite{.relu}.e4m3x2.f16x2,
// element 0 in the low half of the f16x2 word and in the low byte of the result.
template <bool RELU>
__device__ __forceinline__ uint16_t e4m3x2_from_f16x2(uint32_t h2) {
    uint16_t r;
    if constexpr (RELU) asm("cvt.rn.satfinite.relu.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(h2));
    else asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(h2));
    return r;
}
template <bool RELU>
__device__ __forceinline__ uint16_t e5m2x2_from_f16x2(uint32_t h2) {
    uint16_t r;
    if constexpr (RELU) asm("cvt.rn.satfinite.relu.e5m2x2.f16x2 %0, %1;" : "=h"(r) : "r"(h2));
    else asm("cvt.rn.satfinite.e5m2x2.f16x2 %0, %1;" : "=h"(r) : "r"(h2));
    return r;
}
// The exact f16 -> f32 widening of both halves (element 0 = low half).
__device__ __forceinline__ float2 f16x2_to_f32(uint32_t h2) {
    __half2 h = *reinterpret_cast<__half2*>(&h2);
    return __half22float2(h);
}

// f8e8m0x2::pair_from_f32::<RND, OVERFLOW> (narrow.rs:600-617): RZ or RP, optional .satfinite.
template <bool ROUND_UP, bool SATFINITE>
__device__ __forceinline__ uint16_t ue8m0x2_from_f32(float x0, float x1) {
    uint16_t r;
    if constexpr (ROUND_UP && SATFINITE)
        asm("cvt.rp.satfinite.ue8m0x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else if constexpr (ROUND_UP)
        asm("cvt.rp.ue8m0x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else if constexpr (SATFINITE)
        asm("cvt.rz.satfinite.ue8m0x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    else
        asm("cvt.rz.ue8m0x2.f32 %0, %1, %2;" : "=h"(r) : "f"(x1), "f"(x0));
    return r;
}
// Scalar form: the pair instruction with a zero lane (narrow.rs:243-247, :660-664).
template <bool ROUND_UP, bool SATFINITE>
__device__ __forceinline__ uint32_t ue8m0_from_f32(float x) {
    return ue8m0x2_from_f32<ROUND_UP, SATFINITE>(x, 0.0f) & 0xFFu;
}

// ---- narrow -> f32 (exact) ---------------------------------------------------------------------
// to_f32 = to_f16 then the exact widening (narrow.rs:292-299).
__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t h2) {
    __half2 h = *reinterpret_cast<__half2*>(&h2);
    return __half22float2(h);
}
__device__ __forceinline__ float2 e4m3x2_to_f32(uint16_t codes) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(codes));
    return half2_bits_to_float2(h2);
}
__device__ __forceinline__ float2 e5m2x2_to_f32(uint16_t codes) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(codes));
    return half2_bits_to_float2(h2);
}
__device__ __forceinline__ float2 e2m1x2_to_f32(uint32_t byte) {
    uint32_t h2;
    asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
        : "=r"(h2)
        : "r"(byte));
    return half2_bits_to_float2(h2);
}
// FP6 to_f32 = to_f16 (cvt.rn.f16x2.e2m3x2 / .e3m2x2, exact) then widening.
__device__ __forceinline__ float2 e2m3x2_to_f32(uint16_t codes) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e2m3x2 %0, %1;" : "=r"(h2) : "h"(codes));
    return half2_bits_to_float2(h2);
}
__device__ __forceinline__ float2 e3m2x2_to_f32(uint16_t codes) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e3m2x2 %0, %1;" : "=r"(h2) : "h"(codes));
    return half2_bits_to_float2(h2);
}
// to_f16 (narrow.rs:275-291): the exact cvt.rn.f16x2.<fmt>x2 result itself.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t c) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c));
    return h2;
}
__device__ __forceinline__ uint32_t e5m2x2_to_f16x2(uint16_t c) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e5m2x2 %0, %1;" : "=r"(h2) : "h"(c));
    return h2;
}
__device__ __forceinline__ uint32_t e2m3x2_to_f16x2(uint16_t c) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e2m3x2 %0, %1;" : "=r"(h2) : "h"(c));
    return h2;
}
__device__ __forceinline__ uint32_t e3m2x2_to_f16x2(uint16_t c) {
    uint32_t h2;
    asm("cvt.rn.f16x2.e3m2x2 %0, %1;" : "=r"(h2) : "h"(c));
    return h2;
}
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint32_t byte) {
    uint32_t h2;
    asm("{\n\t.reg .b8 t;\n\tcvt.u8.u32 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h2) : "r"(byte));
    return h2;
}
// ue8m0 to_f32 = to_bf16 then widening (narrow.rs:683-690): cvt.rn.bf16x2.ue8m0x2.
__device__ __forceinline__ float2 ue8m0x2_to_f32(uint16_t codes) {
    uint32_t b2;
    asm("cvt.rn.bf16x2.ue8m0x2 %0, %1;" : "=r"(b2) : "h"(codes));
    return make_float2(__uint_as_float(b2 << 16), __uint_as_float(b2 & 0xFFFF0000u));
}
// One E4M3 code -> f32, exact.
__device__ __forceinline__ float e4m3_to_f32(uint32_t code) {
    return e4m3x2_to_f32(static_cast<uint16_t>(code & 0xFFu)).x;
}

// ---- bf16 ------------------------------------------------------------------------------------
// bf16::to_f32 (src/data_types/bfloat16.rs:84-86): exact widening of the two halves of a word.
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// bf16x2 from two f32, RN (bfloat16.rs:104-118): cvt.rn.bf16x2.f32, x0 in the low half.
__device__ __forceinline__ uint32_t bf16x2_from_f32(float x0, float x1) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    return r;
}

// Both bf16 halves of a word, widened exactly to f32 and multiplied by `s` with round-to-nearest:
// one mul.rn.f32x2 (sm_100's packed f32 multiply, two IEEE products; the same results as two
// __fmul_rn). .x is the low half (element 0).
__device__ __forceinline__ float2 bf16x2_mul_f32(uint32_t w, float s) {
    const uint64_t a = (static_cast<uint64_t>(w & 0xFFFF0000u) << 32) | (w << 16);
    const uint64_t b = (static_cast<uint64_t>(__float_as_uint(s)) << 32) | __float_as_uint(s);
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return make_float2(__uint_as_float(static_cast<uint32_t>(r)),
                       __uint_as_float(static_cast<uint32_t>(r >> 32)));
}

// bf16x2::pair_from_f32_with::<Rn, R, O> (bfloat16.rs:446-454): cvt.rn{.relu}{.satfinite}.bf16x2.f32,
// x0 in the low half.
template <bool RELU, bool SAT>
__device__ __forceinline__ uint32_t bf16x2_from_f32_mode(float x0, float x1) {
    uint32_t r;
    if constexpr (RELU && SAT)
        asm("cvt.rn.relu.satfinite.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    else if constexpr (RELU)
        asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    else if constexpr (SAT)
        asm("cvt.rn.satfinite.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    else
        asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(x1), "f"(x0));
    return r;
}

// ---- block-scale helpers -------------------------------------------------------------------
// NaN-propagating amax of the |bf16| values in a word pair: for non-negative bf16 patterns the
// integer order is the float order, and every NaN pattern sorts above infinity, so an unsigned
// 16-bit max of the magnitudes is reduce_f32::<Max, Absolute> with NaN propagation
// (src/warp_collectives.rs:679-700) computed on the raw bits.
__device__ __forceinline__ uint32_t bf16x2_absmax_bits(uint32_t a, uint32_t b) {
    return __vmaxu2(a & 0x7FFF7FFFu, b & 0x7FFF7FFFu);
}
__device__ __forceinline__ uint32_t bf16x2_fold(uint32_t m2) {
    return max(m2 & 0xFFFFu, m2 >> 16);
}

// 2^-(code-127) as f32 for a UE8M0 scale code (2^127 .. 2^-127, the last an f32 subnormal);
// NaN for the NaN code 0xff.
__device__ __forceinline__ float ue8m0_inverse(uint32_t code) {
    if (code == 0xFFu) return __uint_as_float(0x7FFFFFFFu);
    const int e = 127 - static_cast<int>(code);
    return e >= -126 ? __uint_as_float(static_cast<uint32_t>(e + 127) << 23)
                     : __uint_as_float(0x00400000u);
}

// MXFP8 scale code of a block from its amax: from_f32::<TowardZero, SaturateFinite>(amax) minus
// E4M3's emax (8), clamped at 0; NaN stays NaN.
__device__ __forceinline__ uint32_t mxfp8_scale_code(float amax) {
    const uint32_t u = ue8m0_from_f32<false, true>(amax);
    return u == 0xFFu ? 0xFFu : (u > 8u ? u - 8u : 0u);
}

}  // namespace ptxstd::data_types

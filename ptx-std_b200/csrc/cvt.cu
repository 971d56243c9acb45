// Element-wise conversion kernels of the narrow formats (the reference's Vector<E, N>::from_f32 /
// to_f32 family, src/data_types/narrow.rs:354-425, applied over device arrays), their
// stochastic-rounding forms (from_f32_stochastic, narrow.rs:494-505; bf16/f16
// bfloat16.rs:572-598, float16.rs:740-766), plus the exhaustive-sweep kernel that converts f32
// bit patterns generated from the thread index.
#include "common.cuh"
#include "data_types.cuh"

namespace dt = ptxstd::data_types;

namespace {

enum Op : int { kE4M3 = 0, kE5M2 = 1, kE2M1 = 2, kE2M3 = 3, kE3M2 = 4 };

// One f32 pair -> two one-byte codes (x0 in the low byte) for the byte-per-element formats.
template <int OP, bool RELU>
__device__ __forceinline__ uint32_t encode_pair(float x0, float x1) {
    if constexpr (OP == kE4M3) return dt::e4m3x2_from_f32<RELU>(x0, x1);
    else if constexpr (OP == kE5M2) return dt::e5m2x2_from_f32<RELU>(x0, x1);
    else if constexpr (OP == kE2M3) return dt::e2m3x2_from_f32<RELU>(x0, x1);
    else return dt::e3m2x2_from_f32<RELU>(x0, x1);
}

// f32 -> FP8 or FP6 (one code per byte), 4 elements per thread per step (one 16-byte load, one
// 4-byte store).
template <int OP, bool RELU>
__global__ void __launch_bounds__(256) encode_fp8_kernel(const float* __restrict__ x,
                                                         uint8_t* __restrict__ out, size_t n) {
    const size_t n4 = n / 4;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        const uint32_t lo = encode_pair<OP, RELU>(v.x, v.y);
        const uint32_t hi = encode_pair<OP, RELU>(v.z, v.w);
        reinterpret_cast<uint32_t*>(out)[i] = lo | (hi << 16);
    }
    // Tail: the scalar form is the pair instruction with a zero lane (narrow.rs:243-247).
    const size_t t = n4 * 4 + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t < n) {
        out[t] = static_cast<uint8_t>(encode_pair<OP, RELU>(x[t], 0.0f) & 0xFFu);
    }
}

// f32 -> E2M1x2, 8 elements (4 bytes) per thread per step.
template <bool RELU>
__global__ void __launch_bounds__(256) encode_e2m1_kernel(const float* __restrict__ x,
                                                          uint8_t* __restrict__ out, size_t n) {
    const size_t n8 = n / 8;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += stride) {
        const float4 a = reinterpret_cast<const float4*>(x)[2 * i];
        const float4 b = reinterpret_cast<const float4*>(x)[2 * i + 1];
        const uint32_t w = dt::e2m1x2_from_f32<RELU>(a.x, a.y) |
                           (dt::e2m1x2_from_f32<RELU>(a.z, a.w) << 8) |
                           (dt::e2m1x2_from_f32<RELU>(b.x, b.y) << 16) |
                           (dt::e2m1x2_from_f32<RELU>(b.z, b.w) << 24);
        reinterpret_cast<uint32_t*>(out)[i] = w;
    }
    const size_t pairs_done = n8 * 4;
    const size_t t = pairs_done + static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t < n / 2) out[t] = static_cast<uint8_t>(dt::e2m1x2_from_f32<RELU>(x[2 * t], x[2 * t + 1]));
}

// One group of four f32 -> four codes with stochastic rounding (quad_from_f32_stochastic,
// narrow.rs:217-229): one byte each (FP8, FP6) or one nibble each (E2M1, 16 bits).
template <int OP, bool RELU>
__device__ __forceinline__ uint32_t encode_quad_rs(float x0, float x1, float x2, float x3,
                                                   uint32_t rb) {
    if constexpr (OP == kE4M3) return dt::e4m3x4_from_f32_rs<RELU>(x0, x1, x2, x3, rb);
    else if constexpr (OP == kE5M2) return dt::e5m2x4_from_f32_rs<RELU>(x0, x1, x2, x3, rb);
    else if constexpr (OP == kE2M3) return dt::e2m3x4_from_f32_rs<RELU>(x0, x1, x2, x3, rb);
    else if constexpr (OP == kE3M2) return dt::e3m2x4_from_f32_rs<RELU>(x0, x1, x2, x3, rb);
    else return dt::e2m1x4_from_f32_rs<RELU>(x0, x1, x2, x3, rb);
}

// f32 -> codes with stochastic rounding: group g = elements 4g .. 4g+3 with rbits[g]; one
// 16-byte load and one 4-byte (2-byte for E2M1) store per group. A last group of fewer than four
// is padded with zeros and only its real elements are written (narrow.rs:483-486).
template <int OP, bool RELU>
__global__ void __launch_bounds__(256) encode_rs_kernel(const float* __restrict__ x,
                                                        const uint32_t* __restrict__ rbits,
                                                        uint8_t* __restrict__ out, size_t n) {
    const size_t n4 = n / 4;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (size_t i = tid; i < n4; i += stride) {
        const float4 v = reinterpret_cast<const float4*>(x)[i];
        const uint32_t c = encode_quad_rs<OP, RELU>(v.x, v.y, v.z, v.w, rbits[i]);
        if constexpr (OP == kE2M1) reinterpret_cast<uint16_t*>(out)[i] = static_cast<uint16_t>(c);
        else reinterpret_cast<uint32_t*>(out)[i] = c;
    }
    const size_t rem = n - n4 * 4;
    if (tid == 0 && rem != 0) {
        const size_t b = n4 * 4;
        const float x0 = x[b], x1 = rem > 1 ? x[b + 1] : 0.0f, x2 = rem > 2 ? x[b + 2] : 0.0f;
        const uint32_t c = encode_quad_rs<OP, RELU>(x0, x1, x2, 0.0f, rbits[n4]);
        if constexpr (OP == kE2M1) {
            out[b / 2] = static_cast<uint8_t>(c);  // n is even: the two real elements
        } else {
            for (size_t j = 0; j < rem; ++j) out[b + j] = static_cast<uint8_t>(c >> (8 * j));
        }
    }
}

// f32 -> bf16 / f16 with stochastic rounding: pair p = elements 2p, 2p+1 with rbits[p]; an odd
// last element is converted as a pair with a zero lane.
template <bool BF16, bool RELU, bool SAT>
__global__ void __launch_bounds__(256) encode_x2_rs_kernel(const float* __restrict__ x,
                                                           const uint32_t* __restrict__ rbits,
                                                           uint16_t* __restrict__ out, size_t n) {
    const size_t n2 = n / 2;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    const size_t tid = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (size_t i = tid; i < n2; i += stride) {
        const float2 v = reinterpret_cast<const float2*>(x)[i];
        reinterpret_cast<uint32_t*>(out)[i] =
            BF16 ? dt::bf16x2_from_f32_rs<RELU, SAT>(v.x, v.y, rbits[i])
                 : dt::f16x2_from_f32_rs<RELU, SAT>(v.x, v.y, rbits[i]);
    }
    if (tid == 0 && (n & 1)) {
        const uint32_t c = BF16 ? dt::bf16x2_from_f32_rs<RELU, SAT>(x[n - 1], 0.0f, rbits[n2])
                                : dt::f16x2_from_f32_rs<RELU, SAT>(x[n - 1], 0.0f, rbits[n2]);
        out[n - 1] = static_cast<uint16_t>(c);
    }
}

// f16 -> narrow, one pair per thread step: the f16x2 instruction for FP8 (narrow.rs:164-172);
// FP6 and FP4 through the exact f16 -> f32 widening and the f32 instruction (the same real value,
// so the same round-to-nearest code; their f16x2 forms are not accepted by this ptxas).
template <int OP, bool RELU>
__device__ __forceinline__ uint32_t encode_pair_f16(uint32_t h2) {
    if constexpr (OP == kE4M3) return dt::e4m3x2_from_f16x2<RELU>(h2);
    else if constexpr (OP == kE5M2) return dt::e5m2x2_from_f16x2<RELU>(h2);
    else {
        const float2 f = dt::f16x2_to_f32(h2);
        if constexpr (OP == kE2M1) return dt::e2m1x2_from_f32<RELU>(f.x, f.y);
        else return encode_pair<OP, RELU>(f.x, f.y);
    }
}

template <int OP, bool RELU>
__global__ void __launch_bounds__(256) encode_f16_kernel(const uint16_t* __restrict__ x,
                                                         uint8_t* __restrict__ out, size_t n) {
    const size_t n2 = (n + 1) / 2;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t p = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < n2;
         p += stride) {
        const size_t i = 2 * p;
        const uint32_t h2 = x[i] | (i + 1 < n ? static_cast<uint32_t>(x[i + 1]) << 16 : 0u);
        const uint32_t c = encode_pair_f16<OP, RELU>(h2);
        if constexpr (OP == kE2M1) {
            out[p] = static_cast<uint8_t>(c);  // n even: two nibbles
        } else {
            out[i] = static_cast<uint8_t>(c);
            if (i + 1 < n) out[i + 1] = static_cast<uint8_t>(c >> 8);
        }
    }
}

// narrow -> f16 bits (exact), FMT as decode_kernel.
template <int FMT>
__global__ void __launch_bounds__(256) to_f16_kernel(const uint8_t* __restrict__ c,
                                                     uint16_t* __restrict__ out, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
        const uint32_t b = c[i];
        if constexpr (FMT == 2) {
            const uint32_t h2 = dt::e2m1x2_to_f16x2(b);
            out[2 * i] = static_cast<uint16_t>(h2);
            out[2 * i + 1] = static_cast<uint16_t>(h2 >> 16);
        } else {
            uint32_t h2;
            if constexpr (FMT == 0) h2 = dt::e4m3x2_to_f16x2(static_cast<uint16_t>(b));
            else if constexpr (FMT == 1) h2 = dt::e5m2x2_to_f16x2(static_cast<uint16_t>(b));
            else if constexpr (FMT == 4) h2 = dt::e2m3x2_to_f16x2(static_cast<uint16_t>(b));
            else h2 = dt::e3m2x2_to_f16x2(static_cast<uint16_t>(b));
            out[i] = static_cast<uint16_t>(h2);
        }
    }
}

// bf16::from_f32 with RELU / OVERFLOW (bfloat16.rs:104-118, :446-454), one pair per step.
template <bool RELU, bool SAT>
__global__ void __launch_bounds__(256) f32_to_bf16_kernel(const float* __restrict__ x,
                                                          uint16_t* __restrict__ out, size_t n) {
    const size_t n2 = (n + 1) / 2;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t p = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < n2;
         p += stride) {
        const size_t i = 2 * p;
        const uint32_t r = dt::bf16x2_from_f32_mode<RELU, SAT>(x[i], i + 1 < n ? x[i + 1] : 0.0f);
        out[i] = static_cast<uint16_t>(r);
        if (i + 1 < n) out[i + 1] = static_cast<uint16_t>(r >> 16);
    }
}

// Exact f32 value of one narrow code (FMT as decode_kernel: 0 e4m3, 1 e5m2, 2 e2m1 nibble,
// 4 e2m3, 5 e3m2).
template <int FMT>
__device__ __forceinline__ float narrow_to_f32(uint32_t c) {
    if constexpr (FMT == 0) return dt::e4m3x2_to_f32(static_cast<uint16_t>(c)).x;
    else if constexpr (FMT == 1) return dt::e5m2x2_to_f32(static_cast<uint16_t>(c)).x;
    else if constexpr (FMT == 2) return dt::e2m1x2_to_f32(c).x;
    else if constexpr (FMT == 4) return dt::e2m3x2_to_f32(static_cast<uint16_t>(c)).x;
    else return dt::e3m2x2_to_f32(static_cast<uint16_t>(c)).x;
}

// 2^(s - 127) as an f32 (2^-127 is an f32 subnormal); NaN for the NaN code 0xff.
__device__ __forceinline__ float ue8m0_value(uint32_t s) {
    return s == 0xFFu ? __uint_as_float(0x7FC00000u)
           : s != 0u  ? __uint_as_float(s << 23)
                      : __uint_as_float(0x00400000u);
}

// to_bf16_scaled::<RELU, OVERFLOW> (narrow.rs:314-330, :444-465): element i times the UE8M0 scale
// scales[i / block], rounded once to bf16 (RN; .relu clamps negatives to +0; .satfinite clamps
// overflow to the largest finite bf16). The narrow value has at most 4 significant bits, so the
// f32 product is exact (or infinite past 2^128) and the single cvt.rn...bf16x2.f32 is the only
// rounding, which matters only below 2^-126.
template <int FMT, bool RELU, bool SAT>
__global__ void __launch_bounds__(256) to_bf16_scaled_kernel(const uint8_t* __restrict__ codes,
                                                             const uint8_t* __restrict__ scales,
                                                             uint16_t* __restrict__ out, size_t n,
                                                             size_t block) {
    const size_t n2 = (n + 1) / 2;
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t p = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; p < n2;
         p += stride) {
        const size_t i = 2 * p;
        uint32_t c0, c1 = 0;
        if constexpr (FMT == 2) {
            const uint32_t b = codes[p];
            c0 = b & 0xFu;
            c1 = b >> 4;
        } else {
            c0 = codes[i];
            if (i + 1 < n) c1 = codes[i + 1];
        }
        const float v0 = __fmul_rn(narrow_to_f32<FMT>(c0), ue8m0_value(scales[i / block]));
        const float v1 =
            i + 1 < n ? __fmul_rn(narrow_to_f32<FMT>(c1), ue8m0_value(scales[(i + 1) / block]))
                      : 0.0f;
        const uint32_t r = dt::bf16x2_from_f32_mode<RELU, SAT>(v0, v1);
        out[i] = static_cast<uint16_t>(r);
        if (i + 1 < n) out[i + 1] = static_cast<uint16_t>(r >> 16);
    }
}

template <bool ROUND_UP, bool SAT>
__global__ void __launch_bounds__(256) encode_ue8m0_kernel(const float* __restrict__ x,
                                                           uint8_t* __restrict__ out, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
        out[i] = static_cast<uint8_t>(dt::ue8m0_from_f32<ROUND_UP, SAT>(x[i]));
    }
}

// codes -> f32. Formats: 0 e4m3, 1 e5m2, 2 e2m1x2 (two values per byte), 3 ue8m0, 4 e2m3,
// 5 e3m2 (one FP6 value in the low 6 bits of each byte).
template <int FMT>
__global__ void __launch_bounds__(256) decode_kernel(const uint8_t* __restrict__ c,
                                                     float* __restrict__ out, size_t n) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride) {
        const uint32_t b = c[i];
        if constexpr (FMT == 0) {
            out[i] = dt::e4m3x2_to_f32(static_cast<uint16_t>(b)).x;
        } else if constexpr (FMT == 1) {
            out[i] = dt::e5m2x2_to_f32(static_cast<uint16_t>(b)).x;
        } else if constexpr (FMT == 2) {
            const float2 v = dt::e2m1x2_to_f32(b);
            out[2 * i] = v.x;
            out[2 * i + 1] = v.y;
        } else if constexpr (FMT == 4) {
            out[i] = dt::e2m3x2_to_f32(static_cast<uint16_t>(b)).x;
        } else if constexpr (FMT == 5) {
            out[i] = dt::e3m2x2_to_f32(static_cast<uint16_t>(b)).x;
        } else {
            // Scalar ue8m0 to_f32: the pair with ONE (0x7f) in the other lane (narrow.rs:676-679).
            out[i] = dt::ue8m0x2_to_f32(static_cast<uint16_t>(b | 0x7F00u)).x;
        }
    }
}

// Seed of the sweep's random bits: input pattern p takes group p / 4 (p / 2 for bf16/f16) of
// the SplitMix64 stream below.
constexpr uint64_t kSweepSeed = 0x2545F4914F6CDD1Dull;

// Stochastic-rounding sweep variants 12..29: four inputs base + i .. +3 (i a multiple of 4) ->
// four one-byte codes (12..21: e4m3, e5m2, e2m3, e3m2, e2m1 as nibbles, then the same with
// .relu), or two 32-bit words of bf16/f16 pairs (22..29: bf16 plain, .relu, .satfinite, both;
// then f16), written at out + i or out + 2 i.
__device__ __forceinline__ void sweep_rs(int v, uint64_t p0, float x0, float x1, float x2,
                                         float x3, uint8_t* out, uint64_t i, uint64_t valid) {
    if (v < 22) {
        const uint64_t h = dt::splitmix64(kSweepSeed, p0 >> 3);
        const uint32_t rb = ((p0 >> 2) & 1) ? static_cast<uint32_t>(h >> 32)
                                            : static_cast<uint32_t>(h);
        uint32_t c;
        switch (v) {
        case 12: c = dt::e4m3x4_from_f32_rs<false>(x0, x1, x2, x3, rb); break;
        case 13: c = dt::e5m2x4_from_f32_rs<false>(x0, x1, x2, x3, rb); break;
        case 14: c = dt::e2m3x4_from_f32_rs<false>(x0, x1, x2, x3, rb); break;
        case 15: c = dt::e3m2x4_from_f32_rs<false>(x0, x1, x2, x3, rb); break;
        case 16: c = dt::e2m1x4_from_f32_rs<false>(x0, x1, x2, x3, rb); break;
        case 17: c = dt::e4m3x4_from_f32_rs<true>(x0, x1, x2, x3, rb); break;
        case 18: c = dt::e5m2x4_from_f32_rs<true>(x0, x1, x2, x3, rb); break;
        case 19: c = dt::e2m3x4_from_f32_rs<true>(x0, x1, x2, x3, rb); break;
        case 20: c = dt::e3m2x4_from_f32_rs<true>(x0, x1, x2, x3, rb); break;
        default: c = dt::e2m1x4_from_f32_rs<true>(x0, x1, x2, x3, rb); break;
        }
        if (v == 16 || v == 21)  // nibbles -> one per byte
            c = (c & 0xFu) | ((c & 0xF0u) << 4) | ((c & 0xF00u) << 8) | ((c & 0xF000u) << 12);
        if (valid == 4) {
            *reinterpret_cast<uint32_t*>(out + i) = c;
        } else {
            for (uint64_t j = 0; j < valid; ++j) out[i + j] = static_cast<uint8_t>(c >> (8 * j));
        }
        return;
    }
    if (v >= 30) {  // bf16 round-to-nearest: plain, .relu, .satfinite, both
        uint32_t c0, c1;
        switch (v) {
        case 30: c0 = dt::bf16x2_from_f32_mode<false, false>(x0, x1); c1 = dt::bf16x2_from_f32_mode<false, false>(x2, x3); break;
        case 31: c0 = dt::bf16x2_from_f32_mode<true, false>(x0, x1); c1 = dt::bf16x2_from_f32_mode<true, false>(x2, x3); break;
        case 32: c0 = dt::bf16x2_from_f32_mode<false, true>(x0, x1); c1 = dt::bf16x2_from_f32_mode<false, true>(x2, x3); break;
        default: c0 = dt::bf16x2_from_f32_mode<true, true>(x0, x1); c1 = dt::bf16x2_from_f32_mode<true, true>(x2, x3); break;
        }
        uint16_t* o = reinterpret_cast<uint16_t*>(out) + i;
        const uint16_t codes[4] = {static_cast<uint16_t>(c0), static_cast<uint16_t>(c0 >> 16),
                                   static_cast<uint16_t>(c1), static_cast<uint16_t>(c1 >> 16)};
        if (valid == 4) {
            reinterpret_cast<uint32_t*>(o)[0] = c0;
            reinterpret_cast<uint32_t*>(o)[1] = c1;
        } else {
            for (uint64_t j = 0; j < valid; ++j) o[j] = codes[j];
        }
        return;
    }
    // pairs (p0, p0 + 1) and (p0 + 2, p0 + 3): groups p0 / 2 (even) and p0 / 2 + 1
    const uint64_t h = dt::splitmix64(kSweepSeed, p0 >> 2);
    const uint32_t r0 = static_cast<uint32_t>(h), r1 = static_cast<uint32_t>(h >> 32);
    uint32_t c0, c1;
    switch (v) {
    case 22: c0 = dt::bf16x2_from_f32_rs<false, false>(x0, x1, r0); c1 = dt::bf16x2_from_f32_rs<false, false>(x2, x3, r1); break;
    case 23: c0 = dt::bf16x2_from_f32_rs<true, false>(x0, x1, r0); c1 = dt::bf16x2_from_f32_rs<true, false>(x2, x3, r1); break;
    case 24: c0 = dt::bf16x2_from_f32_rs<false, true>(x0, x1, r0); c1 = dt::bf16x2_from_f32_rs<false, true>(x2, x3, r1); break;
    case 25: c0 = dt::bf16x2_from_f32_rs<true, true>(x0, x1, r0); c1 = dt::bf16x2_from_f32_rs<true, true>(x2, x3, r1); break;
    case 26: c0 = dt::f16x2_from_f32_rs<false, false>(x0, x1, r0); c1 = dt::f16x2_from_f32_rs<false, false>(x2, x3, r1); break;
    case 27: c0 = dt::f16x2_from_f32_rs<true, false>(x0, x1, r0); c1 = dt::f16x2_from_f32_rs<true, false>(x2, x3, r1); break;
    case 28: c0 = dt::f16x2_from_f32_rs<false, true>(x0, x1, r0); c1 = dt::f16x2_from_f32_rs<false, true>(x2, x3, r1); break;
    default: c0 = dt::f16x2_from_f32_rs<true, true>(x0, x1, r0); c1 = dt::f16x2_from_f32_rs<true, true>(x2, x3, r1); break;
    }
    uint16_t* o = reinterpret_cast<uint16_t*>(out) + i;
    const uint16_t codes[4] = {static_cast<uint16_t>(c0), static_cast<uint16_t>(c0 >> 16),
                               static_cast<uint16_t>(c1), static_cast<uint16_t>(c1 >> 16)};
    if (valid == 4) {
        reinterpret_cast<uint32_t*>(o)[0] = c0;
        reinterpret_cast<uint32_t*>(o)[1] = c1;
    } else {
        for (uint64_t j = 0; j < valid; ++j) o[j] = codes[j];
    }
}

// Converts the f32 bit patterns base + i, i < n, with variant v; one output byte per input
// (two for variants 22..29).
__global__ void __launch_bounds__(256) sweep_kernel(int v, uint64_t base, uint64_t n,
                                                    uint8_t* __restrict__ out) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n;
         i += stride * 4) {
        if (v >= 12) {
            const uint64_t p = base + i;
            const uint64_t valid = n - i < 4 ? n - i : 4;
            const float x0 = __uint_as_float(static_cast<uint32_t>(p));
            const float x1 = valid > 1 ? __uint_as_float(static_cast<uint32_t>(p + 1)) : 0.0f;
            const float x2 = valid > 2 ? __uint_as_float(static_cast<uint32_t>(p + 2)) : 0.0f;
            const float x3 = valid > 3 ? __uint_as_float(static_cast<uint32_t>(p + 3)) : 0.0f;
            sweep_rs(v, p, x0, x1, x2, x3, out, i, valid);
            continue;
        }
        uint32_t codes = 0;
        for (int j = 0; j < 4; ++j) {
            const float f = __uint_as_float(static_cast<uint32_t>(base + i + j));
            uint32_t c;
            switch (v) {
            case 0: c = dt::e4m3x2_from_f32<false>(f, 0.0f) & 0xFFu; break;
            case 1: c = dt::e5m2x2_from_f32<false>(f, 0.0f) & 0xFFu; break;
            case 2: c = dt::e2m1x2_from_f32<false>(f, 0.0f) & 0xFu; break;
            case 3: c = dt::e4m3x2_from_f32<true>(f, 0.0f) & 0xFFu; break;
            case 4: c = dt::e5m2x2_from_f32<true>(f, 0.0f) & 0xFFu; break;
            case 5: c = dt::e2m1x2_from_f32<true>(f, 0.0f) & 0xFu; break;
            case 6: c = dt::ue8m0_from_f32<false, true>(f); break;
            case 7: c = dt::ue8m0_from_f32<true, true>(f); break;
            case 8: c = dt::e2m3x2_from_f32<false>(f, 0.0f) & 0xFFu; break;
            case 9: c = dt::e3m2x2_from_f32<false>(f, 0.0f) & 0xFFu; break;
            case 10: c = dt::e2m3x2_from_f32<true>(f, 0.0f) & 0xFFu; break;
            default: c = dt::e3m2x2_from_f32<true>(f, 0.0f) & 0xFFu; break;
            }
            codes |= c << (8 * j);
        }
        if (i + 4 <= n) {
            *reinterpret_cast<uint32_t*>(out + i) = codes;
        } else {
            for (uint64_t j = 0; i + j < n; ++j) out[i + j] = static_cast<uint8_t>(codes >> (8 * j));
        }
    }
}

int grid_for(size_t work) {
    const size_t blocks = (work + 255) / 256;
    const size_t cap = static_cast<size_t>(ptxstd::sm_count()) * 8;
    return static_cast<int>(blocks == 0 ? 1 : (blocks < cap ? blocks : cap));
}

template <typename F>
int launch(F f) {
    f();
    return ptxstd::launch_status();
}

template <int FMT>
int launch_scaled(const uint8_t* d_codes, const uint8_t* d_scales, uint16_t* d_out, size_t n,
                  size_t block, int relu, int satfinite, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_scales || !d_out || block == 0 || (FMT == 2 && (n & 1)))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu && satfinite)
            to_bf16_scaled_kernel<FMT, true, true><<<g, 256, 0, s>>>(d_codes, d_scales, d_out, n, block);
        else if (relu)
            to_bf16_scaled_kernel<FMT, true, false><<<g, 256, 0, s>>>(d_codes, d_scales, d_out, n, block);
        else if (satfinite)
            to_bf16_scaled_kernel<FMT, false, true><<<g, 256, 0, s>>>(d_codes, d_scales, d_out, n, block);
        else
            to_bf16_scaled_kernel<FMT, false, false><<<g, 256, 0, s>>>(d_codes, d_scales, d_out, n, block);
    });
}

template <int OP>
int launch_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out, size_t n, int relu,
              ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    const uintptr_t out_align = OP == kE2M1 ? 1 : 3;
    if (!d_x || !d_rbits || !d_out || !ptxstd::aligned16(d_x) ||
        (reinterpret_cast<uintptr_t>(d_rbits) & 3) ||
        (reinterpret_cast<uintptr_t>(d_out) & out_align))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 4 + 1);
    return launch([&] {
        if (relu) encode_rs_kernel<OP, true><<<g, 256, 0, s>>>(d_x, d_rbits, d_out, n);
        else encode_rs_kernel<OP, false><<<g, 256, 0, s>>>(d_x, d_rbits, d_out, n);
    });
}

template <bool BF16>
int launch_x2_rs(const float* d_x, const uint32_t* d_rbits, uint16_t* d_out, size_t n, int relu,
                 int satfinite, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_rbits || !d_out || (reinterpret_cast<uintptr_t>(d_x) & 7) ||
        (reinterpret_cast<uintptr_t>(d_rbits) & 3) || (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 2 + 1);
    return launch([&] {
        if (relu && satfinite)
            encode_x2_rs_kernel<BF16, true, true><<<g, 256, 0, s>>>(d_x, d_rbits, d_out, n);
        else if (relu)
            encode_x2_rs_kernel<BF16, true, false><<<g, 256, 0, s>>>(d_x, d_rbits, d_out, n);
        else if (satfinite)
            encode_x2_rs_kernel<BF16, false, true><<<g, 256, 0, s>>>(d_x, d_rbits, d_out, n);
        else
            encode_x2_rs_kernel<BF16, false, false><<<g, 256, 0, s>>>(d_x, d_rbits, d_out, n);
    });
}

}  // namespace

extern "C" {

int ptxstd_cvt_f32_to_e4m3(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out || !ptxstd::aligned16(d_x) || (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 4 + 1);
    return launch([&] {
        if (relu) encode_fp8_kernel<kE4M3, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_fp8_kernel<kE4M3, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_f32_to_e5m2(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out || !ptxstd::aligned16(d_x) || (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 4 + 1);
    return launch([&] {
        if (relu) encode_fp8_kernel<kE5M2, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_fp8_kernel<kE5M2, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_f32_to_e2m1x2(const float* d_x, uint8_t* d_out, size_t n, int relu,
                             ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out || (n & 1) || !ptxstd::aligned16(d_x) ||
        (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 8 + 4);
    return launch([&] {
        if (relu) encode_e2m1_kernel<true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_e2m1_kernel<false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_f32_to_ue8m0(const float* d_x, uint8_t* d_out, size_t n, int round_up,
                            int satfinite, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n);
    return launch([&] {
        if (round_up && satfinite) encode_ue8m0_kernel<true, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else if (round_up) encode_ue8m0_kernel<true, false><<<g, 256, 0, s>>>(d_x, d_out, n);
        else if (satfinite) encode_ue8m0_kernel<false, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_ue8m0_kernel<false, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_f32_to_e2m3(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out || !ptxstd::aligned16(d_x) || (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 4 + 1);
    return launch([&] {
        if (relu) encode_fp8_kernel<kE2M3, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_fp8_kernel<kE2M3, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_f32_to_e3m2(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out || !ptxstd::aligned16(d_x) || (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n / 4 + 1);
    return launch([&] {
        if (relu) encode_fp8_kernel<kE3M2, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_fp8_kernel<kE3M2, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_e2m3_to_f32(const uint8_t* d_codes, float* d_out, size_t n,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { decode_kernel<4><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}

int ptxstd_cvt_e3m2_to_f32(const uint8_t* d_codes, float* d_out, size_t n,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { decode_kernel<5><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}

int ptxstd_cvt_e4m3_to_f32(const uint8_t* d_codes, float* d_out, size_t n,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { decode_kernel<0><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}

int ptxstd_cvt_e5m2_to_f32(const uint8_t* d_codes, float* d_out, size_t n,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { decode_kernel<1><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}

int ptxstd_cvt_e2m1x2_to_f32(const uint8_t* d_codes, float* d_out, size_t n_bytes,
                             ptxstd_stream stream) {
    if (n_bytes == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch(
        [&] { decode_kernel<2><<<grid_for(n_bytes), 256, 0, s>>>(d_codes, d_out, n_bytes); });
}

int ptxstd_cvt_ue8m0_to_f32(const uint8_t* d_codes, float* d_out, size_t n,
                            ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { decode_kernel<3><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}

int ptxstd_cvt_f32_to_e4m3_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out, size_t n,
                              int relu, ptxstd_stream stream) {
    return launch_rs<kE4M3>(d_x, d_rbits, d_out, n, relu, stream);
}
int ptxstd_cvt_f32_to_e5m2_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out, size_t n,
                              int relu, ptxstd_stream stream) {
    return launch_rs<kE5M2>(d_x, d_rbits, d_out, n, relu, stream);
}
int ptxstd_cvt_f32_to_e2m3_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out, size_t n,
                              int relu, ptxstd_stream stream) {
    return launch_rs<kE2M3>(d_x, d_rbits, d_out, n, relu, stream);
}
int ptxstd_cvt_f32_to_e3m2_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out, size_t n,
                              int relu, ptxstd_stream stream) {
    return launch_rs<kE3M2>(d_x, d_rbits, d_out, n, relu, stream);
}
int ptxstd_cvt_f32_to_e2m1x2_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out,
                                size_t n, int relu, ptxstd_stream stream) {
    if (n & 1) return PTXSTD_EINVAL;
    return launch_rs<kE2M1>(d_x, d_rbits, d_out, n, relu, stream);
}
int ptxstd_cvt_f32_to_bf16_rs(const float* d_x, const uint32_t* d_rbits, uint16_t* d_out,
                              size_t n, int relu, int satfinite, ptxstd_stream stream) {
    return launch_x2_rs<true>(d_x, d_rbits, d_out, n, relu, satfinite, stream);
}
int ptxstd_cvt_f32_to_f16_rs(const float* d_x, const uint32_t* d_rbits, uint16_t* d_out,
                             size_t n, int relu, int satfinite, ptxstd_stream stream) {
    return launch_x2_rs<false>(d_x, d_rbits, d_out, n, relu, satfinite, stream);
}

int ptxstd_cvt_f16_to_e4m3(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu) encode_f16_kernel<kE4M3, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_f16_kernel<kE4M3, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}
int ptxstd_cvt_f16_to_e5m2(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu) encode_f16_kernel<kE5M2, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_f16_kernel<kE5M2, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}
int ptxstd_cvt_f16_to_e2m1x2(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out || (n & 1)) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu) encode_f16_kernel<kE2M1, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_f16_kernel<kE2M1, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}
int ptxstd_cvt_f16_to_e2m3(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu) encode_f16_kernel<kE2M3, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_f16_kernel<kE2M3, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}
int ptxstd_cvt_f16_to_e3m2(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu) encode_f16_kernel<kE3M2, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else encode_f16_kernel<kE3M2, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}
int ptxstd_cvt_e4m3_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { to_f16_kernel<0><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}
int ptxstd_cvt_e5m2_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { to_f16_kernel<1><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}
int ptxstd_cvt_e2m1x2_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { to_f16_kernel<2><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}
int ptxstd_cvt_e2m3_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { to_f16_kernel<4><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}
int ptxstd_cvt_e3m2_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_codes || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { to_f16_kernel<5><<<grid_for(n), 256, 0, s>>>(d_codes, d_out, n); });
}
int ptxstd_cvt_f32_to_bf16(const float* d_x, uint16_t* d_out, size_t n, int relu, int satfinite,
                           ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_x || !d_out) return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for((n + 1) / 2);
    return launch([&] {
        if (relu && satfinite) f32_to_bf16_kernel<true, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else if (relu) f32_to_bf16_kernel<true, false><<<g, 256, 0, s>>>(d_x, d_out, n);
        else if (satfinite) f32_to_bf16_kernel<false, true><<<g, 256, 0, s>>>(d_x, d_out, n);
        else f32_to_bf16_kernel<false, false><<<g, 256, 0, s>>>(d_x, d_out, n);
    });
}

int ptxstd_cvt_e4m3_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream) {
    return launch_scaled<0>(d_codes, d_scales, d_out, n, block, relu, satfinite, stream);
}
int ptxstd_cvt_e5m2_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream) {
    return launch_scaled<1>(d_codes, d_scales, d_out, n, block, relu, satfinite, stream);
}
int ptxstd_cvt_e2m1x2_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                     uint16_t* d_out, size_t n, size_t block, int relu,
                                     int satfinite, ptxstd_stream stream) {
    return launch_scaled<2>(d_codes, d_scales, d_out, n, block, relu, satfinite, stream);
}
int ptxstd_cvt_e2m3_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream) {
    return launch_scaled<4>(d_codes, d_scales, d_out, n, block, relu, satfinite, stream);
}
int ptxstd_cvt_e3m2_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream) {
    return launch_scaled<5>(d_codes, d_scales, d_out, n, block, relu, satfinite, stream);
}

int ptxstd_cvt_sweep(int variant, uint64_t base, uint64_t n, uint8_t* d_out,
                     ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_out || variant < 0 || variant > 33 || base + n > (1ull << 32) ||
        (reinterpret_cast<uintptr_t>(d_out) & 3) || (variant >= 12 && (base & 3)))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { sweep_kernel<<<grid_for(n / 4 + 1), 256, 0, s>>>(variant, base, n, d_out); });
}

}  // extern "C"

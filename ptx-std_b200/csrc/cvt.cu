// Element-wise conversion kernels of the narrow formats (the reference's Vector<E, N>::from_f32 /
// to_f32 family, src/data_types/narrow.rs:354-425, applied over device arrays), plus the
// exhaustive-sweep kernel that converts f32 bit patterns generated from the thread index.
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

// Converts the f32 bit patterns base + i, i < n, with variant v; one output byte per input.
__global__ void __launch_bounds__(256) sweep_kernel(int v, uint64_t base, uint64_t n,
                                                    uint8_t* __restrict__ out) {
    const uint64_t stride = static_cast<uint64_t>(gridDim.x) * blockDim.x;
    for (uint64_t i = (static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; i < n;
         i += stride * 4) {
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

int ptxstd_cvt_sweep(int variant, uint64_t base, uint64_t n, uint8_t* d_out,
                     ptxstd_stream stream) {
    if (n == 0) return PTXSTD_OK;
    if (!d_out || variant < 0 || variant > 11 || base + n > (1ull << 32) ||
        (reinterpret_cast<uintptr_t>(d_out) & 3))
        return PTXSTD_EINVAL;
    auto s = static_cast<cudaStream_t>(stream);
    return launch([&] { sweep_kernel<<<grid_for(n / 4 + 1), 256, 0, s>>>(variant, base, n, d_out); });
}

}  // extern "C"

// Quantise/pack kernels: bf16 activations -> MXFP8 (E4M3 + UE8M0 per 32) and NVFP4 (E2M1 + E4M3
// per 16, f32 global scale). HBM-bound: each thread streams 16-byte vectors (8 bf16) with
// non-allocating loads, four vectors in flight per thread; the lanes holding one block combine
// their amax with shuffle-xor, and every element pair is packed by one `cvt` instruction
// (ptx-std src/data_types/narrow.rs:156-162). Outputs are written as whole 8-byte (MXFP8) or
// 4-byte (NVFP4) words per lane, so each warp store covers a contiguous 256 / 128 bytes.
#include "common.cuh"
#include "data_types.cuh"

namespace dt = ptxstd::data_types;

namespace {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;  // 16-byte vectors in flight per thread

// Offset of scale (r, s) in the blocked "128x4" layout consumed by the block-scaled GEMMs: tiles
// of 128 rows x 4 scale columns stored as 512 contiguous bytes, row-tile major; inside a tile the
// scale of row r, column s sits at (r % 32) * 16 + ((r / 32) % 4) * 4 + s % 4, which is the
// 32-lane x 16-byte source of one tcgen05.cp.32x128b.warpx4 (src/tcgen05/copy.rs:29-30).
__device__ __forceinline__ size_t blocked_sf_offset(size_t r, size_t s, size_t sf_cols) {
    const size_t tile = (r >> 7) * (sf_cols >> 2) + (s >> 2);
    return tile * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (s & 3);
}

// One MXFP8 block is 32 bf16 = 4 vectors = 4 consecutive lanes. Vector v of the flat tensor
// covers elements 8v .. 8v+7; block b = v / 4.
template <bool BLOCKED>
__global__ void __launch_bounds__(kThreads) quantize_mxfp8_kernel(
    const uint4* __restrict__ x, size_t n_vec, uint2* __restrict__ q, uint8_t* __restrict__ sf,
    size_t sf_cols) {
    const uint32_t lane = threadIdx.x & 31u;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const size_t n_warps = (static_cast<size_t>(gridDim.x) * kThreads) >> 5;
    const size_t chunk = 32 * kUnroll;  // vectors per warp step
    for (size_t base = warp * chunk; base < n_vec; base += n_warps * chunk) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t i = base + 32 * u + lane;
            v[u] = i < n_vec ? ptxstd::ld_stream_v4(x + i) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t i = base + 32 * u + lane;
            uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v[u].x, v[u].y),
                                                  dt::bf16x2_absmax_bits(v[u].z, v[u].w)));
            m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
            m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
            const float amax = __uint_as_float(m << 16);
            const uint32_t code = dt::mxfp8_scale_code(amax);
            const float inv = dt::ue8m0_inverse(code);
            const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
            uint32_t p[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                p[k] = dt::e4m3x2_from_f32<false>(__fmul_rn(dt::bf16_lo(w[k]), inv),
                                                  __fmul_rn(dt::bf16_hi(w[k]), inv));
            if (i < n_vec) {
                q[i] = make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
                if ((lane & 3u) == 0) {
                    const size_t b = i >> 2;
                    if constexpr (BLOCKED) {
                        sf[blocked_sf_offset(b / sf_cols, b % sf_cols, sf_cols)] =
                            static_cast<uint8_t>(code);
                    } else {
                        sf[b] = static_cast<uint8_t>(code);
                    }
                }
            }
        }
    }
}

// One NVFP4 block is 16 bf16 = 2 vectors = 2 consecutive lanes.
template <bool BLOCKED>
__global__ void __launch_bounds__(kThreads) quantize_nvfp4_kernel(
    const uint4* __restrict__ x, size_t n_vec, float g, uint32_t* __restrict__ q,
    uint8_t* __restrict__ sf, size_t sf_cols) {
    const uint32_t lane = threadIdx.x & 31u;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
    const size_t n_warps = (static_cast<size_t>(gridDim.x) * kThreads) >> 5;
    const size_t chunk = 32 * kUnroll;
    const float six_g = __fmul_rn(6.0f, g);
    for (size_t base = warp * chunk; base < n_vec; base += n_warps * chunk) {
        uint4 v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t i = base + 32 * u + lane;
            v[u] = i < n_vec ? ptxstd::ld_stream_v4(x + i) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const size_t i = base + 32 * u + lane;
            uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v[u].x, v[u].y),
                                                  dt::bf16x2_absmax_bits(v[u].z, v[u].w)));
            m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
            const float amax = __uint_as_float(m << 16);
            // sf = e4m3(amax / (6 g)); r = 1 / (sf * g), or 0 when that product is 0.
            const float s = __fdiv_rn(amax, six_g);
            const uint32_t code = dt::e4m3x2_from_f32<false>(s, 0.0f) & 0xFFu;
            const float t = __fmul_rn(dt::e4m3_to_f32(code), g);
            const float r = (t == 0.0f) ? 0.0f : __frcp_rn(t);
            const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
            uint32_t packed = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k)
                packed |= dt::e2m1x2_from_f32<false>(__fmul_rn(dt::bf16_lo(w[k]), r),
                                                     __fmul_rn(dt::bf16_hi(w[k]), r))
                          << (8 * k);
            if (i < n_vec) {
                q[i] = packed;
                if ((lane & 1u) == 0) {
                    const size_t b = i >> 1;
                    if constexpr (BLOCKED) {
                        sf[blocked_sf_offset(b / sf_cols, b % sf_cols, sf_cols)] =
                            static_cast<uint8_t>(code);
                    } else {
                        sf[b] = static_cast<uint8_t>(code);
                    }
                }
            }
        }
    }
}

int grid_for(size_t n_vec) {
    const size_t per_block = static_cast<size_t>(kThreads) * kUnroll;
    const size_t need = (n_vec + per_block - 1) / per_block;
    const size_t cap = static_cast<size_t>(ptxstd::sm_count()) * (2048 / kThreads);
    return static_cast<int>(need == 0 ? 1 : (need < cap ? need : cap));
}

}  // namespace

extern "C" {

int ptxstd_quantize_mxfp8_layout(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                                 uint8_t* d_sf, int sf_layout, ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 32 != 0) return PTXSTD_EINVAL;
    if (!d_x || !d_q || !d_sf || !ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_q))
        return PTXSTD_EINVAL;
    if (sf_layout != 0 && sf_layout != 1) return PTXSTD_EINVAL;
    if (sf_layout == 1 && (rows % 128 != 0 || cols % 128 != 0)) return PTXSTD_EINVAL;
    const size_t n_vec = static_cast<size_t>(rows) * static_cast<size_t>(cols) / 8;
    const size_t sf_cols = static_cast<size_t>(cols) / 32;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n_vec);
    if (sf_layout == 1)
        quantize_mxfp8_kernel<true><<<g, kThreads, 0, s>>>(reinterpret_cast<const uint4*>(d_x),
                                                          n_vec, reinterpret_cast<uint2*>(d_q),
                                                          d_sf, sf_cols);
    else
        quantize_mxfp8_kernel<false><<<g, kThreads, 0, s>>>(reinterpret_cast<const uint4*>(d_x),
                                                           n_vec, reinterpret_cast<uint2*>(d_q),
                                                           d_sf, sf_cols);
    return ptxstd::launch_status();
}

int ptxstd_quantize_mxfp8(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                          uint8_t* d_sf, ptxstd_stream stream) {
    return ptxstd_quantize_mxfp8_layout(d_x, rows, cols, d_q, d_sf, 0, stream);
}

int ptxstd_quantize_nvfp4_layout(const uint16_t* d_x, int64_t rows, int64_t cols,
                                 float global_scale, uint8_t* d_q, uint8_t* d_sf, int sf_layout,
                                 ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 16 != 0) return PTXSTD_EINVAL;
    if (!(global_scale > 0.0f) || global_scale == __builtin_huge_valf()) return PTXSTD_EINVAL;
    if (!d_x || !d_q || !d_sf || !ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_q))
        return PTXSTD_EINVAL;
    if (sf_layout != 0 && sf_layout != 1) return PTXSTD_EINVAL;
    if (sf_layout == 1 && (rows % 128 != 0 || cols % 64 != 0)) return PTXSTD_EINVAL;
    const size_t n_vec = static_cast<size_t>(rows) * static_cast<size_t>(cols) / 8;
    const size_t sf_cols = static_cast<size_t>(cols) / 16;
    auto s = static_cast<cudaStream_t>(stream);
    const int g = grid_for(n_vec);
    if (sf_layout == 1)
        quantize_nvfp4_kernel<true><<<g, kThreads, 0, s>>>(
            reinterpret_cast<const uint4*>(d_x), n_vec, global_scale,
            reinterpret_cast<uint32_t*>(d_q), d_sf, sf_cols);
    else
        quantize_nvfp4_kernel<false><<<g, kThreads, 0, s>>>(
            reinterpret_cast<const uint4*>(d_x), n_vec, global_scale,
            reinterpret_cast<uint32_t*>(d_q), d_sf, sf_cols);
    return ptxstd::launch_status();
}

int ptxstd_quantize_nvfp4(const uint16_t* d_x, int64_t rows, int64_t cols, float global_scale,
                          uint8_t* d_q, uint8_t* d_sf, ptxstd_stream stream) {
    return ptxstd_quantize_nvfp4_layout(d_x, rows, cols, global_scale, d_q, d_sf, 0, stream);
}

}  // extern "C"

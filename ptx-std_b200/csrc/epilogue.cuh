// GEMM epilogue stores through the tensor memory accelerator: the bf16 output of one epilogue
// warp (32 rows, one per lane) is written into a swizzled shared-memory staging buffer and leaves
// with a TMA tile store (tma_store_tile::<2>, src/tma/tensor.rs:746), tracked by the bulk
// async-group (bulk_commit_group / bulk_wait_group, src/tma/mod.rs:204-220).
//
// Why: with direct stores each warp instruction writes 16 bytes into 32 different rows, so every
// row segment reaches L2 as a separate half-sector request. On 256 x 256 tiles every CTA of the
// GPU issues those requests in the same few microseconds (the tiles finish in step), and the
// burst delays the next tile's operand loads. A TMA store moves whole row segments of 32, 64 or
// 128 bytes, is asynchronous, and keeps the epilogue warps' instruction count low.
//
// Staging layout: 32 rows x (2 COLS) bytes per buffer, 1024-byte aligned, written with the
// tensor map's swizzle of the same width (CU_TENSOR_MAP_SWIZZLE_{32,64,128}B): the 16-byte chunk
// c of row r sits at chunk position c ^ ((r * 2 COLS / 128) mod (2 COLS / 16)). Eight
// consecutive lanes then hit eight different 16-byte bank groups, so the lanes' 16-byte shared
// stores are conflict-free. The tensor map over C: bf16 [M, N] row-major, box COLS x 32.
#pragma once

#include "common.cuh"
#include "data_types.cuh"
#include "tma_host.h"

namespace ptxstd {
namespace epi {

constexpr uint32_t kRows = 32;  // rows per staging buffer (a warp's lanes)

template <uint32_t COLS>
struct Box {
    static_assert(COLS == 16 || COLS == 32 || COLS == 64, "16, 32 or 64 bf16 columns");
    static constexpr uint32_t kRowBytes = 2 * COLS;        // = the swizzle width
    static constexpr uint32_t kChunks = kRowBytes / 16;    // 16-byte chunks per row
    static constexpr uint32_t kBytes = kRows * kRowBytes;  // staging bytes per buffer
    static constexpr uint32_t kRowShift = COLS == 64 ? 0 : (COLS == 32 ? 1 : 2);
    __device__ static uint32_t offset(uint32_t r, uint32_t c) {
        return r * kRowBytes + ((c ^ ((r >> kRowShift) & (kChunks - 1))) << 4);
    }
};

// Host side: the store map over C (bf16 [M, N] row-major) matching Box<COLS>.
template <uint32_t COLS>
inline int make_store_map(CUtensorMap* map, void* c, uint64_t M, uint64_t N) {
    const CUtensorMapSwizzle sw = COLS == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : COLS == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                                               : CU_TENSOR_MAP_SWIZZLE_32B;
    return make_tmap_2d(map, c, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, N, M, N * 2, COLS, kRows, sw);
}

// Waits (lane 0) until at most PENDING of the TMA stores this warp issued are still reading
// their staging buffers, then syncs the warp. PENDING = 0: every buffer may be rewritten;
// PENDING = 1 with two buffers used in turn: the buffer of the store before last may be.
template <int PENDING = 0>
__device__ __forceinline__ void wait_staging(uint32_t lane) {
    if (lane == 0) bulk_wait_group_read<PENDING>();
    __syncwarp();
}

// Waits (lane 0) until every TMA store this warp issued has completed (before the CTA exits).
__device__ __forceinline__ void drain(uint32_t lane) {
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
}

// Stores accumulator columns [FIRST, FIRST + COLS) of this lane's row (r: fp32 bit patterns),
// times alpha, as bf16 to C at (column col0, row row0 + lane) through the staging buffer `stg`
// (.shared::cta address, 1024-byte aligned, Box<COLS>::kBytes), whose previous store must have
// finished reading it (wait_staging).
template <uint32_t COLS, uint32_t FIRST, uint32_t N>
__device__ __forceinline__ void stage_store(const CUtensorMap* map, uint32_t stg,
                                            const uint32_t (&r)[N], float alpha, int32_t col0,
                                            int32_t row0, uint32_t lane) {
    using B = Box<COLS>;
    static_assert(FIRST + COLS <= N, "columns out of range");
#pragma unroll
    for (uint32_t c = 0; c < B::kChunks; ++c) {
        uint32_t p[4];
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t i = FIRST + 8 * c + 2 * k;
            p[k] = data_types::bf16x2_from_f32(__uint_as_float(r[i]) * alpha,
                                               __uint_as_float(r[i + 1]) * alpha);
        }
        st_shared_v4(stg + B::offset(lane, c), p[0], p[1], p[2], p[3]);
    }
    fence_proxy_async_smem();  // this lane's generic-proxy writes, visible to the TMA unit
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, stg, col0, row0);
        bulk_commit_group();
    }
}

// Stores all N columns of this lane's accumulator row, COLS at a time, through one staging buffer
// (each store waits until the previous one has finished reading it).
template <uint32_t COLS, uint32_t J = 0, uint32_t N>
__device__ __forceinline__ void store_row_block(const CUtensorMap* map, uint32_t stg,
                                                const uint32_t (&r)[N], float alpha,
                                                int32_t col0, int32_t row0, uint32_t lane) {
    if constexpr (J * COLS < N) {
        wait_staging(lane);
        stage_store<COLS, J * COLS>(map, stg, r, alpha, col0 + static_cast<int32_t>(J * COLS),
                                    row0, lane);
        store_row_block<COLS, J + 1>(map, stg, r, alpha, col0, row0, lane);
    }
}

}  // namespace epi
}  // namespace ptxstd

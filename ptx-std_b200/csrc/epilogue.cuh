// GEMM epilogue stores through the tensor memory accelerator: the bf16 output of one epilogue
// warp (32 rows, one per lane) is written into a 128-byte-swizzled shared-memory staging buffer
// and leaves with a TMA tile store (tma_store_tile::<2>, src/tma/tensor.rs:746), tracked by the
// bulk async-group (bulk_commit_group / bulk_wait_group, src/tma/mod.rs:204-220).
//
// Why: with direct stores each warp instruction writes 16 bytes into 32 different rows, so every
// row segment reaches L2 as a separate half-sector request. On a 256 x 256 tile every CTA of the
// GPU issues those requests in the same few microseconds (the tiles finish in step), and the
// burst delays the next tile's operand loads. A TMA store moves whole 128-byte row segments, is
// asynchronous, and keeps the epilogue warps' instruction count low.
//
// Staging layout: 32 rows x 128 bytes (64 bf16 columns) per buffer, 1024-byte aligned; the 16-byte
// chunk c of row r sits at chunk position c ^ (r % 8), which is the tensor map's
// CU_TENSOR_MAP_SWIZZLE_128B pattern and makes the lanes' 16-byte shared stores conflict-free.
// The tensor map over C: bf16 [M, N] row-major, box 64 columns x 32 rows, 128-byte swizzle.
#pragma once

#include "common.cuh"
#include "data_types.cuh"

namespace ptxstd {
namespace epi {

constexpr uint32_t kRows = 32;                       // rows per staging buffer (a warp's lanes)
constexpr uint32_t kCols = 64;                       // bf16 columns per staging buffer
constexpr uint32_t kStageBytes = kRows * kCols * 2;  // 4 KiB

// Waits (lane 0) until the TMA stores this warp issued have finished reading their staging
// buffers, then syncs the warp: after it the buffers may be rewritten.
__device__ __forceinline__ void wait_staging(uint32_t lane) {
    if (lane == 0) bulk_wait_group_read<0>();
    __syncwarp();
}

// Waits (lane 0) until every TMA store this warp issued has completed (before the CTA exits).
__device__ __forceinline__ void drain(uint32_t lane) {
    if (lane == 0) bulk_wait_group<0>();
    __syncwarp();
}

// Stores columns [J * 64, J * 64 + 64) of this lane's accumulator row (r: fp32 bit patterns),
// times alpha, as bf16 to C at (column col0, row row0 + lane) through the staging buffer `stg`
// (.shared::cta address, 1024-byte aligned, kStageBytes bytes), whose previous store must have
// finished reading it (wait_staging).
template <uint32_t J, uint32_t N>
__device__ __forceinline__ void stage_store(const CUtensorMap* map, uint32_t stg,
                                            const uint32_t (&r)[N], float alpha, int32_t col0,
                                            int32_t row0, uint32_t lane) {
    static_assert((J + 1) * kCols <= N, "columns out of range");
#pragma unroll
    for (uint32_t c = 0; c < 8; ++c) {
        uint32_t p[4];
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
            const uint32_t i = J * kCols + 8 * c + 2 * k;
            p[k] = data_types::bf16x2_from_f32(__uint_as_float(r[i]) * alpha,
                                               __uint_as_float(r[i + 1]) * alpha);
        }
        st_shared_v4(stg + lane * 128 + ((c ^ (lane & 7u)) << 4), p[0], p[1], p[2], p[3]);
    }
    fence_proxy_async_smem();  // this lane's generic-proxy writes, visible to the TMA unit
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(map, stg, col0, row0);
        bulk_commit_group();
    }
}

}  // namespace epi
}  // namespace ptxstd

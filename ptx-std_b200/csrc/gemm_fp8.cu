// FP8 E4M3 x E4M3 GEMM on the 5th-generation tensor cores:
//   C[M, N] (bf16, row-major) = sa * sb * A[M, K] * B[N, K]^T, fp32 accumulation,
// A and B K-contiguous E4M3 codes. This is the tcgen05 + TMA + mbarrier pipeline that ptx-std
// documents as its canonical pattern (src/tcgen05/mod.rs:105-162), assembled into a persistent,
// warp-specialised kernel:
//   warp 0        TMA producer: one elected lane streams 128x128-byte A tiles and 256x128-byte B
//                 tiles (128-byte swizzle) into a STAGES-deep ring, arming `full[s]` with the
//                 byte count (tma_load_tile, src/tma/tensor.rs:214-236; arrive_expect_tx,
//                 src/mbarrier.rs:533);
//   warp 1        TMEM owner and MMA issuer: one lane issues tcgen05.mma.kind::f8f6f4 (M=128,
//                 N=256, K=32) four times per stage and commits each stage back to `empty[s]`
//                 (src/tcgen05/mma.rs:434-453, sync.rs:70-80);
//   warps 2..5    epilogue: tcgen05.ld.32x32b of their TMEM lane quarter, scale, RN to bf16,
//                 16-byte stores (src/tcgen05/ld_st.rs:252-300); in the CTA-pair form the bf16
//                 rows go through two swizzled staging buffers per warp and TMA tile stores of
//                 32 rows x 64 columns (epilogue.cuh).
// Two 128x256 fp32 accumulators (all 512 TMEM columns) let the epilogue of tile i overlap the
// main loop of tile i+1. Tiles are visited in groups of 8 M-blocks so that concurrently running
// CTAs share B tiles in L2. Every wait is bounded (kWaitLimitNs); a timeout records
// PTXSTD_ETIMEOUT in the device error word, drains outstanding copies and MMAs, frees TMEM and
// returns.
#include "common.cuh"
#include "data_types.cuh"
#include "epilogue.cuh"
#include "tcgen05.cuh"
#include "tma_host.h"

namespace {

namespace t5 = ptxstd::tcgen05;
namespace dt = ptxstd::data_types;
using ptxstd::mbar_wait;

constexpr uint32_t BM = 128, BN = 256, BK = 128;  // BK in bytes = E4M3 elements
constexpr uint32_t STAGES = 4;
constexpr uint32_t kThreads = 192;
constexpr uint32_t kABytes = BM * BK;
constexpr uint32_t kBBytes = BN * BK;
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kAccCols = BN;
constexpr uint32_t kTmemCols = 2 * kAccCols;
constexpr uint32_t kGroupM = 8;
constexpr uint32_t kMmaK = 32;  // K of one kind::f8f6f4 MMA

struct alignas(1024) Smem {
    uint8_t a[STAGES][kABytes];
    uint8_t b[STAGES][kBBytes];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

// Error-word detail codes: which wait gave up.
enum : uint32_t { kDetailProducer = 0x100, kDetailMma = 0x200, kDetailEpilogue = 0x300 };

__device__ __forceinline__ void tile_coords(uint32_t t, uint32_t num_m, uint32_t num_n,
                                            uint32_t& mb, uint32_t& nb) {
    const uint32_t group_tiles = kGroupM * num_n;
    const uint32_t g = t / group_tiles;
    const uint32_t first_m = g * kGroupM;
    const uint32_t gm = min(num_m - first_m, kGroupM);
    const uint32_t local = t - g * group_tiles;
    mb = first_m + local % gm;
    nb = local / gm;
}

__device__ __forceinline__ void fail(Smem& s, uint32_t* err, uint32_t detail) {
    ptxstd::record_error(err, PTXSTD_ETIMEOUT, detail);
    *reinterpret_cast<volatile uint32_t*>(&s.abort) = 1u;
}
__device__ __forceinline__ bool aborted(Smem& s) {
    return *reinterpret_cast<volatile uint32_t*>(&s.abort) != 0u;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    uint16_t* __restrict__ C, uint32_t M, uint32_t N, uint32_t K, float alpha,
                    uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t num_m = M / BM, num_n = N / BN, num_tiles = num_m * num_n, num_k = K / BK;

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmA);
        ptxstd::prefetch_tensormap(&tmB);
        for (uint32_t i = 0; i < STAGES; ++i) {
            ptxstd::mbar_init(&s.full[i], 1);
            ptxstd::mbar_init(&s.empty[i], 1);
        }
        for (uint32_t i = 0; i < 2; ++i) {
            ptxstd::mbar_init(&s.tfull[i], 1);
            ptxstd::mbar_init(&s.tempty[i], 4);
        }
        ptxstd::mbar_init(&s.drain, 1);
        s.abort = 0;
        ptxstd::fence_mbarrier_init();
    }
    if (warp == 1) {
        t5::tmem_alloc(&s.tmem_base, kTmemCols);
        t5::tmem_relinquish();
    }
    t5::fence_before_thread_sync();
    __syncthreads();
    t5::fence_after_thread_sync();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (ptxstd::elect_one()) {
            uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
            for (uint32_t t = blockIdx.x; t < num_tiles && !aborted(s); t += gridDim.x) {
                uint32_t mb, nb;
                tile_coords(t, num_m, num_n, mb, nb);
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.empty[stage], phase ^ 1u)) {
                        fail(s, err, kDetailProducer | stage);
                        break;
                    }
                    if (aborted(s)) break;
                    ptxstd::mbar_arrive_expect_tx(&s.full[stage], kStageBytes);
                    ptxstd::tma_load_2d(s.a[stage], &tmA, &s.full[stage],
                                        static_cast<int32_t>(kb * BK), static_cast<int32_t>(mb * BM));
                    ptxstd::tma_load_2d(s.b[stage], &tmB, &s.full[stage],
                                        static_cast<int32_t>(kb * BK), static_cast<int32_t>(nb * BN));
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (aborted(s)) {
                // Wait (bounded) for this thread's copies still in flight before the CTA exits.
                for (uint32_t i = 0; i < STAGES; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.full[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (ptxstd::elect_one()) {
            uint32_t idesc = 0;
            t5::idesc_dense(/*E4m3*/ 0, /*E4m3*/ 0, /*F32*/ 1, BM, BN, idesc);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            for (uint32_t t = blockIdx.x; t < num_tiles && !aborted(s); t += gridDim.x) {
                if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u)) {
                    fail(s, err, kDetailMma | 0x10 | acc);
                    break;
                }
                t5::fence_after_thread_sync();
                const uint32_t d = tmem + acc * kAccCols;
                bool ok = true;
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.full[stage], phase)) {
                        fail(s, err, kDetailMma | stage);
                        ok = false;
                        break;
                    }
                    t5::fence_after_thread_sync();
                    const uint64_t ad = t5::smem_desc_k128(ptxstd::smem_u32(s.a[stage]));
                    const uint64_t bd = t5::smem_desc_k128(ptxstd::smem_u32(s.b[stage]));
#pragma unroll
                    for (uint32_t k = 0; k < BK / kMmaK; ++k) {
                        // +32 bytes along K inside the 128-byte swizzle atom (descriptor units
                        // of 16 bytes, SmemDescriptor::add_start_bytes).
                        t5::mma_f8f6f4(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0u);
                    }
                    t5::commit(&s.empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                t5::commit(&s.tfull[acc]);
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            // All MMAs of this thread complete before TMEM is released.
            t5::commit(&s.drain);
            mbar_wait(&s.drain, 0);
        }
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const uint32_t q = warp & 3u;  // TMEM lane quarter this warp may access
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            bool ok = !aborted(s) && mbar_wait(&s.tfull[acc], acc_phase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !aborted(s)) fail(s, err, kDetailEpilogue | acc);
                break;
            }
            t5::fence_after_thread_sync();
            uint32_t mb, nb;
            tile_coords(t, num_m, num_n, mb, nb);
            const uint32_t row = mb * BM + 32 * q + lane;
            uint16_t* crow = C + static_cast<size_t>(row) * N + nb * BN;
            const uint32_t tbase = tmem + ((32 * q) << 16) + acc * kAccCols;
#pragma unroll 1
            for (uint32_t c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                t5::ld_32x32b_x32(tbase + 32 * c, r);
                t5::wait_ld();
                uint32_t p[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    p[j] = dt::bf16x2_from_f32(__uint_as_float(r[2 * j]) * alpha,
                                               __uint_as_float(r[2 * j + 1]) * alpha);
                uint4* dst = reinterpret_cast<uint4*>(crow + 32 * c);
#pragma unroll
                for (int v = 0; v < 4; ++v)
                    dst[v] = make_uint4(p[4 * v], p[4 * v + 1], p[4 * v + 2], p[4 * v + 3]);
            }
            t5::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive(&s.tempty[acc]);
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
    }

    t5::fence_before_thread_sync();
    __syncthreads();
    t5::fence_after_thread_sync();
    if (warp == 1) t5::tmem_dealloc(tmem, kTmemCols);
}


// ---------------------------------------------------------------------------------------------
// CTA-pair form (tcgen05 CtaGroup::Two, src/tcgen05/mod.rs:40-57): a cluster of two CTAs computes
// a 256 x 256 tile. CTA r of the pair TMA-loads A rows [128 r, 128 r + 128) and B rows
// [128 r, 128 r + 128) of the tile into its own smem, each load completing on the leader's (r = 0)
// `full` barrier (tma_load_tile_to_cluster with CtaGroup::Two and no multicast,
// src/tma/tensor.rs:441-480). The leader alone issues tcgen05.mma.cta_group::2 (M = 256, N = 256,
// K = 32), which reads A from each CTA's smem and the two halves of B from both, and accumulates
// each CTA's 128 rows in that CTA's TMEM. Commits go to the matching barrier of both CTAs as two
// unicast commits (one through mapa, src/tcgen05/sync.rs:56-57). Each CTA's epilogue drains its own
// TMEM; the follower's epilogue warps release an accumulator by arriving on the leader's barrier.
// Per MMA each CTA's smem supplies 4 KiB of A and 4 KiB of B, against 4 + 8 KiB in the one-CTA
// form, and the 32 KiB stage lets the ring hold 6 stages.
constexpr uint32_t P_BM = 256, P_BN = 256;          // tile of the pair
constexpr uint32_t P_HALF = 128;                    // rows of A and of B per CTA
constexpr uint32_t P_STAGES = 6;
constexpr uint32_t kPHalfBytes = P_HALF * BK;        // 16 KiB
constexpr uint32_t kPStageBytesPair = 4 * kPHalfBytes;  // both CTAs' A and B halves

struct alignas(1024) SmemPair {
    uint8_t a[P_STAGES][kPHalfBytes];
    uint8_t b[P_STAGES][kPHalfBytes];
    // epilogue staging: two buffers of 32 rows x 64 bf16 columns per epilogue warp
    uint8_t cstage[4][2][ptxstd::epi::Box<64>::kBytes];
    uint64_t full[P_STAGES];   // leader's counts both CTAs' bytes
    uint64_t empty[P_STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];        // leader's: 8 arrivals (4 epilogue warps of each CTA)
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
};
constexpr size_t kSmemPairBytes = sizeof(SmemPair) + 1024;
static_assert(kSmemPairBytes <= 232448, "shared memory budget");

__device__ __forceinline__ void fail_pair(SmemPair& s, uint32_t* err, uint32_t detail) {
    ptxstd::record_error(err, PTXSTD_ETIMEOUT, detail);
    *reinterpret_cast<volatile uint32_t*>(&s.abort) = 1u;
}
__device__ __forceinline__ bool aborted_pair(SmemPair& s) {
    return *reinterpret_cast<volatile uint32_t*>(&s.abort) != 0u;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                         const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, uint32_t M, uint32_t N,
                         uint32_t K, float alpha, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    SmemPair& s = *reinterpret_cast<SmemPair*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t rank = ptxstd::cluster_ctarank();        // 0 = leader
    const uint32_t pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const uint32_t num_m = M / P_BM, num_n = N / P_BN, num_tiles = num_m * num_n, num_k = K / BK;

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmA);
        ptxstd::prefetch_tensormap(&tmB);
        ptxstd::prefetch_tensormap(&tmC);
        for (uint32_t i = 0; i < P_STAGES; ++i) {
            ptxstd::mbar_init(&s.full[i], 1);
            ptxstd::mbar_init(&s.empty[i], 1);
        }
        for (uint32_t i = 0; i < 2; ++i) {
            ptxstd::mbar_init(&s.tfull[i], 1);
            ptxstd::mbar_init(&s.tempty[i], 8);
        }
        ptxstd::mbar_init(&s.drain, 1);
        s.abort = 0;
        ptxstd::fence_mbarrier_init();
    }
    if (warp == 1) {
        t5::tmem_alloc_pair(&s.tmem_base, kTmemCols);
        t5::tmem_relinquish_pair();
    }
    t5::fence_before_thread_sync();
    ptxstd::cluster_sync();  // both CTAs' barriers and TMEM exist before any remote use
    t5::fence_after_thread_sync();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        // ---------------- TMA producer (both CTAs) ----------------
        if (ptxstd::elect_one()) {
            uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
            for (uint32_t t = pair; t < num_tiles && !aborted_pair(s); t += n_pairs) {
                uint32_t mb, nb;
                tile_coords(t, num_m, num_n, mb, nb);
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.empty[stage], phase ^ 1u)) {
                        fail_pair(s, err, kDetailProducer | 0x80 | stage);
                        break;
                    }
                    if (aborted_pair(s)) break;
                    const uint32_t full_leader =
                        ptxstd::mapa_shared(ptxstd::smem_u32(&s.full[stage]), 0);
                    if (rank == 0) ptxstd::mbar_arrive_expect_tx(&s.full[stage], kPStageBytesPair);
                    ptxstd::tma_load_2d_pair(s.a[stage], &tmA, full_leader,
                                             static_cast<int32_t>(kb * BK),
                                             static_cast<int32_t>(mb * P_BM + rank * P_HALF));
                    ptxstd::tma_load_2d_pair(s.b[stage], &tmB, full_leader,
                                             static_cast<int32_t>(kb * BK),
                                             static_cast<int32_t>(nb * P_BN + rank * P_HALF));
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (aborted_pair(s) && rank == 0) {
                for (uint32_t i = 0; i < P_STAGES; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.full[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader only) ----------------
        if (rank == 0 && ptxstd::elect_one()) {
            uint32_t idesc = 0;
            t5::idesc_dense(/*E4m3*/ 0, /*E4m3*/ 0, /*F32*/ 1, P_BM, P_BN, idesc);
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            const uint32_t peer = 1;
            for (uint32_t t = pair; t < num_tiles && !aborted_pair(s); t += n_pairs) {
                if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1u)) {
                    fail_pair(s, err, kDetailMma | 0x90 | acc);
                    break;
                }
                t5::fence_after_thread_sync();
                const uint32_t d = tmem + acc * kAccCols;
                bool ok = true;
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.full[stage], phase)) {
                        fail_pair(s, err, kDetailMma | 0x80 | stage);
                        ok = false;
                        break;
                    }
                    t5::fence_after_thread_sync();
                    const uint64_t ad = t5::smem_desc_k128(ptxstd::smem_u32(s.a[stage]));
                    const uint64_t bd = t5::smem_desc_k128(ptxstd::smem_u32(s.b[stage]));
#pragma unroll
                    for (uint32_t k = 0; k < BK / kMmaK; ++k)
                        t5::mma_f8f6f4_pair(d, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0u);
                    const uint32_t e = ptxstd::smem_u32(&s.empty[stage]);
                    t5::commit_pair(e);
                    t5::commit_pair(ptxstd::mapa_shared(e, peer));
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                const uint32_t f = ptxstd::smem_u32(&s.tfull[acc]);
                t5::commit_pair(f);
                t5::commit_pair(ptxstd::mapa_shared(f, peer));
                if (++acc == 2) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            t5::commit_pair(ptxstd::smem_u32(&s.drain));
            mbar_wait(&s.drain, 0);
        }
    } else {
        // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
        const uint32_t q = warp & 3u;
        const uint32_t stg = ptxstd::smem_u32(s.cstage[warp - 2u][0]);  // two buffers in a row
        uint32_t acc = 0, acc_phase = 0;
        for (uint32_t t = pair; t < num_tiles; t += n_pairs) {
            bool ok = !aborted_pair(s) && mbar_wait(&s.tfull[acc], acc_phase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !aborted_pair(s)) fail_pair(s, err, kDetailEpilogue | 0x80 | acc);
                break;
            }
            t5::fence_after_thread_sync();
            uint32_t mb, nb;
            tile_coords(t, num_m, num_n, mb, nb);
            const int32_t row0 = static_cast<int32_t>(mb * P_BM + rank * P_HALF + 32 * q);
            const int32_t col0 = static_cast<int32_t>(nb * P_BN);
            const uint32_t tbase = tmem + ((32 * q) << 16) + acc * kAccCols;
            // 64 columns at a time: TMEM -> registers -> staging buffer (two in turn) -> TMA store
#pragma unroll 1
            for (uint32_t c = 0; c < P_BN / 64; ++c) {
                uint32_t r[64];
                t5::ld_32x32b_x32(tbase + 64 * c, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
                t5::ld_32x32b_x32(tbase + 64 * c + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
                t5::wait_ld();
                ptxstd::epi::wait_staging<1>(lane);
                const uint32_t buf = stg + (c & 1u) * ptxstd::epi::Box<64>::kBytes;
                ptxstd::epi::stage_store<64, 0>(&tmC, buf, r, alpha,
                                                col0 + static_cast<int32_t>(64 * c), row0, lane);
            }
            t5::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0)
                ptxstd::mbar_arrive_cluster(ptxstd::mapa_shared(ptxstd::smem_u32(&s.tempty[acc]), 0));
            if (++acc == 2) {
                acc = 0;
                acc_phase ^= 1u;
            }
        }
        ptxstd::epi::drain(lane);
    }

    t5::fence_before_thread_sync();
    ptxstd::cluster_sync();  // neither CTA of the pair leaves while the other may still use it
    t5::fence_after_thread_sync();
    if (warp == 1) t5::tmem_dealloc_pair(tmem, kTmemCols);
}

int launch_pair(const uint8_t* d_a, const uint8_t* d_b, uint16_t* d_c, int64_t M, int64_t N,
                int64_t K, float alpha, cudaStream_t stream) {
    CUtensorMap ta, tb, tc;
    int st = ptxstd::make_tmap_2d(&ta, d_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, K, BK, P_HALF,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tb, d_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, BK, P_HALF,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::epi::make_store_map<64>(&tc, d_c, M, N);
    if (st) return st;
    st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_fp8_pair_kernel),
                                      static_cast<int>(kSmemPairBytes));
    if (st) return st;
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemPairBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // As many pairs as can be resident at once (a persistent grid), but no more than tiles.
    static int max_pairs[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PTXSTD_ECUDA;
    if (max_pairs[dev] == 0) {
        cfg.gridDim = dim3(2 * static_cast<uint32_t>(ptxstd::sm_count() / 2));
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm_fp8_pair_kernel, &cfg) != cudaSuccess ||
            clusters <= 0)
            return PTXSTD_ECUDA;
        max_pairs[dev] = clusters;
    }
    const uint32_t tiles = static_cast<uint32_t>((M / P_BM) * (N / P_BN));
    const uint32_t pairs = tiles < static_cast<uint32_t>(max_pairs[dev]) ? tiles
                                                                        : static_cast<uint32_t>(max_pairs[dev]);
    cfg.gridDim = dim3(2 * pairs);
    if (cudaLaunchKernelEx(&cfg, gemm_fp8_pair_kernel, ta, tb, tc, static_cast<uint32_t>(M),
                           static_cast<uint32_t>(N), static_cast<uint32_t>(K), alpha,
                           err) != cudaSuccess)
        return PTXSTD_ECUDA;
    return ptxstd::launch_status();
}

}  // namespace

extern "C" int ptxstd_gemm_fp8(const uint8_t* d_a, const uint8_t* d_b, float sa, float sb,
                               uint16_t* d_c, int64_t M, int64_t N, int64_t K,
                               ptxstd_stream stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M % BM || N % BN || K % BK) return PTXSTD_EINVAL;
    if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return PTXSTD_EINVAL;
    if (!d_a || !d_b || !d_c || !ptxstd::aligned16(d_a) || !ptxstd::aligned16(d_b) ||
        !ptxstd::aligned16(d_c))
        return PTXSTD_EINVAL;
    CUtensorMap ta, tb;
    int st = ptxstd::make_tmap_2d(&ta, d_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, K, BK, BM,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tb, d_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, BK, BN,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_fp8_kernel),
                                      static_cast<int>(kSmemBytes));
    if (st) return st;
    const uint32_t tiles = static_cast<uint32_t>((M / BM) * (N / BN));
    const uint32_t grid = tiles < static_cast<uint32_t>(ptxstd::sm_count())
                              ? tiles
                              : static_cast<uint32_t>(ptxstd::sm_count());
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    const float alpha = sa * sb;
    if (M % P_BM == 0 && N % P_BN == 0)
        return launch_pair(d_a, d_b, d_c, M, N, K, alpha, static_cast<cudaStream_t>(stream));
    gemm_fp8_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
        ta, tb, d_c, static_cast<uint32_t>(M), static_cast<uint32_t>(N),
        static_cast<uint32_t>(K), alpha, err);
    return ptxstd::launch_status();
}

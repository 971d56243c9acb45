// NVFP4 block-scaled GEMM on the 5th-generation tensor cores:
//   C[M, N] (bf16) = ga * gb * sum_k (A[m,k] sfA[m,k/16]) (B[n,k] sfB[n,k/16])
// with A [M, K/2] and B [N, K/2] E2M1 packed two per byte (element 0 in the low nibble, K
// contiguous), E4M3 scales per 16 K elements in the blocked 128x4 layout, f32 global scales ga and
// gb, fp32 accumulation and bf16 RN output. tcgen05.mma.kind::mxf4nvf4.block_scale.block16 (the
// reference's mma_block_scaled with ScaleVectorSize::Block16, src/tcgen05/mma.rs:698-724;
// InstrDescriptor::<Mxf4nvf4>::new(Ue4m3, 128, 256), src/tcgen05/descriptor.rs:644-653).
//
// Per 256-element K stage the producer issues two TMA tile loads (A 128 rows x 128 bytes, B 256
// rows x 128 bytes, 128-byte swizzle) and three 1-D bulk copies of scales: in the blocked layout
// the four 512-byte scale tiles of one 128-row block and one stage are contiguous, so A's scales
// are one 2 KiB copy and B's two. The MMA thread moves each 512-byte tile to TMEM with
// tcgen05.cp.32x128b.warpx4 (src/tcgen05/copy.rs:29-30, :76-116) — 32 lanes x 16 bytes
// replicated to the four lane quarters, which is the scale layout the MMA reads — and issues the
// four K=64 MMAs of the stage. Scale slots in TMEM are per (stage, MMA), so a slot is rewritten
// only after the stage's `empty` barrier has observed the completion of the MMAs that read it.
//
// TMEM: accumulator 128 lanes x 256 f32 columns, plus 4 stages x 4 MMAs x (4 + 8) scale columns.
// The accumulator is single-buffered; eight epilogue warps (two per lane quarter, 128 columns
// each) copy it to registers and release it before converting and storing, so the next tile's
// MMAs wait only for the TMEM reads. In the CTA-pair form the bf16 tile leaves through a
// swizzled staging buffer per warp and TMA tile stores (epilogue.cuh): whole 128-byte row
// segments instead of 16-byte pieces of 32 rows per instruction. At 8192 x 28672 x 8192 on a
// B200 that took a launch from 759 us to 666 us at full clock (913-922 us to 731-738 us once the
// power cap lowers the clock), against 637 us for a copy of the kernel that stores nothing.
#include <atomic>

#include "common.cuh"
#include "data_types.cuh"
#include "epilogue.cuh"
#include "tcgen05.cuh"
#include "tma_host.h"

namespace {

namespace t5 = ptxstd::tcgen05;
namespace dt = ptxstd::data_types;
using ptxstd::mbar_wait;

constexpr uint32_t BM = 128, BN = 256;
constexpr uint32_t BKB = 128;          // K bytes per stage
constexpr uint32_t BK = 2 * BKB;       // K elements per stage (256)
constexpr uint32_t kMmaK = 64;         // K elements of one mxf4nvf4 MMA
constexpr uint32_t kMmas = BK / kMmaK; // 4 per stage
constexpr uint32_t STAGES = 4;
constexpr uint32_t kEpiWarps = 8;
constexpr uint32_t kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kABytes = BM * BKB;
constexpr uint32_t kBBytes = BN * BKB;
constexpr uint32_t kSfaBytes = (BM / 128) * kMmas * 512;  // 2048
constexpr uint32_t kSfbBytes = (BN / 128) * kMmas * 512;  // 4096
constexpr uint32_t kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
constexpr uint32_t kAccCols = BN;
constexpr uint32_t kSfaCols = 4 * (BM / 128);  // per MMA
constexpr uint32_t kSfbCols = 4 * (BN / 128);  // per MMA
constexpr uint32_t kSfSlotCols = kSfaCols + kSfbCols;
constexpr uint32_t kSfBase = kAccCols;
constexpr uint32_t kTmemCols = 512;
static_assert(kSfBase + STAGES * kMmas * kSfSlotCols <= kTmemCols, "TMEM budget");
// Grouped raster: kGroupM row-tiles sweep all column-tiles before moving on. 16 row-tiles (8
// MiB of A at K = 8192 in the pair form) ran 767-782 us against 793-795 us for 8 at 8192 x 28672
// x 8192 on a B200: B is re-read from DRAM once per group.
constexpr uint32_t kGroupM = 16;

struct alignas(1024) Smem {
    uint8_t a[STAGES][kABytes];
    uint8_t b[STAGES][kBBytes];
    uint8_t sfa[STAGES][kSfaBytes];
    uint8_t sfb[STAGES][kSfbBytes];
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull;
    uint64_t tempty;
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum : uint32_t { kDetailProducer = 0x1100, kDetailMma = 0x1200, kDetailEpilogue = 0x1300,
                  kDetailSched = 0x1400 };

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

using ptxstd::bulk_load;

__global__ void __launch_bounds__(kThreads, 1)
    gemm_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA,
                      const __grid_constant__ CUtensorMap tmB, const uint8_t* __restrict__ sfA,
                      const uint8_t* __restrict__ sfB, uint16_t* __restrict__ C, uint32_t M,
                      uint32_t N, uint32_t K, float alpha, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t num_m = M / BM, num_n = N / BN, num_tiles = num_m * num_n, num_k = K / BK;
    const uint32_t sf_tiles_per_row = K / 64;  // 512-byte scale tiles per 128-row block

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmA);
        ptxstd::prefetch_tensormap(&tmB);
        for (uint32_t i = 0; i < STAGES; ++i) {
            ptxstd::mbar_init(&s.full[i], 1);
            ptxstd::mbar_init(&s.empty[i], 1);
        }
        ptxstd::mbar_init(&s.tfull, 1);
        ptxstd::mbar_init(&s.tempty, kEpiWarps);
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
        // ---------------- producer: TMA tiles + bulk scale copies ----------------
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
                                        static_cast<int32_t>(kb * BKB), static_cast<int32_t>(mb * BM));
                    ptxstd::tma_load_2d(s.b[stage], &tmB, &s.full[stage],
                                        static_cast<int32_t>(kb * BKB), static_cast<int32_t>(nb * BN));
                    const size_t ktile = static_cast<size_t>(kb) * kMmas;
                    bulk_load(s.sfa[stage], sfA + (static_cast<size_t>(mb) * sf_tiles_per_row + ktile) * 512,
                              kSfaBytes, &s.full[stage]);
#pragma unroll
                    for (uint32_t j = 0; j < BN / 128; ++j) {
                        const size_t rt = static_cast<size_t>(nb) * (BN / 128) + j;
                        bulk_load(s.sfb[stage] + j * (kMmas * 512),
                                  sfB + (rt * sf_tiles_per_row + ktile) * 512, kMmas * 512,
                                  &s.full[stage]);
                    }
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (aborted(s)) {
                for (uint32_t i = 0; i < STAGES; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.full[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (ptxstd::elect_one()) {
            uint32_t idesc = 0;
            t5::idesc_mxf4nvf4(/*Ue4m3*/ 0, BM, BN, idesc);
            uint32_t stage = 0, phase = 0, acc_phase = 0;
            for (uint32_t t = blockIdx.x; t < num_tiles && !aborted(s); t += gridDim.x) {
                if (!mbar_wait(&s.tempty, acc_phase ^ 1u)) {
                    fail(s, err, kDetailMma | 0x10);
                    break;
                }
                t5::fence_after_thread_sync();
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
                    // All scale copies of the stage first, then its MMAs, so that the copy
                    // latency overlaps the earlier MMAs instead of stalling each one.
#pragma unroll
                    for (uint32_t j = 0; j < kMmas; ++j) {
                        const uint32_t slot = tmem + kSfBase + (stage * kMmas + j) * kSfSlotCols;
                        t5::cp_32x128b_warpx4(
                            slot, t5::smem_desc_nosw(ptxstd::smem_u32(s.sfa[stage] + 512 * j), 0, 128));
#pragma unroll
                        for (uint32_t h = 0; h < BN / 128; ++h)
                            t5::cp_32x128b_warpx4(
                                slot + kSfaCols + 4 * h,
                                t5::smem_desc_nosw(
                                    ptxstd::smem_u32(s.sfb[stage] + h * (kMmas * 512) + 512 * j), 0,
                                    128));
                    }
#pragma unroll
                    for (uint32_t j = 0; j < kMmas; ++j) {
                        const uint32_t slot = tmem + kSfBase + (stage * kMmas + j) * kSfSlotCols;
                        t5::mma_mxf4nvf4_block16(tmem, ad + 2 * j, bd + 2 * j, idesc, slot,
                                                 slot + kSfaCols, (kb | j) != 0u);
                    }
                    t5::commit(&s.empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                t5::commit(&s.tfull);
                acc_phase ^= 1u;
            }
            t5::commit(&s.drain);
            mbar_wait(&s.drain, 0);
        }
    } else {
        // ---------------- epilogue: warps 2..9 ----------------
        const uint32_t q = warp & 3u;              // TMEM lane quarter
        const uint32_t half = (warp - 2u) >> 2;    // which 128 columns
        uint32_t acc_phase = 0;
        for (uint32_t t = blockIdx.x; t < num_tiles; t += gridDim.x) {
            bool ok = !aborted(s) && mbar_wait(&s.tfull, acc_phase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !aborted(s)) fail(s, err, kDetailEpilogue);
                break;
            }
            t5::fence_after_thread_sync();
            uint32_t r[128];
            const uint32_t tbase = tmem + ((32 * q) << 16) + half * 128;
            {
                uint32_t(&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
                uint32_t(&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
                uint32_t(&r2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[64]);
                uint32_t(&r3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[96]);
                t5::ld_32x32b_x32(tbase, r0);
                t5::ld_32x32b_x32(tbase + 32, r1);
                t5::ld_32x32b_x32(tbase + 64, r2);
                t5::ld_32x32b_x32(tbase + 96, r3);
                t5::wait_ld();
            }
            t5::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive(&s.tempty);
            acc_phase ^= 1u;

            uint32_t mb, nb;
            tile_coords(t, num_m, num_n, mb, nb);
            const uint32_t row = mb * BM + 32 * q + lane;
            uint16_t* crow = C + static_cast<size_t>(row) * N + nb * BN + half * 128;
#pragma unroll
            for (uint32_t c = 0; c < 16; ++c) {
                uint32_t p[4];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    p[j] = dt::bf16x2_from_f32(__uint_as_float(r[8 * c + 2 * j]) * alpha,
                                               __uint_as_float(r[8 * c + 2 * j + 1]) * alpha);
                reinterpret_cast<uint4*>(crow)[c] = make_uint4(p[0], p[1], p[2], p[3]);
            }
        }
    }

    t5::fence_before_thread_sync();
    __syncthreads();
    t5::fence_after_thread_sync();
    if (warp == 1) t5::tmem_dealloc(tmem, kTmemCols);
}


// ---------------------------------------------------------------------------------------------
// CTA-pair form (CtaGroup::Two): a cluster of two CTAs computes a 256 x 256 tile; CTA r loads A
// rows [128 r, +128) and B rows [128 r, +128) into its own smem, plus the scales its own TMEM needs:
// A's for its 128 rows and B's for all 256 columns (each CTA accumulates all N columns of its
// rows). Scales are fetched with 2-D TMA over the blocked layout viewed as u32 [tiles, 128] (box
// 128 x 4 = the four 512-byte tiles of one stage), so that, like the operand tiles, they complete
// on the leader's `full` barrier. The leader issues tcgen05.cp.cta_group::2 (each CTA copies its
// own smem scales into its own TMEM) and tcgen05.mma.cta_group::2.kind::mxf4nvf4 (M = 256).
//
// Warp roles, 12 warps in three warpgroups:
//   warp 0      producer (both CTAs): operand tiles and scales into the P_STAGES ring;
//   warp 1      TMEM owner; in the leader, the MMA issuer;
//   warp 2      tile scheduler (leader), dynamic schedule only: the grid holds one cluster per
//               tile, and a running pair takes over the tiles of clusters not started yet by
//               cancelling them
//               (clusterlaunchcontrol.try_cancel, the reference's
//               try_cancel_launch::<CancelDelivery::Block>, src/launch.rs:154-176). It publishes
//               each tile index to both CTAs through a ring of kSlots entries in shared memory
//               (written into the peer with st.shared::cluster, signalled by remote arrives), and
//               kNoTile once a request cancels nothing;
//   warp 3      idle;
//   warps 4-11  epilogue, two per TMEM lane quarter (128 columns each).
// The persistent schedule (the default) launches one pair per two SMs and every role walks the
// static raster pair, pair + n_pairs, ... itself. On 8192 x 28672 x 8192 alone on a B200 it ran
// 681 us against 691 us for the dynamic one, whose per-tile hand-offs cost about 1.5 %; the
// dynamic schedule is for GEMMs that share the GPU with other kernels.
// Warpgroup 0 needs few registers and the epilogue's hold a 128-column accumulator row per
// thread, so warpgroup 0 gives registers back with setmaxnreg.dec (decrease_max_registers,
// src/launch.rs:240) and the two epilogue warpgroups take them with setmaxnreg.inc
// (increase_max_registers, :204). The kernel is launched at kRegsLaunch registers per thread.
constexpr uint32_t P_BM = 256, P_BN = 256, P_HALF = 128;
constexpr uint32_t kPThreads = 384;
constexpr uint32_t kPFirstEpiWarp = 4;
constexpr uint32_t kRegsLaunch = 168;  // 65536 / 384, rounded down to a multiple of 8
constexpr uint32_t kRegsCtl = 80, kRegsEpi = 208;
static_assert(128 * kRegsCtl + 256 * kRegsEpi <= kPThreads * kRegsLaunch, "register split");
constexpr uint32_t kSlots = 4;  // tile-index ring between the scheduler and the other roles
constexpr uint32_t kNoTile = 0xffffffffu;
// roles that read every published tile index: producer (both CTAs), MMA, epilogue (both CTAs)
constexpr uint32_t kSlotReaders = 2 + 1 + 2 * kEpiWarps;
constexpr uint32_t P_STAGES = 5;
constexpr uint32_t kPABytes = P_HALF * BKB;            // 16 KiB
constexpr uint32_t kPBBytes = P_HALF * BKB;            // 16 KiB
constexpr uint32_t kPSfaBytes = kMmas * 512;           // 2 KiB: this CTA's 128 rows
constexpr uint32_t kPSfbBytes = (P_BN / 128) * kMmas * 512;  // 4 KiB: all 256 columns
constexpr uint32_t kPCtaStageBytes = kPABytes + kPBBytes + kPSfaBytes + kPSfbBytes;
constexpr uint32_t kPSfbCols = 4 * (P_BN / 128);
constexpr uint32_t kPSlotCols = 4 + kPSfbCols;
static_assert(kSfBase + P_STAGES * kMmas * kPSlotCols <= kTmemCols, "TMEM budget (pair)");

struct alignas(1024) SmemPair {
    uint8_t a[P_STAGES][kPABytes];
    uint8_t b[P_STAGES][kPBBytes];
    uint8_t sfa[P_STAGES][kPSfaBytes];
    uint8_t sfb[P_STAGES][kPSfbBytes];
    uint8_t cstage[kEpiWarps][ptxstd::epi::Box<64>::kBytes];  // epilogue staging, one per warp
    uint4 clc_resp;  // cluster launch control response (leader)
    uint64_t full[P_STAGES];
    uint64_t empty[P_STAGES];
    uint64_t tfull;
    uint64_t tempty;  // leader's: one arrive per epilogue warp of both CTAs
    uint64_t drain;
    uint64_t clc_bar;               // leader's: completes when a response has arrived
    uint64_t slot_full[kSlots];     // both CTAs: the scheduler has published the slot
    uint64_t slot_empty[kSlots];    // leader's: every reader of both CTAs has read the slot
    uint32_t slot_tile[kSlots];     // both CTAs: published tile indices
    uint32_t tmem_base;
    uint32_t abort;
};
constexpr size_t kSmemPairBytes = sizeof(SmemPair) + 1024;
static_assert(kSmemPairBytes <= 232448, "shared memory budget (pair)");

__device__ __forceinline__ void fail_pair(SmemPair& s, uint32_t* err, uint32_t detail) {
    ptxstd::record_error(err, PTXSTD_ETIMEOUT, detail);
    *reinterpret_cast<volatile uint32_t*>(&s.abort) = 1u;
}
__device__ __forceinline__ bool aborted_pair(SmemPair& s) {
    return *reinterpret_cast<volatile uint32_t*>(&s.abort) != 0u;
}

// Entry `seq` of the published tile sequence: waits (bounded) for slot seq % kSlots and returns
// its tile index, or kNoTile after a timeout (recorded). The caller tells the scheduler it has
// read the slot with release_slot once every lane that needs the index has it. The leader's
// readers synchronise with the scheduler (a thread of their own CTA) at CTA scope; the peer's
// readers, whose slot the scheduler writes remotely, at cluster scope.
__device__ __forceinline__ uint32_t read_slot(SmemPair& s, uint32_t seq, uint32_t rank,
                                              uint32_t* err, uint32_t detail) {
    const uint32_t slot = seq % kSlots, parity = (seq / kSlots) & 1u;
    const bool ok = rank == 0 ? ptxstd::mbar_wait(&s.slot_full[slot], parity)
                              : ptxstd::mbar_wait_cluster(&s.slot_full[slot], parity);
    if (!ok) {
        if (!aborted_pair(s)) fail_pair(s, err, detail);
        return kNoTile;
    }
    return *reinterpret_cast<volatile uint32_t*>(&s.slot_tile[slot]);
}
__device__ __forceinline__ void release_slot(SmemPair& s, uint32_t seq, uint32_t rank) {
    if (rank == 0)
        ptxstd::mbar_arrive(&s.slot_empty[seq % kSlots]);
    else
        ptxstd::mbar_arrive_cluster(
            ptxstd::mapa_shared(ptxstd::smem_u32(&s.slot_empty[seq % kSlots]), 0));
}

// Entry `seq` of this pair's tile sequence, for a role that reads it with one thread.
// Persistent schedule: the static raster pair, pair + n_pairs, ... (no communication).
// Dynamic schedule: the scheduler's published entry, released once read.
template <bool kDynamic>
__device__ __forceinline__ uint32_t take_tile(SmemPair& s, uint32_t seq, uint32_t rank,
                                              uint32_t num_tiles, uint32_t* err,
                                              uint32_t detail) {
    if constexpr (!kDynamic) {
        const uint64_t t = (blockIdx.x >> 1) + static_cast<uint64_t>(seq) * (gridDim.x >> 1);
        return t < num_tiles ? static_cast<uint32_t>(t) : kNoTile;
    } else {
        const uint32_t t = read_slot(s, seq, rank, err, detail);
        if (t != kNoTile) release_slot(s, seq, rank);
        return t;
    }
}

template <bool kDynamic>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_nvfp4_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                           const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmSfa,
                           const __grid_constant__ CUtensorMap tmSfb,
                           const __grid_constant__ CUtensorMap tmC, uint32_t M, uint32_t N,
                           uint32_t K, float alpha, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    SmemPair& s = *reinterpret_cast<SmemPair*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t rank = ptxstd::cluster_ctarank();
    const uint32_t num_m = M / P_BM, num_n = N / P_BN, num_k = K / BK;
    const uint32_t num_tiles = num_m * num_n;
    const uint32_t sf_tiles_per_row = K / 64;

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmA);
        ptxstd::prefetch_tensormap(&tmB);
        ptxstd::prefetch_tensormap(&tmSfa);
        ptxstd::prefetch_tensormap(&tmSfb);
        ptxstd::prefetch_tensormap(&tmC);
        for (uint32_t i = 0; i < P_STAGES; ++i) {
            ptxstd::mbar_init(&s.full[i], 1);
            ptxstd::mbar_init(&s.empty[i], 1);
        }
        ptxstd::mbar_init(&s.tfull, 1);
        ptxstd::mbar_init(&s.tempty, 2 * kEpiWarps);
        ptxstd::mbar_init(&s.drain, 1);
        ptxstd::mbar_init(&s.clc_bar, 1);
        for (uint32_t i = 0; i < kSlots; ++i) {
            ptxstd::mbar_init(&s.slot_full[i], 1);
            ptxstd::mbar_init(&s.slot_empty[i], kSlotReaders);
        }
        s.abort = 0;
        ptxstd::fence_mbarrier_init();
    }
    if (warp == 1) {
        t5::tmem_alloc_pair(&s.tmem_base, kTmemCols);
        t5::tmem_relinquish_pair();
    }
    t5::fence_before_thread_sync();
    ptxstd::cluster_sync();
    t5::fence_after_thread_sync();
    const uint32_t tmem = s.tmem_base;
    // Each role changes its register budget at the top of its own branch, so that the compiler
    // allocates every branch for the budget it runs with.

    if (warp == 0) {
        // ---------------- producer (both CTAs) ----------------
        ptxstd::setmaxnreg_dec<kRegsCtl>();
        if (ptxstd::elect_one()) {
            uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
            uint32_t t = take_tile<kDynamic>(s, 0, rank, num_tiles, err, kDetailProducer | 0xC0);
            for (uint32_t seq = 0; t != kNoTile && !aborted_pair(s); ++seq) {
                uint32_t mb, nb, t_next = kNoTile;
                tile_coords(t, num_m, num_n, mb, nb);
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (kb == 1 || num_k == 1) {
                        // the next tile index, read inside this tile rather than at its end
                        t_next = take_tile<kDynamic>(s, seq + 1, rank, num_tiles, err,
                                                     kDetailProducer | 0xC1);
                    }
                    if (!mbar_wait(&s.empty[stage], phase ^ 1u)) {
                        fail_pair(s, err, kDetailProducer | 0x80 | stage);
                        break;
                    }
                    if (aborted_pair(s)) break;
                    const uint32_t fl = ptxstd::mapa_shared(ptxstd::smem_u32(&s.full[stage]), 0);
                    if (rank == 0) ptxstd::mbar_arrive_expect_tx(&s.full[stage], 2 * kPCtaStageBytes);
                    ptxstd::tma_load_2d_pair(s.a[stage], &tmA, fl, static_cast<int32_t>(kb * BKB),
                                             static_cast<int32_t>(mb * P_BM + rank * P_HALF));
                    ptxstd::tma_load_2d_pair(s.b[stage], &tmB, fl, static_cast<int32_t>(kb * BKB),
                                             static_cast<int32_t>(nb * P_BN + rank * P_HALF));
                    const int32_t ktile = static_cast<int32_t>(kb * kMmas);
                    ptxstd::tma_load_2d_pair(
                        s.sfa[stage], &tmSfa, fl, 0,
                        static_cast<int32_t>((mb * 2 + rank) * sf_tiles_per_row) + ktile);
#pragma unroll
                    for (uint32_t j = 0; j < P_BN / 128; ++j)
                        ptxstd::tma_load_2d_pair(
                            s.sfb[stage] + j * (kMmas * 512), &tmSfb, fl, 0,
                            static_cast<int32_t>((nb * 2 + j) * sf_tiles_per_row) + ktile);
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                t = t_next;
            }
            if (aborted_pair(s) && rank == 0) {
                for (uint32_t i = 0; i < P_STAGES; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.full[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader) ----------------
        ptxstd::setmaxnreg_dec<kRegsCtl>();
        if (rank == 0 && ptxstd::elect_one()) {
            uint32_t idesc = 0;
            t5::idesc_mxf4nvf4(/*Ue4m3*/ 0, P_BM, P_BN, idesc);
            uint32_t stage = 0, phase = 0, acc_phase = 0;
            // the MMA issuer needs only whether another tile follows; it reads the next index
            // inside the current tile, so that no tile boundary waits on the scheduler
            uint32_t t = take_tile<kDynamic>(s, 0, 0, num_tiles, err, kDetailMma | 0xC0);
            for (uint32_t seq = 0; t != kNoTile && !aborted_pair(s); ++seq) {
                uint32_t t_next = kNoTile;
                if (!mbar_wait(&s.tempty, acc_phase ^ 1u)) {
                    fail_pair(s, err, kDetailMma | 0x90);
                    break;
                }
                t5::fence_after_thread_sync();
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
                    for (uint32_t j = 0; j < kMmas; ++j) {
                        const uint32_t slot = tmem + kSfBase + (stage * kMmas + j) * kPSlotCols;
                        t5::cp_32x128b_warpx4_pair(
                            slot, t5::smem_desc_nosw(ptxstd::smem_u32(s.sfa[stage] + 512 * j), 0, 128));
#pragma unroll
                        for (uint32_t h = 0; h < P_BN / 128; ++h)
                            t5::cp_32x128b_warpx4_pair(
                                slot + 4 + 4 * h,
                                t5::smem_desc_nosw(
                                    ptxstd::smem_u32(s.sfb[stage] + h * (kMmas * 512) + 512 * j), 0,
                                    128));
                    }
#pragma unroll
                    for (uint32_t j = 0; j < kMmas; ++j) {
                        const uint32_t slot = tmem + kSfBase + (stage * kMmas + j) * kPSlotCols;
                        t5::mma_mxf4nvf4_block16_pair(tmem, ad + 2 * j, bd + 2 * j, idesc, slot,
                                                      slot + 4, (kb | j) != 0u);
                    }
                    const uint32_t e = ptxstd::smem_u32(&s.empty[stage]);
                    t5::commit_pair(e);
                    t5::commit_pair(ptxstd::mapa_shared(e, 1));
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    if (kb == 0) {
                        t_next = take_tile<kDynamic>(s, seq + 1, 0, num_tiles, err,
                                                     kDetailMma | 0xC1);
                    }
                }
                if (!ok) break;
                const uint32_t f = ptxstd::smem_u32(&s.tfull);
                t5::commit_pair(f);
                t5::commit_pair(ptxstd::mapa_shared(f, 1));
                acc_phase ^= 1u;
                t = t_next;
            }
            t5::commit_pair(ptxstd::smem_u32(&s.drain));
            mbar_wait(&s.drain, 0);
        }
    } else if (warp == 2) {
        // ---------------- tile scheduler (leader) ----------------
        ptxstd::setmaxnreg_dec<kRegsCtl>();
        if (kDynamic && rank == 0 && ptxstd::elect_one()) {
            uint32_t t = blockIdx.x >> 1;  // this cluster's own tile first
            uint32_t resp_phase = 0;
            for (uint32_t seq = 0;; ++seq) {
                const uint32_t slot = seq % kSlots;
                // every reader of both CTAs has read this slot's previous entry
                if (!mbar_wait(&s.slot_empty[slot], ((seq / kSlots) & 1u) ^ 1u)) {
                    fail_pair(s, err, kDetailSched | slot);
                    break;
                }
                s.slot_tile[slot] = t;
                ptxstd::st_shared_cluster_u32(
                    ptxstd::mapa_shared(ptxstd::smem_u32(&s.slot_tile[slot]), 1), t);
                ptxstd::mbar_arrive(&s.slot_full[slot]);
                ptxstd::mbar_arrive_cluster(
                    ptxstd::mapa_shared(ptxstd::smem_u32(&s.slot_full[slot]), 1));
                if (t == kNoTile) break;
                // the next tile: cancel a cluster that has not started and take over its tile
                ptxstd::fence_proxy_async_smem();  // earlier reads of the response come first
                ptxstd::mbar_arrive_expect_tx(&s.clc_bar, 16);
                ptxstd::clc_try_cancel(&s.clc_resp, &s.clc_bar);
                if (!mbar_wait(&s.clc_bar, resp_phase)) {
                    fail_pair(s, err, kDetailSched | 0x10);
                    t = kNoTile;
                    continue;  // publish the end of the sequence
                }
                resp_phase ^= 1u;
                const int32_t x = ptxstd::clc_first_ctaid_x(&s.clc_resp);
                t = x < 0 ? kNoTile : static_cast<uint32_t>(x) >> 1;
            }
        }
    } else if (warp == 3) {
        ptxstd::setmaxnreg_dec<kRegsCtl>();  // idle: its share of registers goes to the epilogue
    } else {
        // ---------------- epilogue: warps 4..11 of both CTAs ----------------
        ptxstd::setmaxnreg_inc<kRegsEpi>();
        const uint32_t q = warp & 3u;
        const uint32_t half = (warp - kPFirstEpiWarp) >> 2;
        uint32_t acc_phase = 0;
        const uint32_t tempty_leader = ptxstd::mapa_shared(ptxstd::smem_u32(&s.tempty), 0);
        const uint32_t stg = ptxstd::smem_u32(s.cstage[warp - kPFirstEpiWarp]);
        for (uint32_t seq = 0;; ++seq) {
            uint32_t t = 0;
            if constexpr (kDynamic) {
                if (lane == 0) t = read_slot(s, seq, rank, err, kDetailEpilogue | 0xC0);
                t = __shfl_sync(0xffffffffu, t, 0);
                if (t != kNoTile && lane == 0) release_slot(s, seq, rank);
            } else {
                t = take_tile<false>(s, seq, rank, num_tiles, err, 0);
            }
            if (t == kNoTile) break;
            bool ok = !aborted_pair(s) && mbar_wait(&s.tfull, acc_phase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !aborted_pair(s)) fail_pair(s, err, kDetailEpilogue | 0x80);
                break;
            }
            t5::fence_after_thread_sync();
            uint32_t r[128];
            const uint32_t tbase = tmem + ((32 * q) << 16) + half * 128;
            {
                uint32_t(&r0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[0]);
                uint32_t(&r1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[32]);
                uint32_t(&r2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[64]);
                uint32_t(&r3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&r[96]);
                t5::ld_32x32b_x32(tbase, r0);
                t5::ld_32x32b_x32(tbase + 32, r1);
                t5::ld_32x32b_x32(tbase + 64, r2);
                t5::ld_32x32b_x32(tbase + 96, r3);
                t5::wait_ld();
            }
            t5::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive_cluster(tempty_leader);
            acc_phase ^= 1u;

            uint32_t mb, nb;
            tile_coords(t, num_m, num_n, mb, nb);
            // 32 rows x 128 columns of bf16 leave as two TMA stores of 32 x 64 through this
            // warp's staging buffer
            const int32_t row0 = static_cast<int32_t>(mb * P_BM + rank * P_HALF + 32 * q);
            const int32_t col0 = static_cast<int32_t>(nb * P_BN + half * 128);
            ptxstd::epi::store_row_block<64>(&tmC, stg, r, alpha, col0, row0, lane);
        }
        ptxstd::epi::drain(lane);
    }

    t5::fence_before_thread_sync();
    ptxstd::cluster_sync();
    t5::fence_after_thread_sync();
    if (warp == 1) t5::tmem_dealloc_pair(tmem, kTmemCols);
}

int launch_pair(const uint8_t* d_a, const uint8_t* d_sfa, const uint8_t* d_b,
                const uint8_t* d_sfb, uint16_t* d_c, int64_t M, int64_t N, int64_t K, float alpha,
                cudaStream_t stream) {
    CUtensorMap ta, tb, tsa, tsb, tc;
    int st = ptxstd::make_tmap_2d(&ta, d_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, M, K / 2, BKB,
                                  P_HALF, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tb, d_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2, BKB,
                              P_HALF, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // blocked scales as u32 [tiles, 128]: one row per 512-byte tile
    st = ptxstd::make_tmap_2d(&tsa, d_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128,
                              (M / 128) * (K / 64), 512, 128, kMmas, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tsb, d_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128,
                              (N / 128) * (K / 64), 512, 128, kMmas, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::epi::make_store_map<64>(&tc, d_c, M, N);
    if (st) return st;
    const bool dynamic = ptxstd_get_gemm_schedule() == PTXSTD_SCHEDULE_DYNAMIC;
    const void* kernel = dynamic ? reinterpret_cast<const void*>(gemm_nvfp4_pair_kernel<true>)
                                 : reinterpret_cast<const void*>(gemm_nvfp4_pair_kernel<false>);
    st = ptxstd::set_max_dynamic_smem(kernel, static_cast<int>(kSmemPairBytes));
    if (st) return st;
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = kSmemPairBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const uint64_t tiles = static_cast<uint64_t>(M / P_BM) * static_cast<uint64_t>(N / P_BN);
    if (2 * tiles >= (1ull << 31)) return PTXSTD_EINVAL;
    cudaError_t e;
    if (dynamic) {
        // one cluster per tile: the clusters that run first take over the tiles of those that
        // have not started (cluster launch control), so no tile waits for one particular pair
        cfg.gridDim = dim3(static_cast<uint32_t>(2 * tiles));
        e = cudaLaunchKernelEx(&cfg, gemm_nvfp4_pair_kernel<true>, ta, tb, tsa, tsb, tc,
                               static_cast<uint32_t>(M), static_cast<uint32_t>(N),
                               static_cast<uint32_t>(K), alpha, err);
    } else {
        // persistent: as many pairs as can be resident at once, but no more than tiles
        static int max_pairs[64] = {};
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PTXSTD_ECUDA;
        if (max_pairs[dev] == 0) {
            cfg.gridDim = dim3(2 * static_cast<uint32_t>(ptxstd::sm_count() / 2));
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, gemm_nvfp4_pair_kernel<false>, &cfg) !=
                    cudaSuccess ||
                clusters <= 0)
                return PTXSTD_ECUDA;
            max_pairs[dev] = clusters;
        }
        const uint64_t pairs = tiles < static_cast<uint64_t>(max_pairs[dev])
                                   ? tiles
                                   : static_cast<uint64_t>(max_pairs[dev]);
        cfg.gridDim = dim3(static_cast<uint32_t>(2 * pairs));
        e = cudaLaunchKernelEx(&cfg, gemm_nvfp4_pair_kernel<false>, ta, tb, tsa, tsb, tc,
                               static_cast<uint32_t>(M), static_cast<uint32_t>(N),
                               static_cast<uint32_t>(K), alpha, err);
    }
    if (e != cudaSuccess) return PTXSTD_ECUDA;
    return ptxstd::launch_status();
}

}  // namespace

// Process-wide choice of tile schedule for the persistent CTA-pair GEMMs.
namespace {
std::atomic<int> g_gemm_schedule{PTXSTD_SCHEDULE_PERSISTENT};
}  // namespace

extern "C" int ptxstd_set_gemm_schedule(int schedule) {
    if (schedule != PTXSTD_SCHEDULE_PERSISTENT && schedule != PTXSTD_SCHEDULE_DYNAMIC)
        return PTXSTD_EINVAL;
    g_gemm_schedule.store(schedule);
    return PTXSTD_OK;
}

extern "C" int ptxstd_get_gemm_schedule(void) { return g_gemm_schedule.load(); }

extern "C" int ptxstd_gemm_nvfp4(const uint8_t* d_a, const uint8_t* d_sfa, float ga,
                                 const uint8_t* d_b, const uint8_t* d_sfb, float gb,
                                 uint16_t* d_c, int64_t M, int64_t N, int64_t K,
                                 ptxstd_stream stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M % BM || N % BN || K % BK) return PTXSTD_EINVAL;
    if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return PTXSTD_EINVAL;
    if (!d_a || !d_b || !d_c || !d_sfa || !d_sfb || !ptxstd::aligned16(d_a) ||
        !ptxstd::aligned16(d_b) || !ptxstd::aligned16(d_c) || !ptxstd::aligned16(d_sfa) ||
        !ptxstd::aligned16(d_sfb))
        return PTXSTD_EINVAL;
    if (M % P_BM == 0 && N % P_BN == 0)
        return launch_pair(d_a, d_sfa, d_b, d_sfb, d_c, M, N, K, ga * gb,
                           static_cast<cudaStream_t>(stream));
    CUtensorMap ta, tb;
    int st = ptxstd::make_tmap_2d(&ta, d_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, M, K / 2, BKB,
                                  BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tb, d_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2, BKB, BN,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_nvfp4_kernel),
                                      static_cast<int>(kSmemBytes));
    if (st) return st;
    const uint32_t tiles = static_cast<uint32_t>((M / BM) * (N / BN));
    const uint32_t sms = static_cast<uint32_t>(ptxstd::sm_count());
    const uint32_t grid = tiles < sms ? tiles : sms;
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    gemm_nvfp4_kernel<<<grid, kThreads, kSmemBytes, static_cast<cudaStream_t>(stream)>>>(
        ta, tb, d_sfa, d_sfb, d_c, static_cast<uint32_t>(M), static_cast<uint32_t>(N),
        static_cast<uint32_t>(K), ga * gb, err);
    return ptxstd::launch_status();
}

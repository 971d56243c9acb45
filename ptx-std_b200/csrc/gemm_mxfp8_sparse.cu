// 2:4-sparse MXFP8 GEMM on the 5th-generation tensor cores, and the 2:4 pruning that feeds it.
//
//   C[M, N] (bf16) = sum_k (A[m,k] 2^(sfA[m,k/64]-127)) (B[n,k] 2^(sfB[n,k/64]-127))
// A is 2:4 structured-sparse: in each group of four consecutive K elements at most two are
// non-zero. It is given compressed, as vals [M, K/2] (the kept E4M3 codes in index order) and
// meta [M, K/8] (one nibble per group, i0 | i1 << 2 with i0 < i1 the kept positions, group g in
// the low nibble of byte g/2 for even g). B [N, K] is dense E4M3. The scales are UE8M0, one per 64
// logical K elements of each operand, in the blocked 128x4 layout (one 512-byte tile per 128
// rows and 256 K). One scale per 64 is what tcgen05.mma.sp.kind::mxf8f6f4.block_scale.block32
// applies: an MMA covers 64 logical K (32 stored A elements) and takes the single scale byte its
// scale-factor id selects.
//
// tcgen05.mma.sp.cta_group::2.kind::mxf8f6f4.block_scale.block32 is the reference's
// mma_block_scaled_sparse with MmaKind::Mxf8f6f4 (src/tcgen05/mma.rs:725-777) and
// InstrDescriptor::<Mxf8f6f4>::new(..).with_sparsity(Sparsity::Sparse)
// (src/tcgen05/descriptor.rs:265-278, :500-506).
//
// A cluster of two CTAs computes a 256 x 256 tile; per 256-element logical K stage CTA r loads:
//   - its 128 rows of vals (128 bytes per row, one 16 KiB TMA box, 128-byte swizzle);
//   - its 128 rows of B (256 bytes per row, two 16 KiB boxes);
//   - its 128 rows of metadata (32 bytes per row, two 16-byte-wide boxes = 2 x 2 KiB, rows of
//     16 bytes, the source layout of tcgen05.cp.128x128b);
//   - one SFA tile (its rows) and two SFB tiles (all 256 columns).
// The leader copies the metadata into TMEM with tcgen05.cp.cta_group::2.128x128b (row i of each
// CTA's 16-byte chunk to lane i, 4 columns; a lane's bits are its row's nibbles in order, so
// MMA j of the stage finds its 64 logical K at column 2 j) and the scales with 32x128b.warpx4,
// then issues the stage's four K = 64 MMAs with scale ids j.
#include "common.cuh"
#include "data_types.cuh"
#include "epilogue.cuh"
#include "tcgen05.cuh"
#include "tma_host.h"

namespace {

namespace t5 = ptxstd::tcgen05;
namespace dt = ptxstd::data_types;
using ptxstd::mbar_wait;

constexpr uint32_t P_BM = 256, P_BN = 256, P_HALF = 128;
constexpr uint32_t BKL = 256;           // logical K elements per stage
constexpr uint32_t kMmaK = 64;          // logical K of one sparse MMA
constexpr uint32_t kMmas = BKL / kMmaK; // 4
constexpr uint32_t STAGES = 4;
constexpr uint32_t kEpiWarps = 8;
constexpr uint32_t kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kABytes = P_HALF * BKL / 2;        // 16 KiB of compressed values
constexpr uint32_t kBBoxBytes = P_HALF * 128;         // 16 KiB: 128 K bytes of 128 rows
constexpr uint32_t kBBytes = 2 * kBBoxBytes;          // 256 K
constexpr uint32_t kMetaChunkBytes = P_HALF * 16;     // 128 rows x 16 bytes (128 logical K)
constexpr uint32_t kMetaBytes = 2 * kMetaChunkBytes;
constexpr uint32_t kSfaBytes = 512;
constexpr uint32_t kSfbBytes = (P_BN / 128) * 512;
constexpr uint32_t kCtaStageBytes = kABytes + kBBytes + kMetaBytes + kSfaBytes + kSfbBytes;
constexpr uint32_t kAccCols = P_BN;
// per-stage TMEM slot: metadata 8 columns, SFA 4, SFB 8
constexpr uint32_t kMetaCols = 8, kSfaCol = 8, kSfbCol = 12, kSlotCols = 20;
static_assert(kMetaCols == kSfaCol && kSfbCol + 4 * (P_BN / 128) == kSlotCols, "slot layout");
constexpr uint32_t kSfBase = kAccCols;
constexpr uint32_t kTmemCols = 512;
static_assert(kSfBase + STAGES * kSlotCols <= kTmemCols, "TMEM budget");
static_assert(kSlotCols % 4 == 0, "metadata and scale slots start on 4-column boundaries");
// Grouped raster of kGroupM row-tiles; 16 measured 2-4 % ahead of 8 at 8192^3 (five interleaved
// repetitions each on one B200, bit-identical output).
constexpr uint32_t kGroupM = 16;
// Epilogue stores: 16 bf16 columns (32-byte row segments, whole L2 sectors) per TMA store, so that
// the 1 KiB staging buffers of the eight epilogue warps fit beside the four 53.5 KiB stages.
constexpr uint32_t kCCols = 16;

struct alignas(1024) Smem {
    uint8_t a[STAGES][kABytes];
    uint8_t b[STAGES][2][kBBoxBytes];
    uint8_t meta[STAGES][2][kMetaChunkBytes];
    uint8_t sfa[STAGES][kSfaBytes];
    uint8_t sfb[STAGES][kSfbBytes];
    uint8_t cstage[kEpiWarps][ptxstd::epi::Box<kCCols>::kBytes];  // epilogue staging per warp
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull;
    uint64_t tempty;  // leader's: one arrive per epilogue warp of both CTAs
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum : uint32_t { kDetailProducer = 0x1900, kDetailMma = 0x1A00, kDetailEpilogue = 0x1B00 };

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
    gemm_mxfp8_sparse_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                                  const __grid_constant__ CUtensorMap tmMeta,
                                  const __grid_constant__ CUtensorMap tmB,
                                  const __grid_constant__ CUtensorMap tmSfa,
                                  const __grid_constant__ CUtensorMap tmSfb,
                                  const __grid_constant__ CUtensorMap tmC, uint32_t M, uint32_t N,
                                  uint32_t K, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t rank = ptxstd::cluster_ctarank();
    const uint32_t pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const uint32_t num_m = M / P_BM, num_n = N / P_BN, num_tiles = num_m * num_n;
    const uint32_t num_k = K / BKL;
    const uint32_t sf_tiles_per_row = K / 256;  // 512-byte scale tiles per 128-row block

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmA);
        ptxstd::prefetch_tensormap(&tmMeta);
        ptxstd::prefetch_tensormap(&tmB);
        ptxstd::prefetch_tensormap(&tmSfa);
        ptxstd::prefetch_tensormap(&tmSfb);
        ptxstd::prefetch_tensormap(&tmC);
        for (uint32_t i = 0; i < STAGES; ++i) {
            ptxstd::mbar_init(&s.full[i], 1);
            ptxstd::mbar_init(&s.empty[i], 1);
        }
        ptxstd::mbar_init(&s.tfull, 1);
        ptxstd::mbar_init(&s.tempty, 2 * kEpiWarps);
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
            for (uint32_t t = pair; t < num_tiles && !aborted(s); t += n_pairs) {
                uint32_t mb, nb;
                tile_coords(t, num_m, num_n, mb, nb);
                const int32_t arow = static_cast<int32_t>(mb * P_BM + rank * P_HALF);
                const int32_t brow = static_cast<int32_t>(nb * P_BN + rank * P_HALF);
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.empty[stage], phase ^ 1u)) {
                        fail(s, err, kDetailProducer | stage);
                        break;
                    }
                    if (aborted(s)) break;
                    const uint32_t fl = ptxstd::mapa_shared(ptxstd::smem_u32(&s.full[stage]), 0);
                    if (rank == 0) ptxstd::mbar_arrive_expect_tx(&s.full[stage], 2 * kCtaStageBytes);
                    ptxstd::tma_load_2d_pair(s.a[stage], &tmA, fl,
                                             static_cast<int32_t>(kb * (BKL / 2)), arow);
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h) {
                        ptxstd::tma_load_2d_pair(s.b[stage][h], &tmB, fl,
                                                 static_cast<int32_t>(kb * BKL + 128 * h), brow);
                        ptxstd::tma_load_2d_pair(s.meta[stage][h], &tmMeta, fl,
                                                 static_cast<int32_t>(kb * (BKL / 8) + 16 * h),
                                                 arow);
                    }
                    ptxstd::tma_load_2d_pair(
                        s.sfa[stage], &tmSfa, fl, 0,
                        static_cast<int32_t>((mb * 2 + rank) * sf_tiles_per_row + kb));
#pragma unroll
                    for (uint32_t j = 0; j < P_BN / 128; ++j)
                        ptxstd::tma_load_2d_pair(
                            s.sfb[stage] + j * 512, &tmSfb, fl, 0,
                            static_cast<int32_t>((nb * 2 + j) * sf_tiles_per_row + kb));
                    issued |= 1u << stage;
                    issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            if (aborted(s) && rank == 0) {
                for (uint32_t i = 0; i < STAGES; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.full[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer (leader) ----------------
        if (rank == 0 && ptxstd::elect_one()) {
            uint32_t idesc0 = 0;
            t5::idesc_mxf8f6f4(/*E4m3*/ 0, /*E4m3*/ 0, P_BM, P_BN, idesc0);
            t5::idesc_with_field(idesc0, 2, 1, 1, idesc0);  // Sparsity::Sparse
            uint32_t idesc[kMmas];
#pragma unroll
            for (uint32_t j = 0; j < kMmas; ++j) {
                uint32_t t0 = 0;
                t5::idesc_with_field(idesc0, 29, 2, j, t0);  // scale-factor A id
                t5::idesc_with_field(t0, 4, 2, j, idesc[j]);  // scale-factor B id
            }
            uint32_t stage = 0, phase = 0, acc_phase = 0;
            for (uint32_t t = pair; t < num_tiles && !aborted(s); t += n_pairs) {
                if (!mbar_wait(&s.tempty, acc_phase ^ 1u)) {
                    fail(s, err, kDetailMma | 0x90);
                    break;
                }
                t5::fence_after_thread_sync();
                bool ok = true;
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.full[stage], phase)) {
                        fail(s, err, kDetailMma | 0x80 | stage);
                        ok = false;
                        break;
                    }
                    t5::fence_after_thread_sync();
                    const uint32_t slot = tmem + kSfBase + stage * kSlotCols;
#pragma unroll
                    for (uint32_t h = 0; h < 2; ++h)
                        t5::cp_128x128b_pair(
                            slot + 4 * h,
                            t5::smem_desc_nosw(ptxstd::smem_u32(s.meta[stage][h]), 0, 128));
                    t5::cp_32x128b_warpx4_pair(
                        slot + kSfaCol, t5::smem_desc_nosw(ptxstd::smem_u32(s.sfa[stage]), 0, 128));
#pragma unroll
                    for (uint32_t h = 0; h < P_BN / 128; ++h)
                        t5::cp_32x128b_warpx4_pair(
                            slot + kSfbCol + 4 * h,
                            t5::smem_desc_nosw(ptxstd::smem_u32(s.sfb[stage] + 512 * h), 0, 128));
                    const uint64_t ad = t5::smem_desc_k128(ptxstd::smem_u32(s.a[stage]));
#pragma unroll
                    for (uint32_t j = 0; j < kMmas; ++j) {
                        // vals: 32 bytes per MMA; B: 64 bytes per MMA, two MMAs per 128-byte box
                        const uint64_t bd =
                            t5::smem_desc_k128(ptxstd::smem_u32(s.b[stage][j >> 1])) + 4 * (j & 1);
                        t5::mma_sp_mxf8f6f4_block32_pair(tmem, ad + 2 * j, bd, slot + 2 * j,
                                                         idesc[j], slot + kSfaCol,
                                                         slot + kSfbCol, (kb | j) != 0u);
                    }
                    const uint32_t e = ptxstd::smem_u32(&s.empty[stage]);
                    t5::commit_pair(e);
                    t5::commit_pair(ptxstd::mapa_shared(e, 1));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                const uint32_t f = ptxstd::smem_u32(&s.tfull);
                t5::commit_pair(f);
                t5::commit_pair(ptxstd::mapa_shared(f, 1));
                acc_phase ^= 1u;
            }
            t5::commit_pair(ptxstd::smem_u32(&s.drain));
            mbar_wait(&s.drain, 0);
        }
    } else {
        // ---------------- epilogue: warps 2..9 of both CTAs ----------------
        const uint32_t q = warp & 3u;
        const uint32_t half = (warp - 2u) >> 2;
        uint32_t acc_phase = 0;
        const uint32_t tempty_leader = ptxstd::mapa_shared(ptxstd::smem_u32(&s.tempty), 0);
        const uint32_t stg = ptxstd::smem_u32(s.cstage[warp - 2u]);
        for (uint32_t t = pair; t < num_tiles; t += n_pairs) {
            bool ok = !aborted(s) && mbar_wait(&s.tfull, acc_phase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !aborted(s)) fail(s, err, kDetailEpilogue | 0x80);
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
            const int32_t row0 = static_cast<int32_t>(mb * P_BM + rank * P_HALF + 32 * q);
            const int32_t col0 = static_cast<int32_t>(nb * P_BN + half * 128);
            ptxstd::epi::store_row_block<kCCols>(&tmC, stg, r, 1.0f, col0, row0, lane);
        }
        ptxstd::epi::drain(lane);
    }

    t5::fence_before_thread_sync();
    ptxstd::cluster_sync();  // neither CTA of the pair leaves while the other may still use it
    t5::fence_after_thread_sync();
    if (warp == 1) t5::tmem_dealloc_pair(tmem, kTmemCols);
}

// 2:4 pruning: each thread takes 8 codes (two groups) of a row -> 4 kept codes, 1 metadata byte.
// Magnitude = code & 0x7F (E4M3 codes order like their magnitudes); ties to the lower index.
__device__ __forceinline__ uint32_t prune_group(uint32_t q4, uint32_t& kept) {
    uint32_t mag[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) mag[i] = (q4 >> (8 * i)) & 0x7Fu;
    uint32_t best = 0;
#pragma unroll
    for (uint32_t i = 1; i < 4; ++i)
        if (mag[i] > mag[best]) best = i;
    uint32_t second = best == 0 ? 1 : 0;
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i)
        if (i != best && mag[i] > mag[second]) second = i;
    const uint32_t i0 = min(best, second), i1 = max(best, second);
    kept = ((q4 >> (8 * i0)) & 0xFFu) | (((q4 >> (8 * i1)) & 0xFFu) << 8);
    return i0 | (i1 << 2);
}

__global__ void __launch_bounds__(256) prune_24_kernel(const uint8_t* __restrict__ codes,
                                                        uint8_t* __restrict__ vals,
                                                        uint8_t* __restrict__ meta, size_t n8) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
         i += stride) {
        const uint2 q = reinterpret_cast<const uint2*>(codes)[i];
        uint32_t k0, k1;
        const uint32_t m0 = prune_group(q.x, k0), m1 = prune_group(q.y, k1);
        reinterpret_cast<uint32_t*>(vals)[i] = k0 | (k1 << 16);
        meta[i] = static_cast<uint8_t>(m0 | (m1 << 4));
    }
}

}  // namespace

extern "C" int ptxstd_prune_24_e4m3(const uint8_t* d_codes, int64_t rows, int64_t cols,
                                    uint8_t* d_vals, uint8_t* d_meta, ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 8 != 0) return PTXSTD_EINVAL;
    if (!d_codes || !d_vals || !d_meta || (reinterpret_cast<uintptr_t>(d_codes) & 7) ||
        (reinterpret_cast<uintptr_t>(d_vals) & 3))
        return PTXSTD_EINVAL;
    const size_t n8 = static_cast<size_t>(rows) * static_cast<size_t>(cols) / 8;
    const size_t blocks = (n8 + 255) / 256;
    const size_t cap = static_cast<size_t>(ptxstd::sm_count()) * 8;
    prune_24_kernel<<<static_cast<int>(blocks < cap ? blocks : cap), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(d_codes, d_vals, d_meta, n8);
    return ptxstd::launch_status();
}

extern "C" int ptxstd_gemm_mxfp8_sparse(const uint8_t* d_vals, const uint8_t* d_meta,
                                        const uint8_t* d_sfa, const uint8_t* d_b,
                                        const uint8_t* d_sfb, uint16_t* d_c, int64_t M, int64_t N,
                                        int64_t K, ptxstd_stream stream) {
    if (M <= 0 || N <= 0 || K <= 0 || M % P_BM || N % P_BN || K % BKL) return PTXSTD_EINVAL;
    if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return PTXSTD_EINVAL;
    if (!d_vals || !d_meta || !d_b || !d_c || !d_sfa || !d_sfb || !ptxstd::aligned16(d_vals) ||
        !ptxstd::aligned16(d_meta) || !ptxstd::aligned16(d_b) || !ptxstd::aligned16(d_c) ||
        !ptxstd::aligned16(d_sfa) || !ptxstd::aligned16(d_sfb))
        return PTXSTD_EINVAL;
    CUtensorMap ta, tm, tb, tsa, tsb, tc;
    int st = ptxstd::make_tmap_2d(&ta, d_vals, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, M, K / 2,
                                  BKL / 2, P_HALF, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tm, d_meta, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 8, M, K / 8, 16,
                              P_HALF, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tb, d_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, 128, P_HALF,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // blocked scales as u32 [tiles, 128]: one row per 512-byte tile (128 rows x 256 K)
    st = ptxstd::make_tmap_2d(&tsa, d_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128,
                              (M / 128) * (K / 256), 512, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tsb, d_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128,
                              (N / 128) * (K / 256), 512, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::epi::make_store_map<kCCols>(&tc, d_c, M, N);
    if (st) return st;
    st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_mxfp8_sparse_pair_kernel),
                                      static_cast<int>(kSmemBytes));
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
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int max_pairs[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PTXSTD_ECUDA;
    if (max_pairs[dev] == 0) {
        cfg.gridDim = dim3(2 * static_cast<uint32_t>(ptxstd::sm_count() / 2));
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm_mxfp8_sparse_pair_kernel, &cfg) !=
                cudaSuccess ||
            clusters <= 0)
            return PTXSTD_ECUDA;
        max_pairs[dev] = clusters;
    }
    const uint32_t tiles = static_cast<uint32_t>((M / P_BM) * (N / P_BN));
    const uint32_t pairs =
        tiles < static_cast<uint32_t>(max_pairs[dev]) ? tiles : static_cast<uint32_t>(max_pairs[dev]);
    cfg.gridDim = dim3(2 * pairs);
    if (cudaLaunchKernelEx(&cfg, gemm_mxfp8_sparse_pair_kernel, ta, tm, tb, tsa, tsb, tc,
                           static_cast<uint32_t>(M), static_cast<uint32_t>(N),
                           static_cast<uint32_t>(K), err) != cudaSuccess)
        return PTXSTD_ECUDA;
    return ptxstd::launch_status();
}

// MXFP8 block-scaled GEMM (OCP MX: E4M3 elements, one UE8M0 scale per 32 K elements) on the
// 5th-generation tensor cores:
//   C[M, N] (bf16) = sum_k (A[m,k] 2^(sfA[m,k/32]-127)) (B[n,k] 2^(sfB[n,k/32]-127))
// A [M, K] and B [N, K] E4M3 with K contiguous; scales in the blocked 128x4 layout, i.e. the
// output of ptxstd_quantize_mxfp8_layout with sf_layout 1, so a quantised activation feeds the GEMM
// without a relayout; fp32 accumulation and bf16 RN output.
// tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale.block32: the reference's mma_block_scaled
// with MmaKind::Mxf8f6f4 and ScaleVectorSize::Block32 (src/tcgen05/mma.rs:58-97, :698-724), and
// InstrDescriptor::<Mxf8f6f4>::new(E4m3, E4m3, 256, 256) with its scale-factor ids
// (src/tcgen05/descriptor.rs:601-611, :660-813).
//
// ptxstd_gemm_mx runs the same kernel for any pair of kind::mxf8f6f4 element types (E4M3, E5M2,
// E2M3, E3M2, E2M1; A and B may differ), set in the instruction descriptor. For K = 32 MMAs the
// 4- and 6-bit types take one byte per element in shared memory (16-element groups padded to 16
// bytes, src/tcgen05/descriptor.rs:306-315), so the tiles, TMA boxes and shared-memory
// descriptors are those of FP8; operands come in that padded layout, as ptxstd_quantize_mx
// writes it.
//
// A cluster of two CTAs computes a 256 x 256 tile. CTA r loads A rows [128 r, +128) and B rows
// [128 r, +128) of the tile, A's scales for its rows and B's scales for all 256 columns (each
// CTA accumulates all N columns of its rows), everything completing on the leader's `full`
// barrier. Per 128-element K stage that is 16 KiB of A, 16 KiB of B and three 512-byte scale
// tiles: in the blocked layout one tile holds the 4 scales (128 K elements) of 128 rows, so one
// tile per 128 rows and stage. The leader moves the tiles to TMEM with
// tcgen05.cp.cta_group::2.32x128b.warpx4 (each CTA from its own smem to its own TMEM) and issues
// the stage's four K=32 MMAs; MMA j reads scale byte j of the same TMEM words, selected by the
// instruction descriptor's scale-factor ids. Scale slots in TMEM are per stage, so a slot is
// rewritten only after the stage's `empty` barrier has observed the MMAs that read it.
//
// TMEM: one 256-column f32 accumulator plus 6 stages x 12 scale columns. Two accumulators
// (512 columns) would leave no room for the scales, so eight epilogue warps (two per lane quarter,
// 128 columns each) copy the accumulator to registers and release it before converting and
// storing. The bf16 tile leaves through a swizzled staging buffer per warp and TMA tile stores
// of 32 rows x 32 columns (epilogue.cuh).
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
constexpr uint32_t BK = 128;            // K elements (= bytes) per stage
constexpr uint32_t kMmaK = 32;          // K elements of one mxf8f6f4 MMA
constexpr uint32_t kMmas = BK / kMmaK;  // 4 per stage, one scale byte each
constexpr uint32_t STAGES = 6;
constexpr uint32_t kEpiWarps = 8;
constexpr uint32_t kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kABytes = P_HALF * BK;                 // 16 KiB
constexpr uint32_t kBBytes = P_HALF * BK;                 // 16 KiB
constexpr uint32_t kSfaBytes = 512;                       // this CTA's 128 rows
constexpr uint32_t kSfbBytes = (P_BN / 128) * 512;        // all 256 columns
constexpr uint32_t kCtaStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;
constexpr uint32_t kAccCols = P_BN;
constexpr uint32_t kSlotCols = 4 + 4 * (P_BN / 128);      // SFA 4 columns, SFB 8
constexpr uint32_t kSfBase = kAccCols;
constexpr uint32_t kTmemCols = 512;
static_assert(kSfBase + STAGES * kSlotCols <= kTmemCols, "TMEM budget");
constexpr uint32_t kGroupM = 8;
// Epilogue stores: 32 bf16 columns (64-byte row segments) per TMA store, so that the 2 KiB
// staging buffers of the eight epilogue warps fit beside six stages.
constexpr uint32_t kCCols = 32;

struct alignas(1024) Smem {
    uint8_t a[STAGES][kABytes];
    uint8_t b[STAGES][kBBytes];
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

enum : uint32_t { kDetailProducer = 0x1500, kDetailMma = 0x1600, kDetailEpilogue = 0x1700 };

// Grouped raster: kGroupM row-tiles sweep all column-tiles before moving on (L2 reuse of B).
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

// mma_block_scaled::<Two, Mxf8f6f4, Block32>: D[tmem] (+)= (A . SFA) (B . SFB)^T, M = 256 over the
// pair, scales read from TMEM at [sfa], [sfb] (byte chosen by the descriptor's scale ids).
__device__ __forceinline__ void mma_mxf8f6f4_block32_pair(uint32_t d_tmem, uint64_t a_desc,
                                                          uint64_t b_desc, uint32_t idesc,
                                                          uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale.block32 [%0], %1, %2, %3, [%4], "
        "[%5], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
        : "memory");
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_mxfp8_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                           const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmSfa,
                           const __grid_constant__ CUtensorMap tmSfb,
                           const __grid_constant__ CUtensorMap tmC, uint32_t M, uint32_t N,
                           uint32_t K, uint32_t atype, uint32_t btype, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t rank = ptxstd::cluster_ctarank();
    const uint32_t pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
    const uint32_t num_m = M / P_BM, num_n = N / P_BN, num_tiles = num_m * num_n, num_k = K / BK;
    const uint32_t sf_tiles_per_row = K / 128;  // 512-byte scale tiles per 128-row block

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmA);
        ptxstd::prefetch_tensormap(&tmB);
        ptxstd::prefetch_tensormap(&tmC);
        ptxstd::prefetch_tensormap(&tmSfa);
        ptxstd::prefetch_tensormap(&tmSfb);
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
                for (uint32_t kb = 0; kb < num_k; ++kb) {
                    if (!mbar_wait(&s.empty[stage], phase ^ 1u)) {
                        fail(s, err, kDetailProducer | stage);
                        break;
                    }
                    if (aborted(s)) break;
                    const uint32_t fl = ptxstd::mapa_shared(ptxstd::smem_u32(&s.full[stage]), 0);
                    if (rank == 0) ptxstd::mbar_arrive_expect_tx(&s.full[stage], 2 * kCtaStageBytes);
                    ptxstd::tma_load_2d_pair(s.a[stage], &tmA, fl, static_cast<int32_t>(kb * BK),
                                             static_cast<int32_t>(mb * P_BM + rank * P_HALF));
                    ptxstd::tma_load_2d_pair(s.b[stage], &tmB, fl, static_cast<int32_t>(kb * BK),
                                             static_cast<int32_t>(nb * P_BN + rank * P_HALF));
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
            t5::idesc_mxf8f6f4(atype, btype, P_BM, P_BN, idesc0);
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
                    const uint64_t ad = t5::smem_desc_k128(ptxstd::smem_u32(s.a[stage]));
                    const uint64_t bd = t5::smem_desc_k128(ptxstd::smem_u32(s.b[stage]));
                    const uint32_t slot = tmem + kSfBase + stage * kSlotCols;
                    t5::cp_32x128b_warpx4_pair(
                        slot, t5::smem_desc_nosw(ptxstd::smem_u32(s.sfa[stage]), 0, 128));
#pragma unroll
                    for (uint32_t h = 0; h < P_BN / 128; ++h)
                        t5::cp_32x128b_warpx4_pair(
                            slot + 4 + 4 * h,
                            t5::smem_desc_nosw(ptxstd::smem_u32(s.sfb[stage] + 512 * h), 0, 128));
#pragma unroll
                    for (uint32_t j = 0; j < kMmas; ++j)
                        mma_mxf8f6f4_block32_pair(tmem, ad + 2 * j, bd + 2 * j, idesc[j], slot,
                                                  slot + 4, (kb | j) != 0u);
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

}  // namespace

namespace {
bool mx_type_ok(int t) { return t == 0 || t == 1 || t == 3 || t == 4 || t == 5; }
}  // namespace

extern "C" int ptxstd_gemm_mx(const uint8_t* d_a, int a_type, const uint8_t* d_sfa,
                              const uint8_t* d_b, int b_type, const uint8_t* d_sfb, uint16_t* d_c,
                              int64_t M, int64_t N, int64_t K, ptxstd_stream stream) {
    if (!mx_type_ok(a_type) || !mx_type_ok(b_type)) return PTXSTD_EINVAL;
    if (M <= 0 || N <= 0 || K <= 0 || M % P_BM || N % P_BN || K % BK) return PTXSTD_EINVAL;
    if (M >= (1ll << 31) || N >= (1ll << 31) || K >= (1ll << 31)) return PTXSTD_EINVAL;
    if (!d_a || !d_b || !d_c || !d_sfa || !d_sfb || !ptxstd::aligned16(d_a) ||
        !ptxstd::aligned16(d_b) || !ptxstd::aligned16(d_c) || !ptxstd::aligned16(d_sfa) ||
        !ptxstd::aligned16(d_sfb))
        return PTXSTD_EINVAL;
    CUtensorMap ta, tb, tsa, tsb, tc;
    int st = ptxstd::make_tmap_2d(&ta, d_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, M, K, BK, P_HALF,
                                  CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tb, d_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, K, N, K, BK, P_HALF,
                              CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    // blocked scales as u32 [tiles, 128]: one row per 512-byte tile, one tile per box
    st = ptxstd::make_tmap_2d(&tsa, d_sfa, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128,
                              (M / 128) * (K / 128), 512, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::make_tmap_2d(&tsb, d_sfb, CU_TENSOR_MAP_DATA_TYPE_UINT32, 128,
                              (N / 128) * (K / 128), 512, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    st = ptxstd::epi::make_store_map<kCCols>(&tc, d_c, M, N);
    if (st) return st;
    st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_mxfp8_pair_kernel),
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
    // as many pairs as can be resident at once (a persistent grid), but no more than tiles
    static int max_pairs[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PTXSTD_ECUDA;
    if (max_pairs[dev] == 0) {
        cfg.gridDim = dim3(2 * static_cast<uint32_t>(ptxstd::sm_count() / 2));
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, gemm_mxfp8_pair_kernel, &cfg) !=
                cudaSuccess ||
            clusters <= 0)
            return PTXSTD_ECUDA;
        max_pairs[dev] = clusters;
    }
    const uint32_t tiles = static_cast<uint32_t>((M / P_BM) * (N / P_BN));
    const uint32_t pairs =
        tiles < static_cast<uint32_t>(max_pairs[dev]) ? tiles : static_cast<uint32_t>(max_pairs[dev]);
    cfg.gridDim = dim3(2 * pairs);
    if (cudaLaunchKernelEx(&cfg, gemm_mxfp8_pair_kernel, ta, tb, tsa, tsb, tc,
                           static_cast<uint32_t>(M), static_cast<uint32_t>(N),
                           static_cast<uint32_t>(K), static_cast<uint32_t>(a_type),
                           static_cast<uint32_t>(b_type), err) != cudaSuccess)
        return PTXSTD_ECUDA;
    return ptxstd::launch_status();
}

extern "C" int ptxstd_gemm_mxfp8(const uint8_t* d_a, const uint8_t* d_sfa, const uint8_t* d_b,
                                 const uint8_t* d_sfb, uint16_t* d_c, int64_t M, int64_t N,
                                 int64_t K, ptxstd_stream stream) {
    return ptxstd_gemm_mx(d_a, 0, d_sfa, d_b, 0, d_sfb, d_c, M, N, K, stream);
}

// Quantise/pack kernels: bf16 activations -> MXFP8 (E4M3 + UE8M0 per 32) and NVFP4 (E2M1 + E4M3
// per 16, f32 global scale). HBM-bound, so the kernel is built around bytes in flight:
//
//   - a persistent grid of one CTA per SM walks fixed-size chunks of the flat input;
//   - one producer lane streams each chunk into a multi-stage shared-memory ring with a 1-D bulk
//     async copy (cp.async.bulk, ptx-std src/tma/bulk.rs:60) that completes on the stage's
//     mbarrier (arrive_expect_tx, src/mbarrier.rs:533) — 128 KiB in flight per SM by default,
//     with no register cost;
//   - CW consumer warps read the stage with 16-byte shared loads, lane l of warp w taking
//     vector (w * 32 + l) of each (32 CW)-vector row so that every warp load is one contiguous,
//     conflict-free 512-byte row; the lanes holding one block (4 for MXFP8, 2 for NVFP4) combine
//     their amax with shuffle-xor; each element pair is packed by one `cvt` instruction
//     (src/data_types/narrow.rs:156-162); payload words go straight to global memory as 8-byte
//     (MXFP8) or 4-byte (NVFP4) stores, so a warp store covers 256 / 128 contiguous bytes;
//   - consumers release a stage with one arrive per warp on its `empty` barrier.
//
// The stochastic-rounding forms (Mxfp8Rs, Nvfp4Rs) keep the scale recipe and round the elements
// with cvt.rs (narrow.rs:217-229); the random bits of vector v (elements 8 v .. 8 v + 7, two
// groups of four) are both words of SplitMix64 output v of the caller's seed, so no random bits
// are read from memory.
//
// Every wait is bounded; a timeout records PTXSTD_ETIMEOUT, and the producer drains its copies
// before the CTA exits.
#include "common.cuh"
#include "data_types.cuh"

namespace dt = ptxstd::data_types;
using ptxstd::mbar_wait;

namespace {

// Tiling of the ring: CW consumer warps, VPL 16-byte vectors per lane per stage, ST stages.
template <uint32_t CW, uint32_t VPL, uint32_t ST>
struct QCfg {
    static constexpr uint32_t kConsumerWarps = CW;
    static constexpr uint32_t kVecsPerLane = VPL;
    static constexpr uint32_t kStages = ST;
    static constexpr uint32_t kChunkVecs = 32 * CW * VPL;  // 16-byte vectors per stage
    static constexpr uint32_t kChunkElems = kChunkVecs * 8;
    static constexpr uint32_t kChunkBytes = kChunkVecs * 16;
    static constexpr uint32_t kThreads = 32 * (CW + 1);
    struct alignas(128) Smem {
        uint8_t buf[ST][kChunkBytes];
        uint64_t full[ST];
        uint64_t empty[ST];
        uint32_t abort;
    };
    static constexpr size_t kSmemBytes = sizeof(Smem) + 128;
};
// Default: 24 consumer warps x 2 vectors per lane = 24 KiB stages, 6 stages (144 KiB in flight
// per SM). Best of a sweep on B200 at 8192 x 8192 (35.1 us vs 36.8 for 16x2x8, 35.9 for 16x4x4,
// 45.4 for 8x4x8): with ~10 instructions per element the consumers need enough warps per
// scheduler to hide latency, and the ring supplies the bytes in flight. A later sweep at the same
// size (MXFP8, GB/s over five interleaved runs) kept it: 24x2x6 6061-6138, 16x4x4 6072-6092,
// 28x2x6 5989-6022, 24x2x7 5906-5993, 24x4x3 5883-5922, 24x2x8 5814-5897.
using DefaultCfg = QCfg<24, 2, 6>;

enum : uint32_t { kDetailProducer = 0x2100, kDetailConsumer = 0x2200 };

// Offset of scale (r, s) in the blocked "128x4" layout consumed by the block-scaled GEMMs: tiles
// of 128 rows x 4 scale columns stored as 512 contiguous bytes, row-tile major; inside a tile the
// scale of row r, column s sits at (r % 32) * 16 + ((r / 32) % 4) * 4 + s % 4, which is the
// 32-lane x 16-byte source of one tcgen05.cp.32x128b.warpx4 (src/tcgen05/copy.rs:29-30).
__device__ __forceinline__ size_t blocked_sf_offset(size_t r, size_t s, size_t sf_cols) {
    const size_t tile = (r >> 7) * (sf_cols >> 2) + (s >> 2);
    return tile * 512 + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (s & 3);
}

template <bool BLOCKED>
__device__ __forceinline__ void store_scale(uint8_t* sf, size_t b, size_t sf_cols, uint32_t code) {
    if constexpr (BLOCKED)
        sf[blocked_sf_offset(b / sf_cols, b % sf_cols, sf_cols)] = static_cast<uint8_t>(code);
    else
        sf[b] = static_cast<uint8_t>(code);
}

// Per-vector work of the two formats. `w` holds 8 bf16; `gv` is the vector's flat index.
template <bool BLOCKED>
struct Mxfp8 {
    static constexpr uint32_t kLanesPerBlock = 4;  // 32 elements
    float six_g;  // unused
    __device__ __forceinline__ void operator()(const uint4 v, bool valid, size_t gv, uint32_t lane,
                                               uint8_t* q, uint8_t* sf, size_t sf_cols) const {
        uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v.x, v.y),
                                              dt::bf16x2_absmax_bits(v.z, v.w)));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const uint32_t code = dt::mxfp8_scale_code(__uint_as_float(m << 16));
        const float inv = dt::ue8m0_inverse(code);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t p[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = dt::bf16x2_mul_f32(w[k], inv);
            p[k] = dt::e4m3x2_from_f32<false>(f.x, f.y);
        }
        if (valid) {
            reinterpret_cast<uint2*>(q)[gv] = make_uint2(p[0] | (p[1] << 16), p[2] | (p[3] << 16));
            if ((lane & 3u) == 0) store_scale<BLOCKED>(sf, gv >> 2, sf_cols, code);
        }
    }
};

template <bool BLOCKED>
struct Nvfp4 {
    static constexpr uint32_t kLanesPerBlock = 2;  // 16 elements
    float g, six_g;
    __device__ __forceinline__ void operator()(const uint4 v, bool valid, size_t gv, uint32_t lane,
                                               uint8_t* q, uint8_t* sf, size_t sf_cols) const {
        uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v.x, v.y),
                                              dt::bf16x2_absmax_bits(v.z, v.w)));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        // sf = e4m3(amax / (6 g)); r = 1 / (sf * g), or 0 when that product is 0.
        const float s = __fdiv_rn(__uint_as_float(m << 16), six_g);
        const uint32_t code = dt::e4m3x2_from_f32<false>(s, 0.0f) & 0xFFu;
        const float t = __fmul_rn(dt::e4m3_to_f32(code), g);
        const float r = (t == 0.0f) ? 0.0f : __frcp_rn(t);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t packed = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 f = dt::bf16x2_mul_f32(w[k], r);
            packed |= dt::e2m1x2_from_f32<false>(f.x, f.y) << (8 * k);
        }
        if (valid) {
            reinterpret_cast<uint32_t*>(q)[gv] = packed;
            if ((lane & 1u) == 0) store_scale<BLOCKED>(sf, gv >> 1, sf_cols, code);
        }
    }
};

// OCP MX quantisation to any element type of kind::mxf8f6f4, named by its tcgen05 code T
// (F8f6f4ElementType, src/tcgen05/descriptor.rs:316-327): 0 E4M3, 1 E5M2, 3 E2M3, 4 E3M2,
// 5 E2M1. The scale is the MXFP8 recipe with the format's own emax (floor-pow2 of the block amax,
// TowardZero + SaturateFinite, minus emax, clamped at 0); the elements are RN .satfinite. The
// payload is written in the tensor cores' operand layout, one byte per element in memory
// (descriptor.rs:306-315): FP8 codes as they are; FP6 as groups of 16 six-bit codes packed
// little-endian into 12 bytes plus 4 zero bytes; FP4 as 16 nibbles in 8 bytes plus 8 zero bytes.
// A 16-element group is the vectors of two neighbouring lanes, so the even lane gathers the bits
// that spill into its 8 bytes from its partner with one shuffle.
template <bool BLOCKED, uint32_t T>
struct MxAny {
    static constexpr uint32_t kLanesPerBlock = 4;  // 32 elements
    static constexpr uint32_t kEmax = T == 0 ? 8u : T == 1 ? 15u : T == 4 ? 4u : 2u;
    float six_g;  // unused
    __device__ __forceinline__ void operator()(const uint4 v, bool valid, size_t gv, uint32_t lane,
                                               uint8_t* q, uint8_t* sf, size_t sf_cols) const {
        uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v.x, v.y),
                                              dt::bf16x2_absmax_bits(v.z, v.w)));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const uint32_t u = dt::ue8m0_from_f32<false, true>(__uint_as_float(m << 16));
        const uint32_t code = u == 0xFFu ? 0xFFu : (u > kEmax ? u - kEmax : 0u);
        const float inv = dt::ue8m0_inverse(code);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t lo, hi;  // this vector's 8 bytes of the payload
        if constexpr (T == 0 || T == 1) {
            uint32_t p[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = dt::bf16x2_mul_f32(w[k], inv);
                p[k] = T == 0 ? dt::e4m3x2_from_f32<false>(f.x, f.y)
                              : dt::e5m2x2_from_f32<false>(f.x, f.y);
            }
            lo = p[0] | (p[1] << 16);
            hi = p[2] | (p[3] << 16);
        } else if constexpr (T == 3 || T == 4) {
            uint64_t bits = 0;  // element i of the vector at bits 6i .. 6i+5
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = dt::bf16x2_mul_f32(w[k], inv);
                const uint32_t c2 = T == 3 ? dt::e2m3x2_from_f32<false>(f.x, f.y)
                                           : dt::e3m2x2_from_f32<false>(f.x, f.y);
                bits |= static_cast<uint64_t>(c2 & 0x3Fu) << (12 * k);
                bits |= static_cast<uint64_t>((c2 >> 8) & 0x3Fu) << (12 * k + 6);
            }
            const uint32_t b_lo = static_cast<uint32_t>(bits);
            const uint32_t b_hi = static_cast<uint32_t>(bits >> 32);  // bits 32 .. 47
            const uint32_t partner_lo = __shfl_xor_sync(0xffffffffu, b_lo, 1);
            if (lane & 1u) {
                // elements 8..15 hold group bits 48..95; bytes 8..15 = group bits 64..95 + pad
                lo = (b_lo >> 16) | (b_hi << 16);
                hi = 0u;
            } else {
                // bytes 0..7 = group bits 0..63: own 48 bits, then the partner's first 16
                lo = b_lo;
                hi = b_hi | (partner_lo << 16);
            }
        } else {
            uint32_t packed = 0;  // 8 nibbles, element 0 in the low nibble
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = dt::bf16x2_mul_f32(w[k], inv);
                packed |= dt::e2m1x2_from_f32<false>(f.x, f.y) << (8 * k);
            }
            const uint32_t partner = __shfl_xor_sync(0xffffffffu, packed, 1);
            lo = (lane & 1u) ? 0u : packed;
            hi = (lane & 1u) ? 0u : partner;
        }
        if (valid) {
            reinterpret_cast<uint2*>(q)[gv] = make_uint2(lo, hi);
            if ((lane & 3u) == 0) store_scale<BLOCKED>(sf, gv >> 2, sf_cols, code);
        }
    }
};

template <uint32_t T>
int launch_mx(const uint16_t* x, size_t n, uint8_t* q, uint8_t* sf, size_t sf_cols, int blocked,
              cudaStream_t s);

// Stochastic-rounding MXFP8: the same scale; elements 8 gv .. 8 gv + 3 with the low word of
// splitmix64(seed, gv), elements + 4 .. + 7 with the high word.
template <bool BLOCKED>
struct Mxfp8Rs {
    static constexpr uint32_t kLanesPerBlock = 4;
    uint64_t seed;
    __device__ __forceinline__ void operator()(const uint4 v, bool valid, size_t gv, uint32_t lane,
                                               uint8_t* q, uint8_t* sf, size_t sf_cols) const {
        uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v.x, v.y),
                                              dt::bf16x2_absmax_bits(v.z, v.w)));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
        const uint32_t code = dt::mxfp8_scale_code(__uint_as_float(m << 16));
        const float inv = dt::ue8m0_inverse(code);
        const uint64_t h = dt::splitmix64(seed, gv);
        const float2 a = dt::bf16x2_mul_f32(v.x, inv), b = dt::bf16x2_mul_f32(v.y, inv);
        const float2 c = dt::bf16x2_mul_f32(v.z, inv), d = dt::bf16x2_mul_f32(v.w, inv);
        const uint32_t lo =
            dt::e4m3x4_from_f32_rs<false>(a.x, a.y, b.x, b.y, static_cast<uint32_t>(h));
        const uint32_t hi =
            dt::e4m3x4_from_f32_rs<false>(c.x, c.y, d.x, d.y, static_cast<uint32_t>(h >> 32));
        if (valid) {
            reinterpret_cast<uint2*>(q)[gv] = make_uint2(lo, hi);
            if ((lane & 3u) == 0) store_scale<BLOCKED>(sf, gv >> 2, sf_cols, code);
        }
    }
};

// Stochastic-rounding NVFP4: the same scale and reciprocal; elements with cvt.rs e2m1x4.
template <bool BLOCKED>
struct Nvfp4Rs {
    static constexpr uint32_t kLanesPerBlock = 2;
    float g, six_g;
    uint64_t seed;
    __device__ __forceinline__ void operator()(const uint4 v, bool valid, size_t gv, uint32_t lane,
                                               uint8_t* q, uint8_t* sf, size_t sf_cols) const {
        uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v.x, v.y),
                                              dt::bf16x2_absmax_bits(v.z, v.w)));
        m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
        const float s = __fdiv_rn(__uint_as_float(m << 16), six_g);
        const uint32_t code = dt::e4m3x2_from_f32<false>(s, 0.0f) & 0xFFu;
        const float t = __fmul_rn(dt::e4m3_to_f32(code), g);
        const float r = (t == 0.0f) ? 0.0f : __frcp_rn(t);
        const uint64_t h = dt::splitmix64(seed, gv);
        const float2 a = dt::bf16x2_mul_f32(v.x, r), b = dt::bf16x2_mul_f32(v.y, r);
        const float2 c = dt::bf16x2_mul_f32(v.z, r), d = dt::bf16x2_mul_f32(v.w, r);
        const uint32_t lo =
            dt::e2m1x4_from_f32_rs<false>(a.x, a.y, b.x, b.y, static_cast<uint32_t>(h));
        const uint32_t hi =
            dt::e2m1x4_from_f32_rs<false>(c.x, c.y, d.x, d.y, static_cast<uint32_t>(h >> 32));
        if (valid) {
            reinterpret_cast<uint32_t*>(q)[gv] = lo | (hi << 16);
            if ((lane & 1u) == 0) store_scale<BLOCKED>(sf, gv >> 1, sf_cols, code);
        }
    }
};

template <class Cfg, class Op>
__global__ void __launch_bounds__(Cfg::kThreads, 1)
    quantize_kernel(const uint16_t* __restrict__ x, size_t n_elems, Op op, uint8_t* __restrict__ q,
                    uint8_t* __restrict__ sf, size_t sf_cols, uint32_t* err) {
    using Smem = typename Cfg::Smem;
    constexpr uint32_t CW = Cfg::kConsumerWarps, VPL = Cfg::kVecsPerLane, ST = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                       ~static_cast<uintptr_t>(127));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const size_t n_chunks = (n_elems + Cfg::kChunkElems - 1) / Cfg::kChunkElems;
    const size_t n_vec = n_elems / 8;

    // Programmatic dependent launch: the next kernel of the stream may start its prologue on the
    // SMs this grid frees; it reads nothing of ours before its own griddepcontrol.wait.
    asm volatile("griddepcontrol.launch_dependents;");

    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < ST; ++i) {
            ptxstd::mbar_init(&s.full[i], 1);
            ptxstd::mbar_init(&s.empty[i], CW);
        }
        s.abort = 0;
        ptxstd::fence_mbarrier_init();
    }
    __syncthreads();
    // The previous kernel of the stream (which may have produced x, or still read q and sf) has
    // completed and its memory is visible from here on.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    volatile uint32_t* abort_flag = &s.abort;

    if (warp == CW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
            for (size_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
                if (!mbar_wait(&s.empty[stage], phase ^ 1u)) {
                    ptxstd::record_error(err, PTXSTD_ETIMEOUT, kDetailProducer | stage);
                    *abort_flag = 1u;
                    break;
                }
                if (*abort_flag) break;
                const size_t e0 = c * Cfg::kChunkElems;
                const uint32_t bytes = static_cast<uint32_t>(
                    min(static_cast<size_t>(Cfg::kChunkElems), n_elems - e0) * 2);
                ptxstd::mbar_arrive_expect_tx(&s.full[stage], bytes);
                ptxstd::bulk_load(s.buf[stage], x + e0, bytes, &s.full[stage]);
                issued |= 1u << stage;
                issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == ST) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            if (*abort_flag) {
                for (uint32_t i = 0; i < ST; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.full[i], (issued_parity >> i) & 1u);
            }
        }
    } else {
        // ---------------- consumers ----------------
        uint32_t stage = 0, phase = 0;
        for (size_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
            bool ok = !*abort_flag && mbar_wait(&s.full[stage], phase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !*abort_flag) {
                    ptxstd::record_error(err, PTXSTD_ETIMEOUT, kDetailConsumer | stage);
                    *abort_flag = 1u;
                }
                break;
            }
            const uint4* buf = reinterpret_cast<const uint4*>(s.buf[stage]);
            const size_t v0 = c * Cfg::kChunkVecs;
            // vectors of this chunk that exist (all of them except in the last chunk)
            const uint32_t live = static_cast<uint32_t>(
                min(static_cast<size_t>(Cfg::kChunkVecs), n_vec - v0));
            uint4 v[VPL];
#pragma unroll
            for (uint32_t j = 0; j < VPL; ++j) {
                const uint32_t lv = (j * CW + warp) * 32 + lane;
                v[j] = lv < live ? buf[lv] : make_uint4(0, 0, 0, 0);
            }
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive(&s.empty[stage]);
#pragma unroll
            for (uint32_t j = 0; j < VPL; ++j) {
                const uint32_t lv = (j * CW + warp) * 32 + lane;
                op(v[j], lv < live, v0 + lv, lane, q, sf, sf_cols);
            }
            if (++stage == ST) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
}

template <class Cfg, class Op>
int launch(const uint16_t* x, size_t n_elems, Op op, uint8_t* q, uint8_t* sf, size_t sf_cols,
           cudaStream_t stream) {
    int st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(quantize_kernel<Cfg, Op>),
                                          static_cast<int>(Cfg::kSmemBytes));
    if (st) return st;
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    const size_t chunks = (n_elems + Cfg::kChunkElems - 1) / Cfg::kChunkElems;
    const size_t sms = static_cast<size_t>(ptxstd::sm_count());
    const int grid = static_cast<int>(chunks < sms ? chunks : sms);
    // Launched with programmatic stream serialisation, so that back-to-back calls overlap the
    // launch and the barrier set-up with the previous kernel's last chunks.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(static_cast<uint32_t>(grid));
    cfg.blockDim = dim3(Cfg::kThreads);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, quantize_kernel<Cfg, Op>, x, n_elems, op, q, sf, sf_cols, err) !=
        cudaSuccess)
        return PTXSTD_ECUDA;
    return ptxstd::launch_status();
}

template <uint32_t T>
int launch_mx(const uint16_t* x, size_t n, uint8_t* q, uint8_t* sf, size_t sf_cols, int blocked,
              cudaStream_t s) {
    if (blocked) return launch<DefaultCfg>(x, n, MxAny<true, T>{0.0f}, q, sf, sf_cols, s);
    return launch<DefaultCfg>(x, n, MxAny<false, T>{0.0f}, q, sf, sf_cols, s);
}

}  // namespace

extern "C" {

int ptxstd_quantize_mx(const uint16_t* d_x, int64_t rows, int64_t cols, int elem_type,
                       uint8_t* d_q, uint8_t* d_sf, int sf_layout, ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 32 != 0) return PTXSTD_EINVAL;
    if (!d_x || !d_q || !d_sf || !ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_q))
        return PTXSTD_EINVAL;
    if (sf_layout != 0 && sf_layout != 1) return PTXSTD_EINVAL;
    if (sf_layout == 1 && (rows % 128 != 0 || cols % 128 != 0)) return PTXSTD_EINVAL;
    const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
    const size_t sf_cols = static_cast<size_t>(cols) / 32;
    auto s = static_cast<cudaStream_t>(stream);
    switch (elem_type) {
    case 0: return launch_mx<0>(d_x, n, d_q, d_sf, sf_cols, sf_layout, s);
    case 1: return launch_mx<1>(d_x, n, d_q, d_sf, sf_cols, sf_layout, s);
    case 3: return launch_mx<3>(d_x, n, d_q, d_sf, sf_cols, sf_layout, s);
    case 4: return launch_mx<4>(d_x, n, d_q, d_sf, sf_cols, sf_layout, s);
    case 5: return launch_mx<5>(d_x, n, d_q, d_sf, sf_cols, sf_layout, s);
    default: return PTXSTD_EINVAL;
    }
}

int ptxstd_quantize_mxfp8_layout(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                                 uint8_t* d_sf, int sf_layout, ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 32 != 0) return PTXSTD_EINVAL;
    if (!d_x || !d_q || !d_sf || !ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_q))
        return PTXSTD_EINVAL;
    if (sf_layout != 0 && sf_layout != 1) return PTXSTD_EINVAL;
    if (sf_layout == 1 && (rows % 128 != 0 || cols % 128 != 0)) return PTXSTD_EINVAL;
    const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
    const size_t sf_cols = static_cast<size_t>(cols) / 32;
    auto s = static_cast<cudaStream_t>(stream);
    if (sf_layout == 1) return launch<DefaultCfg>(d_x, n, Mxfp8<true>{0.0f}, d_q, d_sf, sf_cols, s);
    return launch<DefaultCfg>(d_x, n, Mxfp8<false>{0.0f}, d_q, d_sf, sf_cols, s);
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
    const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
    const size_t sf_cols = static_cast<size_t>(cols) / 16;
    auto s = static_cast<cudaStream_t>(stream);
    // six_g = 6 * g as one IEEE rounding, as in the recipe.
    const float six_g = 6.0f * global_scale;
    if (sf_layout == 1)
        return launch<DefaultCfg>(d_x, n, Nvfp4<true>{global_scale, six_g}, d_q, d_sf, sf_cols, s);
    return launch<DefaultCfg>(d_x, n, Nvfp4<false>{global_scale, six_g}, d_q, d_sf, sf_cols, s);
}

int ptxstd_quantize_nvfp4(const uint16_t* d_x, int64_t rows, int64_t cols, float global_scale,
                          uint8_t* d_q, uint8_t* d_sf, ptxstd_stream stream) {
    return ptxstd_quantize_nvfp4_layout(d_x, rows, cols, global_scale, d_q, d_sf, 0, stream);
}

int ptxstd_quantize_mxfp8_rs(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                             uint8_t* d_sf, int sf_layout, uint64_t seed, ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 32 != 0) return PTXSTD_EINVAL;
    if (!d_x || !d_q || !d_sf || !ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_q))
        return PTXSTD_EINVAL;
    if (sf_layout != 0 && sf_layout != 1) return PTXSTD_EINVAL;
    if (sf_layout == 1 && (rows % 128 != 0 || cols % 128 != 0)) return PTXSTD_EINVAL;
    const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
    const size_t sf_cols = static_cast<size_t>(cols) / 32;
    auto s = static_cast<cudaStream_t>(stream);
    if (sf_layout == 1) return launch<DefaultCfg>(d_x, n, Mxfp8Rs<true>{seed}, d_q, d_sf, sf_cols, s);
    return launch<DefaultCfg>(d_x, n, Mxfp8Rs<false>{seed}, d_q, d_sf, sf_cols, s);
}

int ptxstd_quantize_nvfp4_rs(const uint16_t* d_x, int64_t rows, int64_t cols, float global_scale,
                             uint8_t* d_q, uint8_t* d_sf, int sf_layout, uint64_t seed,
                             ptxstd_stream stream) {
    if (rows <= 0 || cols <= 0 || cols % 16 != 0) return PTXSTD_EINVAL;
    if (!(global_scale > 0.0f) || global_scale == __builtin_huge_valf()) return PTXSTD_EINVAL;
    if (!d_x || !d_q || !d_sf || !ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_q))
        return PTXSTD_EINVAL;
    if (sf_layout != 0 && sf_layout != 1) return PTXSTD_EINVAL;
    if (sf_layout == 1 && (rows % 128 != 0 || cols % 64 != 0)) return PTXSTD_EINVAL;
    const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
    const size_t sf_cols = static_cast<size_t>(cols) / 16;
    auto s = static_cast<cudaStream_t>(stream);
    const float six_g = 6.0f * global_scale;
    if (sf_layout == 1)
        return launch<DefaultCfg>(d_x, n, Nvfp4Rs<true>{global_scale, six_g, seed}, d_q, d_sf,
                                  sf_cols, s);
    return launch<DefaultCfg>(d_x, n, Nvfp4Rs<false>{global_scale, six_g, seed}, d_q, d_sf,
                              sf_cols, s);
}

}  // extern "C"

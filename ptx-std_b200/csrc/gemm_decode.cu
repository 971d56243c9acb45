// Decode-shape GEMM: y[M, N] (bf16, M <= 16 tokens) = MXFP8(x)[M, K] * NVFP4(W)[N, K]^T * gw.
//
// x is bf16 and is quantised on the fly to MXFP8 (E4M3 + UE8M0 per 32, the recipe of
// ptxstd_quantize_mxfp8); W is E2M1 packed two per byte with E4M3 scales per 16 (blocked 128x4
// layout) and an f32 global scale. No block-scaled tcgen05 kind takes one UE8M0/32 operand and one
// E4M3/16 operand (kind::mxf8f6f4 wants UE8M0 on both, kind::mxf4nvf4 wants E2M1 on both;
// src/tcgen05/descriptor.rs:589-653), so both operands are brought to f16 exactly and multiplied
// with tcgen05.mma.kind::f16 (fp32 accumulation):
//   - W: e2m1 x e4m3 has at most 6 significant bits and lies in [2^-10, 2688], so
//     cvt.rn.f16x2.e2m1x2 followed by one f16x2 multiply by the scale is exact;
//   - x: q * 2^(code - 127) is rewritten per token row as f16 q * 2^(code - maxcode_row), exact
//     for blocks within 15 binades of the row's largest block; the factor 2^(maxcode_row - 127) is
//     applied to the fp32 result.
// The op is weight-streaming (HBM-bound): each W byte is read once.
//
// Kernel 1, decode_prep (one CTA per token row; CTA 0 also clears the per-block counters):
//   MXFP8-quantises x and writes the f16 B operand pre-swizzled (K-major, 128-byte swizzle, 8 KiB
//   per 256-K stage) so that the main kernel fetches it with one 1-D bulk copy per stage. Its 16
//   CTAs leave the other SMs free, so the main kernel's weight stream starts at once.
// Kernel 2, gemm_decode (persistent, one CTA per SM, launched with programmatic dependent launch so
//   its setup and first weight loads overlap kernel 1):
//   work = (128-row W block, 256-K stage) units split evenly over the CTAs ("stream-K"), each
//           CTA walking its range in the order of unit_runs;
//   warp 0: weight producer: W tile 128 x 128 bytes + W scales 2 KiB per stage into an 8-stage
//           ring that the dequant warps release as soon as they have read it (so the HBM stream
//           never waits on MMA completion, nor on kernel 1), loaded with an L2 evict-first policy;
//   warp kXWarp: x-image producer: the 8 KiB f16 B operand per stage into a 4-stage ring released by
//           the MMA commit (it waits for kernel 1 with griddepcontrol.wait);
//   warp 1: TMEM owner + MMA issuer: 16 MMAs of M=128 (W rows), N=16 (tokens), K=16 per stage with
//           the A operand in TMEM, into one of two accumulators (one per W-block segment);
//   warps 2 .. 2 + kDqWarps - 1: dequantise W rows into TMEM (tcgen05.st; kDqPerQ warps per lane
//           quarter in kTeams teams that take the units in turn, each warp a 64 * kSubs-element
//           K slice of its team's units; three A buffers);
//   warps kEpiWarp .. kEpiWarp + 3 (one per lane quarter): at the end of each W-block segment,
//           drain the accumulator, off the dequant / MMA path (the MMA already fills the other
//           accumulator). A block that lies inside this CTA's range is converted to bf16 straight
//           from registers, transposed through shared memory and written to y in 16-byte row
//           chunks. A block shared with neighbouring CTAs is written as an fp32 partial to this
//           CTA's slot; a per-block counter elects the CTA that arrives last, which sums the
//           partials of all contributors in CTA order (so the result is the same bits whichever
//           CTA is last) and writes y the same way.
// Output routing (decode_out.h): one local y, or, for the N-sharded multi-GPU path, the y of every
// rank over NVLink (the epilogue's stores go to each rank's copy; counters and bounded waits order
// the steps; kernel 3, decode_done, waits until every rank's pieces have arrived).
#include <mutex>

#include "common.cuh"
#include "data_types.cuh"
#include "decode_out.h"
#include "tcgen05.cuh"
#include "tma_host.h"

namespace {

namespace t5 = ptxstd::tcgen05;
namespace dt = ptxstd::data_types;
using ptxstd::mbar_wait;

constexpr uint32_t BM = 128;            // W rows per block (MMA M)
constexpr uint32_t BKS = 256;           // K elements per stage
constexpr uint32_t kWStageBytes = BM * BKS / 2;   // 16 KiB packed E2M1
constexpr uint32_t kSfStageBytes = BM * BKS / 16; // 2 KiB E4M3
constexpr uint32_t kTok = 16;           // MMA N (tokens, padded)
constexpr uint32_t kXStageBytes = kTok * BKS * 2; // 8 KiB f16
constexpr uint32_t kWRingBytes = kWStageBytes + kSfStageBytes;   // one weight stage
constexpr uint32_t WST = 8;             // weight ring: released by the dequant warps after their loads
// On its first pass through the ring the weight producer keeps at most kRamp stages in flight.
// The CTAs that start late (on the SMs that held the prep kernel's CTAs) then do not find HBM
// queued up with every other CTA's full 8-stage burst; measured on a B200 at M = 16, K = 8192:
// N = 57344 56.0 -> 54.6 us per call, N = 28672 33.8 -> 33.4 us (2 and 4 stages gained less).
constexpr uint32_t kRamp = 3;
constexpr uint32_t XST = 4;             // x-image ring: released by the MMA commit
constexpr uint32_t kDqPerQ = 4;                    // dequant warps per TMEM lane quarter
constexpr uint32_t kDqWarps = 4 * kDqPerQ;
// The dequant warps form kTeams teams that take the units in turn (team t: the CTA's units
// t, t + kTeams, ...), so each warp has kTeams units' time for the latency of one unit (shared
// memory loads, the TMEM store and its wait, the barrier hand-offs).
constexpr uint32_t kTeams = 2;
constexpr uint32_t kTeamWarpsPerQ = kDqPerQ / kTeams;   // warps of a team per lane quarter
constexpr uint32_t kTeamWarps = 4 * kTeamWarpsPerQ;     // arrivals per unit on wempty / afull
constexpr uint32_t kSubs = 4 / kTeamWarpsPerQ;          // 64-K slices of a row per warp and unit
static_assert(kDqPerQ % kTeams == 0 && 4 % kTeamWarpsPerQ == 0, "team layout");
constexpr uint32_t kFirstDqWarp = 2;
constexpr uint32_t kXWarp = kFirstDqWarp + kDqWarps;   // x-image producer warp
constexpr uint32_t kEpiWarp = kXWarp + 1;              // first of the four epilogue warps
constexpr uint32_t kThreads = 32 * (kEpiWarp + 4);
constexpr uint32_t kACols = BKS / 2;    // f16 pairs per row per stage = 128 TMEM columns
constexpr uint32_t kABufs = 3;          // A operand buffers in TMEM
constexpr uint32_t kDBufs = 2;          // accumulators (one per W-block segment in flight)
constexpr uint32_t kDCol = kABufs * kACols;  // accumulator columns after the A buffers
static_assert(kDCol + kDBufs * kTok <= 512, "TMEM budget");
// Parity waits only tell a phase from the one before it. A team at unit i has already waited on
// its unit i - kTeams, so (a) with kTeams <= kABufs the MMA has finished unit i - 2 kABufs when
// the team waits for buffer i % kABufs to be freed from unit i - kABufs, and (b) with
// WST % kTeams == 0 the team itself consumed unit i - WST of stage i % WST. Either way no wait is
// ever two phases ahead of its barrier.
static_assert(kTeams <= kABufs && WST % kTeams == 0, "team count vs. A buffers and weight ring");
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kPrepThreads = 1024;
constexpr uint32_t kFinMax = 5;  // contributors of a shared block staged in shared memory at once

struct alignas(1024) Smem {
    uint8_t w[WST][kWStageBytes];
    uint8_t x[XST][kXStageBytes];
    uint8_t sf[WST][kSfStageBytes];
    // finishing a shared block: up to kFinMax contributors' partial rows, fetched at once
    float4 fin[kFinMax][BM][kTok / 4];
    uint16_t ytile[4][kTok][32];  // per epilogue warp: its 32 block columns x 16 tokens, bf16
    float fac[4][kTok];           // per epilogue warp: token factors x gw (kept out of registers)
    uint64_t wfull[WST];
    uint64_t wempty[WST];
    uint64_t xfull[XST];
    uint64_t xempty[XST];
    uint64_t afull[kABufs];
    uint64_t aempty[kABufs];
    uint64_t dfull[kDBufs];
    uint64_t dempty[kDBufs];
    uint64_t segA;
    uint64_t segB;
    uint64_t drain;
    uint32_t tmem_base;
    uint32_t abort;
    uint32_t finalize;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory budget");

enum : uint32_t { kDetailProducer = 0x3100, kDetailMma = 0x3200, kDetailDq = 0x3300,
                  kDetailXProducer = 0x3400, kDetailEpi = 0x3500 };

// Workspace layout (bytes), for a grid of G CTAs:
//   partial slots [G][2][128 rows][16 tokens] f32: the fp32 partial sums of the W blocks that a
//     CTA shares with its neighbours (slot 0: its first segment, slot 1: its last one);
//   counters [N/128] u32 (1024-byte aligned end): per block, the contributors that have arrived;
//   x image [K/256][8 KiB]; factors [16] f32.
// Only the counters must start at zero, and decode_prep clears them (N/128 words) on every call;
// a slot is always written before it is read.
constexpr size_t kSlotBytes = static_cast<size_t>(BM) * kTok * 4;  // 8 KiB
struct Workspace {
    float* slots;
    uint32_t* counters;
    uint8_t* ximg;
    float* factors;
};
__host__ __device__ inline size_t ws_counters_off(size_t G) { return G * 2 * kSlotBytes; }
__host__ __device__ inline size_t ws_ximg_off(size_t G, size_t N) {
    return ws_counters_off(G) + (((N / BM) * 4 + 1023) & ~static_cast<size_t>(1023));
}
__host__ __device__ inline size_t ws_factors_off(size_t G, size_t N, size_t K) {
    return ws_ximg_off(G, N) + K * kTok * 2;
}
__host__ __device__ inline size_t ws_bytes(size_t G, size_t N, size_t K) {
    return ws_factors_off(G, N, K) + 64;
}
__host__ __device__ inline Workspace ws_layout(uint8_t* ws, size_t G, size_t N, size_t K) {
    return Workspace{reinterpret_cast<float*>(ws),
                     reinterpret_cast<uint32_t*>(ws + ws_counters_off(G)),
                     ws + ws_ximg_off(G, N),
                     reinterpret_cast<float*>(ws + ws_factors_off(G, N, K))};
}

// Stream-K bookkeeping: unit u of U = (N/128) * (K/256) is (block u / S, stage u % S); CTA c of G
// owns [floor(U c / G), floor(U (c + 1) / G)), so unit u belongs to CTA floor((u G + G - 1) / U).
__host__ __device__ inline uint64_t unit_begin(uint64_t U, uint64_t G, uint64_t c) {
    return U * c / G;
}
__host__ __device__ inline uint32_t unit_owner(uint64_t U, uint64_t G, uint64_t u) {
    return static_cast<uint32_t>((u * G + G - 1) / U);
}

// Host side: CTAs of the GEMM kernel on the current device: one per SM, but at least
// kMinUnitsPerCta units each, which bounds how many CTAs share a block (and so how many partials
// the last of them reads back) when there is little work.
// With K = 8192 (32 units per block), 8 units per CTA keep a shared block to at most 5
// contributors, which the finishing CTA fetches in one round trip (kFinMax). Measured on a B200
// against one CTA per SM at M = 16, K = 8192: N = 3584 12.2 us (13.5 before), N = 1024 12.0 us
// (10.4); at N >= 7168 every SM gets more than 8 units anyway.
constexpr size_t kMinUnitsPerCta = 8;
inline size_t decode_grid(size_t N, size_t K) {
    const size_t units = (N / BM) * (K / BKS);
    const size_t sms = static_cast<size_t>(ptxstd::sm_count());
    size_t g = units / kMinUnitsPerCta;
    if (g < 1) g = 1;
    return g < sms ? g : sms;
}
inline size_t decode_ws_bytes(size_t N, size_t K) { return ws_bytes(decode_grid(N, K), N, K); }

// Byte offset of f16 element (row r < 16, k) in the x image: per 256-K stage 8 KiB made of four
// 64-element K atoms of 16 rows x 128 bytes, 16-byte chunks XOR-swizzled by row % 8.
__device__ __forceinline__ uint32_t ximg_offset(uint32_t r, uint32_t k) {
    const uint32_t stage = k / BKS, kk = k % BKS;
    const uint32_t atom = kk / 64, byte = (kk % 64) * 2;
    return stage * kXStageBytes + atom * (kTok * 128) + r * 128 +
           (((byte >> 4) ^ (r & 7)) << 4) + (byte & 15);
}

// MXFP8 scale code of the 32-element block whose four 16-byte vectors are held by this lane and
// its three neighbours (lanes 4j .. 4j + 3); all 32 lanes of the warp take part.
__device__ __forceinline__ uint32_t prep_block_code(const uint4& v) {
    uint32_t m = dt::bf16x2_fold(__vmaxu2(dt::bf16x2_absmax_bits(v.x, v.y),
                                          dt::bf16x2_absmax_bits(v.z, v.w)));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    return dt::mxfp8_scale_code(__uint_as_float(m << 16));
}

// ---------------------------------------------------------------------------------------------
// Kernel 1: x -> MXFP8 -> f16 B-operand image and per-row factors, one CTA per token row (rows
// >= M write zeros); CTA 0 also clears the block counters. Sixteen small CTAs leave the other SMs
// to the GEMM kernel, whose weight stream starts while this one runs.
__global__ void __launch_bounds__(kPrepThreads)
    decode_prep_kernel(const uint16_t* __restrict__ x, uint32_t M, uint32_t K, uint8_t* ws,
                       uint32_t N, uint32_t G, const ptxstd::decode::Out out) {
    asm volatile("griddepcontrol.launch_dependents;");
    if (out.nranks != 0 && blockIdx.x == 0 && threadIdx.x < out.nranks) {
        // peer-to-peer output: this rank starts a step (see decode_out.h)
        namespace pd = ptxstd::decode;
        if (threadIdx.x == 0) out.sig[out.rank][pd::kSigStep] += 1u;
        atomicAdd_system(out.sig[threadIdx.x] + pd::kSigReady + out.rank, 1u);
    }
    const Workspace w = ws_layout(ws, G, N, K);
    if (blockIdx.x == 0)
        for (uint32_t i = threadIdx.x; i < N / BM; i += blockDim.x) w.counters[i] = 0;
    const uint32_t r = blockIdx.x;
    __shared__ uint32_t red[kPrepThreads / 32];
    // 16-byte vectors of the row (K % 256 == 0, so a multiple of 32: every warp runs the loops
    // below the same number of times, as the block shuffles need). A 32-element block is the
    // vectors of four neighbouring lanes.
    const uint32_t nvec = K / 8;
    const uint4* xrow = reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * K);
    // pass 1: block scale codes and the row's largest code. A thread's first vector and its code
    // stay in registers for pass 2 (at K <= 8192 that is the thread's only vector).
    uint4 v0 = make_uint4(0, 0, 0, 0);
    uint32_t code0 = 0, maxcode = 0;
    if (r < M) {
        for (uint32_t i = threadIdx.x; i < nvec; i += kPrepThreads) {
            const uint4 v = xrow[i];
            const uint32_t code = prep_block_code(v);
            if (i == threadIdx.x) {
                v0 = v;
                code0 = code;
            }
            if (code != 0xFFu) maxcode = max(maxcode, code);
        }
    }
    for (int o = 16; o > 0; o >>= 1) maxcode = max(maxcode, __shfl_xor_sync(0xffffffffu, maxcode, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = maxcode;
    __syncthreads();
    maxcode = 0;
    for (uint32_t i = 0; i < kPrepThreads / 32; ++i) maxcode = max(maxcode, red[i]);
    if (threadIdx.x == 0) {
        // 2^(maxcode - 127) in f32 (maxcode <= 254; 0 for padding rows)
        w.factors[r] = r < M ? (maxcode >= 1 ? __uint_as_float(maxcode << 23)
                                             : __uint_as_float(0x00400000u))
                             : 0.0f;
    }
    // pass 2: elements as f16 q * 2^(code - maxcode), one 16-byte chunk of the image per vector
    for (uint32_t i = threadIdx.x; i < nvec; i += kPrepThreads) {
        uint32_t h[4] = {0u, 0u, 0u, 0u};
        if (r < M) {
            const bool first = i == threadIdx.x;
            const uint4 v = first ? v0 : xrow[i];
            const uint32_t code = first ? code0 : prep_block_code(v);
            const float inv = dt::ue8m0_inverse(code);
            // factor 2^(code - maxcode) in f32 (>= 2^-254 is not representable: flush below 2^-149)
            const int d = static_cast<int>(code) - static_cast<int>(maxcode);
            const float rel = code == 0xFFu ? __uint_as_float(0x7FFFFFFFu)
                              : d >= -126   ? __uint_as_float(static_cast<uint32_t>(d + 127) << 23)
                              : d >= -149   ? __uint_as_float(1u << (d + 149))
                                            : 0.0f;
            const uint32_t ww[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const uint16_t qq = dt::e4m3x2_from_f32<false>(__fmul_rn(dt::bf16_lo(ww[k]), inv),
                                                               __fmul_rn(dt::bf16_hi(ww[k]), inv));
                const float2 qf = dt::e4m3x2_to_f32(qq);
                asm("cvt.rn.f16x2.f32 %0, %1, %2;"
                    : "=r"(h[k])
                    : "f"(__fmul_rn(qf.y, rel)), "f"(__fmul_rn(qf.x, rel)));
            }
        }
        *reinterpret_cast<uint4*>(w.ximg + ximg_offset(r, i * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// ---------------------------------------------------------------------------------------------
// Kernel 2.
__device__ __forceinline__ void fail(Smem& s, uint32_t* err, uint32_t detail) {
    ptxstd::record_error(err, PTXSTD_ETIMEOUT, detail);
    *reinterpret_cast<volatile uint32_t*>(&s.abort) = 1u;
}
__device__ __forceinline__ bool aborted(Smem& s) {
    return *reinterpret_cast<volatile uint32_t*>(&s.abort) != 0u;
}

// Eight E2M1 values (one 32-bit word, element 0 in the low nibble) times an f16x2 scale ->
// four f16x2 words: the word is unpacked into its four bytes, each converted by one
// cvt.rn.f16x2.e2m1x2 (narrow.rs pair_to_f16) and multiplied by the scale. Exact: e2m1 x e4m3
// has at most 6 significant bits and lies in [2^-10, 2688].
__device__ __forceinline__ void dequant8(uint32_t w, uint32_t scale2, uint32_t* o) {
    asm("{\n\t.reg .b8 t0, t1, t2, t3;\n\t.reg .b32 u0, u1, u2, u3;\n\t"
        "mov.b32 {t0, t1, t2, t3}, %4;\n\t"
        "cvt.rn.f16x2.e2m1x2 u0, t0;\n\tcvt.rn.f16x2.e2m1x2 u1, t1;\n\t"
        "cvt.rn.f16x2.e2m1x2 u2, t2;\n\tcvt.rn.f16x2.e2m1x2 u3, t3;\n\t"
        "mul.rn.f16x2 %0, u0, %5;\n\tmul.rn.f16x2 %1, u1, %5;\n\t"
        "mul.rn.f16x2 %2, u2, %5;\n\tmul.rn.f16x2 %3, u3, %5;\n\t}"
        : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
        : "r"(w), "r"(scale2));
}

// tcgen05.st.32x32b.x32: 32 consecutive columns of this warp's lane quarter.
__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t* v) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, "
        "%29, %30, %31, %32};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
        "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
        "r"(v[29]), "r"(v[30]), "r"(v[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 16-byte asynchronous copy global (L2) -> this thread's shared memory, and the wait for all of
// this thread's copies: the partial rows of a shared block are all in flight at once.
__device__ __forceinline__ void cp_async_16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(ptxstd::smem_u32(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}
// A from TMEM: tcgen05.mma.cta_group::1.kind::f16 [d], [a], b_desc, idesc.
__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d, uint32_t a, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Bounded wait until a peer-written counter reaches `target` (wrap-safe), acquire at system scope.
__device__ __forceinline__ bool wait_counter(const uint32_t* p, uint32_t target) {
    const uint64_t t0 = ptxstd::global_timer();
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
        if (static_cast<int32_t>(v - target) >= 0) return true;
        if (ptxstd::global_timer() - t0 > ptxstd::kWaitLimitNs) return false;
    }
}

// Unit u of U = nblocks * S is (block u / S, stage u % S); CTA c owns [c U / G, (c+1) U / G).
__device__ __forceinline__ void unit_range(uint64_t U, uint32_t& u0, uint32_t& u1) {
    u0 = static_cast<uint32_t>(U * blockIdx.x / gridDim.x);
    u1 = static_cast<uint32_t>(U * (blockIdx.x + 1) / gridDim.x);
}

// The order in which a CTA works through its range [u0, u1), as runs of units of one W block (one
// accumulator each): run A, the part of the block the range starts in; the whole blocks; run B,
// the part of the block it ends in. In range order (A, whole blocks, B) the CTA's last run is the
// head of a block it shares with the next CTA, which finished that block's tail long before, so
// the call ends on that block's finish (partial, counter, the others' partials fetched and
// summed). When every CTA holds whole blocks (U / G >= 2 S), the order A, B, whole blocks ends
// each CTA on a whole block stored straight from registers instead, and the shared blocks are
// finished while the weight stream goes on; the whole blocks then take their K stages from
// u0 % S on (wrapping), so that the CTAs keep reading different K stages (and x-image stages) at
// any moment, as they do in range order. Every role walks the same runs.
struct UnitRuns {
    uint32_t nbA, ksA, nA;  // run A: block nbA, stages ksA .. ksA + nA - 1
    uint32_t nbB, nB;       // run B (if nB > 0): block nbB, stages 0 .. nB - 1
    uint32_t nbM, nM, rot;  // whole blocks nbM .. nbM + nM - 1, stages rot, rot + 1, ... mod S
    uint32_t nruns, b_first;
};
__device__ __forceinline__ UnitRuns unit_runs(uint32_t u0, uint32_t u1, uint32_t S,
                                              bool b_first) {
    UnitRuns o = {};
    if (u0 >= u1) return o;
    const uint32_t f1 = min(u1, (u0 / S + 1) * S);  // end of run A
    o.nbA = u0 / S, o.ksA = u0 % S, o.nA = f1 - u0, o.nruns = 1;
    if (f1 == u1) return o;
    const uint32_t l0 = ((u1 - 1) / S) * S;  // start of run B, >= f1
    o.nbB = l0 / S, o.nB = u1 - l0;
    o.nbM = f1 / S, o.nM = (l0 - f1) / S;
    o.b_first = b_first ? 1u : 0u;
    o.rot = b_first ? u0 % S : 0u;
    o.nruns = 2 + o.nM;
    return o;
}
// Run r of o: its block, first stage and unit count; unit k of the run is stage (ks0 + k) mod S.
__device__ __forceinline__ void unit_run(const UnitRuns& o, uint32_t r, uint32_t S, uint32_t& nb,
                                         uint32_t& ks0, uint32_t& cnt) {
    const uint32_t rb = o.b_first ? 1u : o.nM + 1;  // the index of run B
    if (r == 0) {
        nb = o.nbA, ks0 = o.ksA, cnt = o.nA;
    } else if (r == rb) {
        nb = o.nbB, ks0 = 0, cnt = o.nB;
    } else {
        nb = o.nbM + r - (o.b_first ? 2u : 1u), ks0 = o.rot, cnt = S;
    }
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_decode_kernel(const __grid_constant__ CUtensorMap tmW, const uint8_t* __restrict__ sfW,
                       uint8_t* ws, const __grid_constant__ ptxstd::decode::Out out, uint32_t M,
                       uint32_t N, uint32_t K, float gw, uint32_t* err, uint32_t b_first) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
    const uint32_t warp = ptxstd::warp_id();
    const uint32_t lane = ptxstd::lane_id();
    const uint32_t S = K / BKS;
    const uint64_t U = static_cast<uint64_t>(N / BM) * S;
    uint32_t u0, u1;
    unit_range(U, u0, u1);
    const Workspace wsp = ws_layout(ws, gridDim.x, N, K);

    if (warp == 0 && lane == 0) {
        ptxstd::prefetch_tensormap(&tmW);
        for (uint32_t i = 0; i < WST; ++i) {
            ptxstd::mbar_init(&s.wfull[i], 1);
            ptxstd::mbar_init(&s.wempty[i], kTeamWarps);
        }
        for (uint32_t i = 0; i < XST; ++i) {
            ptxstd::mbar_init(&s.xfull[i], 1);
            ptxstd::mbar_init(&s.xempty[i], 1);
        }
        for (uint32_t i = 0; i < kABufs; ++i) {
            ptxstd::mbar_init(&s.afull[i], kTeamWarps);
            ptxstd::mbar_init(&s.aempty[i], 1);
        }
        for (uint32_t i = 0; i < kDBufs; ++i) {
            ptxstd::mbar_init(&s.dfull[i], 1);
            ptxstd::mbar_init(&s.dempty[i], 4);
        }
        ptxstd::mbar_init(&s.segA, 4);
        ptxstd::mbar_init(&s.segB, 1);
        ptxstd::mbar_init(&s.drain, 1);
        s.abort = 0;
        s.finalize = 0;
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
        // ---------------- weight producer: W tiles + W scales (no dependency on decode_prep) ----
        if (ptxstd::elect_one()) {
            uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
            const uint32_t sf_tiles_per_row = K / 64;
            // each weight byte is read once: evict-first keeps the partial slots and the x image
            // in L2 (N = 57344: 57.3 -> 56.5 us per call; N = 28672: 34.7 -> 34.0 us)
            const uint64_t pol = ptxstd::policy_evict_first();
            const UnitRuns ord = unit_runs(u0, u1, S, b_first != 0);
            bool stop = false;
            for (uint32_t r = 0, i = 0; r < ord.nruns && !stop; ++r) {
            uint32_t nb, ks0, cnt;
            unit_run(ord, r, S, nb, ks0, cnt);
            for (uint32_t k = 0, ks = ks0; k < cnt; ++k, ++i, ks = (ks + 1 == S) ? 0 : ks + 1) {
                if (!mbar_wait(&s.wempty[stage], phase ^ 1u)) {
                    fail(s, err, kDetailProducer | stage);
                    stop = true;
                    break;
                }
                // first pass: stage i - kRamp has landed before stage i is requested (its first
                // phase; it is refilled only after the producer wraps around)
                if (i >= kRamp && i < WST && !mbar_wait(&s.wfull[i - kRamp], 0)) {
                    fail(s, err, kDetailProducer | 0x40);
                    stop = true;
                    break;
                }
                if (aborted(s)) {
                    stop = true;
                    break;
                }
                ptxstd::mbar_arrive_expect_tx(&s.wfull[stage], kWRingBytes);
                ptxstd::tma_load_2d_hint(s.w[stage], &tmW, &s.wfull[stage],
                                         static_cast<int32_t>(ks * (BKS / 2)),
                                         static_cast<int32_t>(nb * BM), pol);
                ptxstd::bulk_load_hint(
                    s.sf[stage], sfW + (static_cast<size_t>(nb) * sf_tiles_per_row + ks * 4) * 512,
                    kSfStageBytes, &s.wfull[stage], pol);
                issued |= 1u << stage;
                issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == WST) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            }
            if (aborted(s)) {
                for (uint32_t i = 0; i < WST; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.wfull[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == kXWarp) {
        // ---------------- x-image producer (waits for decode_prep) ----------------
        if (ptxstd::elect_one()) {
            asm volatile("griddepcontrol.wait;" ::: "memory");
            uint32_t stage = 0, phase = 0, issued = 0, issued_parity = 0;
            const UnitRuns ord = unit_runs(u0, u1, S, b_first != 0);
            bool stop = false;
            for (uint32_t r = 0; r < ord.nruns && !stop; ++r) {
            uint32_t nb, ks0, cnt;
            unit_run(ord, r, S, nb, ks0, cnt);
            for (uint32_t k = 0, ks = ks0; k < cnt; ++k, ks = (ks + 1 == S) ? 0 : ks + 1) {
                if (!mbar_wait(&s.xempty[stage], phase ^ 1u)) {
                    fail(s, err, kDetailXProducer | stage);
                    stop = true;
                    break;
                }
                if (aborted(s)) {
                    stop = true;
                    break;
                }
                ptxstd::mbar_arrive_expect_tx(&s.xfull[stage], kXStageBytes);
                ptxstd::bulk_load(s.x[stage], wsp.ximg + static_cast<size_t>(ks) * kXStageBytes,
                                  kXStageBytes, &s.xfull[stage]);
                issued |= 1u << stage;
                issued_parity = (issued_parity & ~(1u << stage)) | (phase << stage);
                if (++stage == XST) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
            }
            if (aborted(s)) {
                for (uint32_t i = 0; i < XST; ++i)
                    if (issued & (1u << i)) mbar_wait(&s.xfull[i], (issued_parity >> i) & 1u);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (ptxstd::elect_one()) {
            uint32_t idesc = 0;
            t5::idesc_dense(/*F16*/ 0, /*F16*/ 0, /*F32*/ 1, BM, kTok, idesc);
            uint32_t stage = 0, phase = 0, abuf = 0, aphase = 0, dbuf = 0, dphase = 0;
            const UnitRuns ord = unit_runs(u0, u1, S, b_first != 0);
            bool stop = false;
            for (uint32_t r = 0; r < ord.nruns && !stop; ++r) {
            uint32_t nb, ks0, cnt;
            unit_run(ord, r, S, nb, ks0, cnt);
            for (uint32_t k = 0; k < cnt; ++k) {
                if (aborted(s)) {
                    stop = true;
                    break;
                }
                const bool first = k == 0;        // one accumulator per run
                const bool last = k + 1 == cnt;
                if (first) {
                    // the epilogue warps have drained this accumulator's previous segment
                    if (!mbar_wait(&s.dempty[dbuf], dphase ^ 1u)) {
                        fail(s, err, kDetailMma | 0x30);
                        stop = true;
                        break;
                    }
                }
                const uint32_t d = tmem + kDCol + dbuf * kTok;
                if (!mbar_wait(&s.afull[abuf], aphase) || !mbar_wait(&s.xfull[stage], phase)) {
                    fail(s, err, kDetailMma | stage);
                    stop = true;
                    break;
                }
                t5::fence_after_thread_sync();
                const uint32_t xs = ptxstd::smem_u32(s.x[stage]);
                const uint32_t a = tmem + abuf * kACols;
#pragma unroll
                for (uint32_t j = 0; j < BKS / 16; ++j) {
                    // B: K atom j / 4 (2 KiB apart), +32 bytes per K=16 step inside the atom.
                    const uint64_t bd = t5::smem_desc_k128(xs + (j / 4) * (kTok * 128) + (j % 4) * 32);
                    mma_f16_tmem_a(d, a + 8 * j, bd, idesc, (!first || j != 0) ? 1u : 0u);
                }
                t5::commit(&s.aempty[abuf]);
                t5::commit(&s.xempty[stage]);
                if (last) {
                    t5::commit(&s.dfull[dbuf]);
                    if (++dbuf == kDBufs) {
                        dbuf = 0;
                        dphase ^= 1u;
                    }
                }
                if (++stage == XST) {
                    stage = 0;
                    phase ^= 1u;
                }
                if (++abuf == kABufs) {
                    abuf = 0;
                    aphase ^= 1u;
                }
            }
            }
            t5::commit(&s.drain);
            mbar_wait(&s.drain, 0);
        }
    } else if (warp < kXWarp) {
        // ---------------- dequant (warps kFirstDqWarp .. kXWarp - 1) ----------------
        const uint32_t q = warp & 3u;                        // lane quarter = W rows 32q .. 32q+31
        const uint32_t h = (warp - kFirstDqWarp) >> 2;       // 0 .. kDqPerQ - 1
        const uint32_t team = h % kTeams;
        const uint32_t slice0 = (h / kTeams) * kSubs;        // first 64-K slice of this warp
        const uint32_t row = 32 * q + lane;                  // W row within the block
        const uint32_t taddr = tmem + ((32 * q) << 16) + slice0 * 32;
        const uint32_t n_units = u1 - u0;
        for (uint32_t i = team; i < n_units; i += kTeams) {
            // i-th unit of this CTA: weight stage i % WST, A buffer i % kABufs
            const uint32_t stage = i % WST, phase = (i / WST) & 1u;
            const uint32_t abuf = i % kABufs, aphase = (i / kABufs) & 1u;
            bool ok = mbar_wait(&s.wfull[stage], phase) && !aborted(s);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0 && !aborted(s)) fail(s, err, kDetailDq | stage);
                break;
            }
            // packed W: two swizzled 16-byte chunks of this row per 64-K slice; scales: one
            // 4-byte word of the blocked scale tile per slice
            const uint8_t* wrow = s.w[stage] + row * 128;
            uint4 pk[2 * kSubs];
            uint32_t sc[kSubs];
#pragma unroll
            for (uint32_t j = 0; j < kSubs; ++j) {
#pragma unroll
                for (uint32_t c2 = 0; c2 < 2; ++c2) {
                    const uint32_t c = 2 * (slice0 + j) + c2;
                    pk[2 * j + c2] = *reinterpret_cast<const uint4*>(wrow + ((c ^ (row & 7)) << 4));
                }
                sc[j] = *reinterpret_cast<const uint32_t*>(
                    s.sf[stage] + (slice0 + j) * 512 + (row & 31) * 16 + (row >> 5) * 4);
            }
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive(&s.wempty[stage]);
            bool okA = mbar_wait(&s.aempty[abuf], aphase ^ 1u);
            okA = __all_sync(0xffffffffu, okA);
            if (!okA) {
                if (lane == 0) fail(s, err, kDetailDq | 0x40);
                break;
            }
            t5::fence_after_thread_sync();
#pragma unroll
            for (uint32_t j = 0; j < kSubs; ++j) {
                // dequantise 64 elements into 32 f16x2 words (exact: e2m1 x e4m3 fits f16)
                uint32_t out[32];
#pragma unroll
                for (uint32_t c2 = 0; c2 < 2; ++c2) {
                    // chunk c2 covers 32 K elements: scale bytes 2 c2 and 2 c2 + 1 of the word
                    const uint32_t sbytes = (sc[j] >> (16 * c2)) & 0xFFFFu;
                    uint32_t s2;
                    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(s2) : "h"(static_cast<uint16_t>(sbytes)));
                    const uint32_t slo = __byte_perm(s2, 0, 0x1010);  // scale of the first 16
                    const uint32_t shi = __byte_perm(s2, 0, 0x3232);  // scale of the next 16
                    const uint4 v = pk[2 * j + c2];
                    const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (uint32_t k = 0; k < 4; ++k)
                        dequant8(wv[k], k < 2 ? slo : shi, &out[c2 * 16 + k * 4]);
                }
                tmem_st_x32(taddr + abuf * kACols + 32 * j, out);
            }
            tmem_wait_st();
            t5::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive(&s.afull[abuf]);
        }
    } else if (warp >= kEpiWarp) {
        // ---------------- epilogue (warps kEpiWarp .. kEpiWarp + 3) ----------------
        // decode_prep clears y32 and the counters and writes the token factors.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const uint32_t q = warp & 3u;
        const uint32_t row = 32 * q + lane;                    // W row of the block (TMEM lane)
        // the token factors times gw, in shared memory rather than in 16 registers
        float* fac = s.fac[warp - kEpiWarp];
        if (lane < kTok) fac[lane] = __ldcg(wsp.factors + lane) * gw;
        __syncwarp();
        const UnitRuns ord = unit_runs(u0, u1, S, b_first != 0);
        uint32_t n_runs = ord.nruns;
        namespace pd = ptxstd::decode;
        if (out.nranks != 0) {
            // Peer-to-peer output: every rank's stream has passed its readers of the previous
            // step before any of this step's stores reach its y. Waited here, long before the
            // first accumulator is ready, so the wait hides behind the pipeline.
            const uint32_t step = __ldcg(out.sig[out.rank] + pd::kSigStep);
            bool okr = lane >= out.nranks ||
                       wait_counter(out.sig[out.rank] + pd::kSigReady + lane, step);
            okr = __all_sync(0xffffffffu, okr);
            if (!okr) {
                if (lane == 0) fail(s, err, kDetailEpi | 0x40);
                n_runs = 0;  // no stores, no completion signal
            }
        }
        uint32_t dbuf = 0, dphase = 0, sphase = 0;
        const uint32_t e = warp - kEpiWarp;
        const uint32_t G = gridDim.x, c = blockIdx.x;
        for (uint32_t r = 0; r < n_runs; ++r) {
            // one W-block run, in the MMA's order
            uint32_t nb, ks0, cnt;
            unit_run(ord, r, S, nb, ks0, cnt);
            bool ok = mbar_wait(&s.dfull[dbuf], dphase);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) fail(s, err, kDetailEpi | 0x10);
                break;
            }
            t5::fence_after_thread_sync();
            uint32_t acc[kTok];
            t5::ld_32x32b_x16(tmem + ((32 * q) << 16) + kDCol + dbuf * kTok, acc);
            t5::wait_ld();
            t5::fence_before_thread_sync();
            __syncwarp();
            if (lane == 0) ptxstd::mbar_arrive(&s.dempty[dbuf]);
            if (++dbuf == kDBufs) {
                dbuf = 0;
                dphase ^= 1u;
            }
            // this row's 16 token sums over the segment, with the token factors applied
            float p[kTok];
#pragma unroll
            for (uint32_t t = 0; t < kTok; ++t) p[t] = __uint_as_float(acc[t]) * fac[t];
            // CTAs c_first .. c_last contribute to block nb; a block that lies inside one CTA's
            // range is stored straight from these registers
            const uint64_t b0 = static_cast<uint64_t>(nb) * S;
            const uint32_t c_first = unit_owner(U, G, b0), c_last = unit_owner(U, G, b0 + S - 1);
            bool store = c_first == c_last;
            if (!store) {
                // A shared block: this CTA's partial goes to its slot (0 for the segment its range
                // starts in, 1 otherwise); the CTA that arrives last sums every contributor's
                // partial in the order c_first .. c_last, so the result does not depend on which
                // CTA finishes last.
                const uint32_t side = unit_begin(U, G, c) >= b0 ? 0u : 1u;
                float4* slot = reinterpret_cast<float4*>(
                    wsp.slots + ((static_cast<size_t>(c) * 2 + side) * BM + row) * kTok);
#pragma unroll
                for (uint32_t i = 0; i < kTok / 4; ++i)
                    __stcg(slot + i, make_float4(p[4 * i], p[4 * i + 1], p[4 * i + 2], p[4 * i + 3]));
                ptxstd::fence_acq_rel_gpu();
                __syncwarp();
                // All four warps have written (segA); the first counts this CTA in and tells the
                // others whether it completes the block (segB). mbarriers rather than bar.sync so
                // that every wait stays bounded.
                if (lane == 0) ptxstd::mbar_arrive(&s.segA);
                if (warp == kEpiWarp) {
                    bool okA = mbar_wait(&s.segA, sphase);
                    okA = __all_sync(0xffffffffu, okA);
                    if (!okA) {
                        if (lane == 0) fail(s, err, kDetailEpi | 0x20);
                        break;
                    }
                    if (lane == 0) {
                        const uint32_t before = atomicAdd(wsp.counters + nb, 1u);
                        *reinterpret_cast<volatile uint32_t*>(&s.finalize) =
                            (before + 1 == c_last - c_first + 1) ? 1u : 0u;
                        ptxstd::mbar_arrive(&s.segB);
                    }
                }
                bool okB = mbar_wait(&s.segB, sphase);
                okB = __all_sync(0xffffffffu, okB);
                if (!okB) {
                    if (lane == 0) fail(s, err, kDetailEpi | 0x30);
                    break;
                }
                sphase ^= 1u;
                store = *reinterpret_cast<volatile uint32_t*>(&s.finalize) != 0u;
                if (store) {
                    ptxstd::fence_acq_rel_gpu();
                    float sum[kTok];
#pragma unroll
                    for (uint32_t t = 0; t < kTok; ++t) sum[t] = 0.0f;
                    // every contributor's partial from its slot, this CTA's own included, added
                    // in contributor order; up to kFinMax rows at a time are fetched together
                    // into this thread's shared-memory staging rows, so they cost one round trip
                    for (uint32_t cb = c_first; cb <= c_last; cb += kFinMax) {
                        const uint32_t nc = min(kFinMax, c_last - cb + 1);
                        for (uint32_t j = 0; j < nc; ++j) {
                            const uint32_t cc = cb + j;
                            const uint32_t sd = unit_begin(U, G, cc) >= b0 ? 0u : 1u;
                            const float4* src = reinterpret_cast<const float4*>(
                                wsp.slots + ((static_cast<size_t>(cc) * 2 + sd) * BM + row) * kTok);
#pragma unroll
                            for (uint32_t i = 0; i < kTok / 4; ++i)
                                cp_async_16(&s.fin[j][row][i], src + i);
                        }
                        cp_async_wait_all();
                        for (uint32_t j = 0; j < nc; ++j) {
#pragma unroll
                            for (uint32_t i = 0; i < kTok / 4; ++i) {
                                const float4 f = s.fin[j][row][i];
                                sum[4 * i] += f.x;
                                sum[4 * i + 1] += f.y;
                                sum[4 * i + 2] += f.z;
                                sum[4 * i + 3] += f.w;
                            }
                        }
                    }
#pragma unroll
                    for (uint32_t t = 0; t < kTok; ++t) p[t] = sum[t];
                }
            }
            if (store) {
                // this warp's 32 block rows (= 32 output columns) x 16 tokens, as bf16, into its
                // tile, then 16 tokens x 32 columns = 64 chunks of 8 columns; lane takes chunks lane
                // and lane + 32 (token ch / 4, columns 8 (ch % 4) ..) -> 16-byte stores into y[t][..]
                // of every output (this GPU's only, or every rank's over NVLink)
#pragma unroll
                for (uint32_t t = 0; t < kTok; t += 2) {
                    const uint32_t pk = dt::bf16x2_from_f32(p[t], p[t + 1]);
                    s.ytile[e][t][lane] = static_cast<uint16_t>(pk);
                    s.ytile[e][t + 1][lane] = static_cast<uint16_t>(pk >> 16);
                }
                __syncwarp();
                const size_t c0 = out.col0 + static_cast<size_t>(nb) * BM + 32 * q;
                const uint32_t nout = out.nranks != 0 ? out.nranks : 1u;
#pragma unroll
                for (uint32_t h = 0; h < 2; ++h) {
                    const uint32_t ch = lane + 32 * h, t = ch >> 2, g = ch & 3u;
                    if (t >= M) continue;
                    const uint4 v = *reinterpret_cast<const uint4*>(&s.ytile[e][t][8 * g]);
                    const size_t off = static_cast<size_t>(t) * out.ldy + c0 + 8 * g;
                    for (uint32_t r = 0; r < nout; ++r)
                        *reinterpret_cast<uint4*>(out.y[r] + off) = v;
                }
                __syncwarp();
            }
        }
    }
    t5::fence_before_thread_sync();
    __syncthreads();
    t5::fence_after_thread_sync();
    if (warp == 1) t5::tmem_dealloc(tmem, kTmemCols);
}

// Kernel 3, peer-to-peer output only. It starts after kernel 2 has completed on this GPU, so
// every store kernel 2 made (into every rank's y) happens before it. Thread r releases them to
// rank r (one system-scope fence, then DONE[this rank] += 1 on rank r), then waits until rank r has
// done the same here for this step. Signalling from a fresh kernel keeps the fence off kernel 2's
// epilogue, where it would wait for the NVLink stores still in flight (measured at about 8 us per
// step on 2 GPUs). A device with an error recorded (a timed-out wait of this step, or any earlier
// failure not yet read) withholds its signal, so that every rank's wait fails too instead of
// reading an incomplete y.
__global__ void __launch_bounds__(32) decode_done_kernel(const ptxstd::decode::Out out,
                                                         uint32_t* err) {
    namespace pd = ptxstd::decode;
    const uint32_t r = threadIdx.x;
    if (r >= out.nranks) return;
    if (*reinterpret_cast<volatile uint32_t*>(err) == 0u) {
        ptxstd::fence_acq_rel_sys();
        atomicAdd_system(out.sig[r] + pd::kSigDone + out.rank, 1u);
    }
    const uint32_t step = __ldcg(out.sig[out.rank] + pd::kSigStep);
    if (!wait_counter(out.sig[out.rank] + pd::kSigDone + r, step))
        ptxstd::record_error(err, PTXSTD_ETIMEOUT, kDetailEpi | 0x50 | r);
}

int launch_decode(const uint16_t* x, const uint8_t* W, const uint8_t* sfW, float gw,
                  const ptxstd::decode::Out& out, int64_t M, int64_t N, int64_t K, uint8_t* ws,
                  cudaStream_t stream) {
    CUtensorMap tw;
    int st = ptxstd::make_tmap_2d(&tw, W, CU_TENSOR_MAP_DATA_TYPE_UINT8, K / 2, N, K / 2,
                                  BKS / 2, BM, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = ptxstd::set_max_dynamic_smem(reinterpret_cast<const void*>(gemm_decode_kernel),
                                      static_cast<int>(kSmemBytes));
    if (st) return st;
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    const uint32_t grid = static_cast<uint32_t>(decode_grid(static_cast<size_t>(N),
                                                             static_cast<size_t>(K)));
    if (grid == 0) return PTXSTD_ECUDA;
    decode_prep_kernel<<<kTok, kPrepThreads, 0, stream>>>(x, static_cast<uint32_t>(M),
                                                         static_cast<uint32_t>(K), ws,
                                                         static_cast<uint32_t>(N), grid, out);
    st = ptxstd::launch_status();
    if (st) return st;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // whole blocks first only when every CTA holds at least two blocks' worth of units
    const uint64_t units = static_cast<uint64_t>(N / BM) * static_cast<uint64_t>(K / BKS);
    const uint32_t b_first = units / grid >= 2ull * static_cast<uint64_t>(K / BKS) ? 1u : 0u;
    if (cudaLaunchKernelEx(&cfg, gemm_decode_kernel, tw, sfW, ws, out, static_cast<uint32_t>(M),
                           static_cast<uint32_t>(N), static_cast<uint32_t>(K), gw,
                           err, b_first) != cudaSuccess)
        return PTXSTD_ECUDA;
    st = ptxstd::launch_status();
    if (st || out.nranks == 0) return st;
    decode_done_kernel<<<1, 32, 0, stream>>>(out, err);
    return ptxstd::launch_status();
}

// Shape, pointer and alignment checks shared by every decode entry point.
int check_args(const uint16_t* x, const uint8_t* W, const uint8_t* sfW, float gw, int64_t M,
               int64_t N, int64_t K, const void* ws) {
    if (M <= 0 || M > static_cast<int64_t>(kTok) || N <= 0 || K <= 0 || N % BM || K % BKS)
        return PTXSTD_EINVAL;
    if (N >= (1ll << 31) || K >= (1ll << 30)) return PTXSTD_EINVAL;
    if (!(gw == gw) || !x || !W || !sfW || !ws) return PTXSTD_EINVAL;
    if (!ptxstd::aligned16(x) || !ptxstd::aligned16(W) || !ptxstd::aligned16(sfW) ||
        (reinterpret_cast<uintptr_t>(ws) & 1023u))
        return PTXSTD_EINVAL;
    return PTXSTD_OK;
}

ptxstd::decode::Out local_out(uint16_t* y, int64_t N) {
    ptxstd::decode::Out o = {};
    o.y[0] = y;
    o.ldy = static_cast<uint64_t>(N);
    return o;
}

}  // namespace

int ptxstd::decode::launch(const uint16_t* x, const uint8_t* W, const uint8_t* sfW, float gw,
                           const Out& out, int64_t M, int64_t N, int64_t K, uint8_t* ws,
                           cudaStream_t stream) {
    if (check_args(x, W, sfW, gw, M, N, K, ws) || out.nranks > kMaxRanks ||
        (out.nranks != 0 && out.rank >= out.nranks) || out.ldy < out.col0 + N ||
        out.ldy % 8 != 0 || out.col0 % 8 != 0)  // 16-byte output chunks
        return PTXSTD_EINVAL;
    for (uint32_t r = 0; r < (out.nranks != 0 ? out.nranks : 1u); ++r)
        if (!out.y[r] || !ptxstd::aligned16(out.y[r]) || (out.nranks != 0 && !out.sig[r]))
            return PTXSTD_EINVAL;
    return launch_decode(x, W, sfW, gw, out, M, N, K, ws, stream);
}

extern "C" {

size_t ptxstd_gemm_decode_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0) return 0;
    return decode_ws_bytes(static_cast<size_t>(N), static_cast<size_t>(K));
}

int ptxstd_gemm_decode(const uint16_t* d_x, const uint8_t* d_w, const uint8_t* d_sfw, float gw,
                       uint16_t* d_y, int64_t M, int64_t N, int64_t K, void* d_workspace,
                       size_t workspace_bytes, ptxstd_stream stream) {
    if (check_args(d_x, d_w, d_sfw, gw, M, N, K, d_workspace) || !d_y || !ptxstd::aligned16(d_y))
        return PTXSTD_EINVAL;
    if (workspace_bytes < decode_ws_bytes(static_cast<size_t>(N), static_cast<size_t>(K)))
        return PTXSTD_EINVAL;
    return launch_decode(d_x, d_w, d_sfw, gw, local_out(d_y, N), M, N, K,
                         static_cast<uint8_t*>(d_workspace),
                         static_cast<cudaStream_t>(stream));
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Decode GEMM without allocation.
//
// Some callers cannot allocate the workspace that ptxstd_gemm_decode asks for: a serving loop
// whose device-memory plan is fixed at start-up must not call cudaMalloc / cudaFree per request
// (both can synchronise the device and fragment a carefully sized pool), and a thin C or Rust
// binding may own only the input and output buffers, with no allocator of its own to create a
// workspace. For them the scratch lives in this file-scope device array instead. The array
// belongs to this file's device module, which the CUDA runtime loads onto a device (lazily, by
// default) at the first use of the module there: the first call of either decode entry point on
// that device. From then until the process exits that device holds the 4 MiB, for the regular
// ptxstd_gemm_decode as much as for this one. A caller that must not reserve memory while serving
// makes one warm-up call per device at start-up, which also does the address look-up below.
//
// In host code `g_decode_scratch` is only a host-side stand-in for the symbol, not a device
// address; its device address is fetched with cudaGetSymbolAddress, once per device, with that
// device current, on the first call on that device, and kept for the life of the process. That
// first call should come before any stream capture. A device reset (cudaDeviceReset) or a new
// primary context invalidates the kept address; the library does not support calls across one.
// All calls on a device share the one array: decode_prep clears the parts that must start at
// zero on every call, and calls that overlap on the GPU (e.g. on two streams) race on it. The
// array is 1024-byte aligned, the alignment ptxstd_gemm_decode asks of a caller's workspace.
static __device__ __align__(1024) uint8_t g_decode_scratch[PTXSTD_DECODE_NOALLOC_SCRATCH_BYTES];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_ptr[64] = {};

int decode_scratch_address(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return PTXSTD_ECUDA;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_decode_scratch) != cudaSuccess || p == nullptr)
            return PTXSTD_ECUDA;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return PTXSTD_OK;
}

}  // namespace

extern "C" int ptxstd_gemm_decode_noalloc(const uint16_t* d_x, const uint8_t* d_w,
                                          const uint8_t* d_sfw, float gw, uint16_t* d_y,
                                          int64_t M, int64_t N, int64_t K, ptxstd_stream stream) {
    if (M <= 0 || M > static_cast<int64_t>(kTok) || N <= 0 || K <= 0 || N % BM || K % BKS)
        return PTXSTD_EINVAL;
    if (N >= (1ll << 31) || K >= (1ll << 30)) return PTXSTD_EINVAL;
    if (!(gw == gw) || !d_x || !d_w || !d_sfw || !d_y) return PTXSTD_EINVAL;
    if (!ptxstd::aligned16(d_x) || !ptxstd::aligned16(d_w) || !ptxstd::aligned16(d_sfw) ||
        !ptxstd::aligned16(d_y))
        return PTXSTD_EINVAL;
    // The shape's scratch must fit the fixed array.
    if (decode_ws_bytes(static_cast<size_t>(N), static_cast<size_t>(K)) >
        static_cast<size_t>(PTXSTD_DECODE_NOALLOC_SCRATCH_BYTES))
        return PTXSTD_EINVAL;
    void* scratch = nullptr;
    const int st = decode_scratch_address(&scratch);
    if (st) return st;
    return launch_decode(d_x, d_w, d_sfw, gw, local_out(d_y, N), M, N, K,
                         static_cast<uint8_t*>(scratch),
                         static_cast<cudaStream_t>(stream));
}

// tcgen05 for sm_100a: the descriptor encodings of ptx-std's src/tcgen05/descriptor.rs as
// constexpr host+device C++, and the device instructions of src/tcgen05/{alloc,mma,copy,ld_st,
// sync}.rs as inline PTX. All instructions here use .cta_group::1 (one kernel, one CTA group, as
// src/tcgen05/mod.rs:40-44 requires).
#pragma once

#include <cstdint>

#include "common.cuh"

#if defined(__CUDACC__)
#define PTXSTD_HD __host__ __device__
#else
#define PTXSTD_HD
#endif

namespace ptxstd::tcgen05 {

// ---- enums (src/tcgen05/descriptor.rs:31-392, src/tcgen05/mod.rs:322-337) ----------------------
enum class MmaKind : int { F16 = 0, Tf32 = 1, F8f6f4 = 2, I8 = 3, Mxf8f6f4 = 4, Mxf4 = 5,
                           Mxf4nvf4 = 6 };
enum class Swizzle : uint32_t { None = 0, Bytes128Atom32B = 1, Bytes128 = 2, Bytes64 = 4,
                                Bytes32 = 6 };
enum class Major : uint32_t { K = 0, Mn = 1 };
enum class F16Type : uint32_t { F16 = 0, Bf16 = 1 };
enum class FloatAcc : uint32_t { F16 = 0, F32 = 1 };
enum class F8f6f4Type : uint32_t { E4m3 = 0, E5m2 = 1, E2m3 = 3, E3m2 = 4, E2m1 = 5 };
enum class I8Type : uint32_t { U8 = 0, S8 = 1 };
enum class Nvf4ScaleType : uint32_t { Ue4m3 = 0, Ue8m0 = 1, Ue5m3 = 2 };

// Setter fields of InstrDescriptor (descriptor.rs:400-411): bit position and width.
enum class IdescField : int {
    Sparsity = 0,          // bit 2, all kinds
    SparsitySelector = 1,  // bits 0-1, F16 / Tf32
    Saturate = 2,          // bit 3, I8
    NegateA = 3,           // bit 13, all but I8
    NegateB = 4,           // bit 14, all but I8
    MajorA = 5,            // bit 15, F16 Tf32 F8f6f4 I8 Mxf8f6f4
    MajorB = 6,            // bit 16, same kinds
    MaxBShift = 7,         // bits 30-31, F16 Tf32 F8f6f4 I8
    ScaleAId = 8,          // bits 29-30, block-scaled kinds
    ScaleBId = 9,          // bits 4-5, block-scaled kinds
    K = 10,                // bit 31, Mxf4 / Mxf4nvf4
};

// ---- instruction descriptor -------------------------------------------------------------------
// Each encoder returns false where the reference's const fn asserts.
PTXSTD_HD constexpr bool encode_n(uint32_t n, uint32_t& f) {
    if (n % 8 != 0 || n < 8 || n > 256) return false;  // descriptor.rs:450-457
    f = (n >> 3) << 17;
    return true;
}
PTXSTD_HD constexpr bool encode_m(uint32_t m, uint32_t& f) {
    if (m % 16 != 0 || m < 16 || m > 256) return false;  // descriptor.rs:460-467
    f = (m >> 4) << 24;
    return true;
}
PTXSTD_HD constexpr bool encode_m_block_scaled(uint32_t m, uint32_t& f) {
    if (m != 128 && m != 256) return false;  // descriptor.rs:470-476
    f = (m >> 7) << 27;
    return true;
}

// InstrDescriptor::<F16 | F8f6f4>::new: d << 4 | a << 7 | b << 10 | N | M (descriptor.rs:520-564).
PTXSTD_HD constexpr bool idesc_dense(uint32_t a, uint32_t b, uint32_t d, uint32_t m, uint32_t n,
                                     uint32_t& out) {
    uint32_t fm = 0, fn = 0;
    if (!encode_m(m, fm) || !encode_n(n, fn)) return false;
    out = (d << 4) | (a << 7) | (b << 10) | fn | fm;
    return true;
}
// InstrDescriptor::<Mxf8f6f4>::new: ue8m0 scales (1 << 23) (descriptor.rs:601-611).
PTXSTD_HD constexpr bool idesc_mxf8f6f4(uint32_t a, uint32_t b, uint32_t m, uint32_t n,
                                        uint32_t& out) {
    uint32_t fm = 0, fn = 0;
    if (!encode_m_block_scaled(m, fm) || !encode_n(n, fn)) return false;
    out = (a << 7) | (b << 10) | (1u << 23) | fn | fm;
    return true;
}
// InstrDescriptor::<Mxf4nvf4>::new: e2m1 A and B, scale type << 23 (descriptor.rs:644-653).
PTXSTD_HD constexpr bool idesc_mxf4nvf4(uint32_t scale_type, uint32_t m, uint32_t n,
                                        uint32_t& out) {
    uint32_t fm = 0, fn = 0;
    if (scale_type > 2 || !encode_m_block_scaled(m, fm) || !encode_n(n, fn)) return false;
    out = (1u << 7) | (1u << 10) | (scale_type << 23) | fn | fm;
    return true;
}
// with_field (descriptor.rs:494-498).
PTXSTD_HD constexpr bool idesc_with_field(uint32_t desc, uint32_t shift, uint32_t width,
                                          uint32_t value, uint32_t& out) {
    if (value >= (1u << width)) return false;
    const uint32_t mask = ((1u << width) - 1u) << shift;
    out = (desc & ~mask) | (value << shift);
    return true;
}
// The setters of each kind (descriptor.rs:400-411, :660-813): field -> (shift, width), or false
// when the kind has no such setter.
PTXSTD_HD constexpr bool idesc_field_of(MmaKind k, IdescField f, uint32_t& shift,
                                        uint32_t& width) {
    const bool scaled = k == MmaKind::Mxf8f6f4 || k == MmaKind::Mxf4 || k == MmaKind::Mxf4nvf4;
    switch (f) {
    case IdescField::Sparsity: shift = 2; width = 1; return true;
    case IdescField::SparsitySelector:
        shift = 0; width = 2; return k == MmaKind::F16 || k == MmaKind::Tf32;
    case IdescField::Saturate: shift = 3; width = 1; return k == MmaKind::I8;
    case IdescField::NegateA: shift = 13; width = 1; return k != MmaKind::I8;
    case IdescField::NegateB: shift = 14; width = 1; return k != MmaKind::I8;
    case IdescField::MajorA:
        shift = 15; width = 1; return k != MmaKind::Mxf4 && k != MmaKind::Mxf4nvf4;
    case IdescField::MajorB:
        shift = 16; width = 1; return k != MmaKind::Mxf4 && k != MmaKind::Mxf4nvf4;
    case IdescField::MaxBShift: shift = 30; width = 2; return !scaled;
    case IdescField::ScaleAId: shift = 29; width = 2; return scaled;
    case IdescField::ScaleBId: shift = 4; width = 2; return scaled;
    case IdescField::K: shift = 31; width = 1; return k == MmaKind::Mxf4 || k == MmaKind::Mxf4nvf4;
    }
    return false;
}

// ---- shared memory descriptor (descriptor.rs:47-250) -------------------------------------------
PTXSTD_HD constexpr bool smem_offset_field(uint32_t bytes, uint64_t& f) {
    if (bytes % 16 != 0 || bytes > 0x3FFFFu) return false;  // descriptor.rs:100-108
    f = bytes >> 4;
    return true;
}
PTXSTD_HD constexpr bool valid_swizzle(uint32_t s) {
    return s == 0 || s == 1 || s == 2 || s == 4 || s == 6;
}
// from_shared_address (descriptor.rs:152-162): start >> 4 in bits 0-13, LBO >> 4 at 16, SBO >> 4
// at 32, the constant 0b001 at 46, swizzle at 61.
PTXSTD_HD constexpr bool smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo, uint32_t swz,
                                   uint64_t& out) {
    uint64_t l = 0, s = 0;
    if (!valid_swizzle(swz) || !smem_offset_field(lbo, l) || !smem_offset_field(sbo, s))
        return false;
    out = static_cast<uint64_t>((start & 0x3FFFFu) >> 4) | (l << 16) | (s << 32) | (1ull << 46) |
          (static_cast<uint64_t>(swz) << 61);
    return true;
}
// Fast device form for a K-major operand with 128-byte swizzling: LBO 16 (unused), SBO 1024
// (8 rows x 128 bytes), the same encoding as smem_desc(start, 16, 1024, Bytes128).
PTXSTD_HD constexpr uint64_t smem_desc_k128(uint32_t start) {
    return static_cast<uint64_t>((start & 0x3FFFFu) >> 4) | (1ull << 16) | (64ull << 32) |
           (1ull << 46) | (2ull << 61);
}
// Descriptor of an unswizzled K-major 8-row core-matrix source (used for tcgen05.cp of scale
// factors): 16-byte rows, SBO = 128 bytes between 8-row groups, LBO unused.
PTXSTD_HD constexpr uint64_t smem_desc_nosw(uint32_t start, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((start & 0x3FFFFu) >> 4) |
           (static_cast<uint64_t>(lbo >> 4) << 16) | (static_cast<uint64_t>(sbo >> 4) << 32) |
           (1ull << 46);
}
// with_base_offset (descriptor.rs:176-183).
PTXSTD_HD constexpr bool smem_desc_with_base_offset(uint64_t d, uint32_t bo, uint64_t& out) {
    if (bo >= 8) return false;
    if (bo != 0 && (d & (1ull << 52))) return false;
    out = (d & ~(7ull << 49)) | (static_cast<uint64_t>(bo) << 49);
    return true;
}
// add_start_bytes (descriptor.rs:231-237).
PTXSTD_HD constexpr bool smem_desc_add_start_bytes(uint64_t d, uint32_t bytes, uint64_t& out) {
    if (bytes % 16 != 0) return false;
    out = d + (bytes >> 4);
    return true;
}

// ---- zero-column mask (descriptor.rs:820-942) ----------------------------------------------
PTXSTD_HD constexpr bool zero_mask_new(uint32_t zeroed, uint32_t used, uint64_t& out) {
    if (zeroed < 1 || zeroed > 256 || used < 1 || used > 256) return false;
    out = (1ull << 39) | (static_cast<uint64_t>(zeroed - 1) << 40) |
          (static_cast<uint64_t>(used - 1) << 48);
    return true;
}
PTXSTD_HD constexpr bool zero_mask_with_sub_mask_start(uint64_t m, uint32_t sub, uint32_t span,
                                                       uint32_t count, uint64_t& out) {
    if (sub >= 4 || count >= 256 || span > 1) return false;
    const uint32_t cs = 8 * sub, ss = 32 + sub;
    out = (m & ~((0xFFull << cs) | (1ull << ss))) | (static_cast<uint64_t>(count) << cs) |
          (static_cast<uint64_t>(span) << ss);
    return true;
}
PTXSTD_HD constexpr bool zero_mask_with_column_shift(uint64_t m, uint32_t shift, uint64_t& out) {
    if (shift > 32) return false;
    out = (m & ~(0x3Full << 56)) | (static_cast<uint64_t>(shift) << 56);
    return true;
}

// Compile-time pins against the reference's own known answers
// (examples/tcgen05_ptxas/descriptor.rs:71, :99, :132, :158-160).
namespace detail {
constexpr uint32_t idesc_f8(uint32_t a, uint32_t b, uint32_t d, uint32_t m, uint32_t n) {
    uint32_t o = 0;
    return idesc_dense(a, b, d, m, n, o) ? o : 0xFFFFFFFFu;
}
constexpr uint32_t idesc_nv(uint32_t st, uint32_t m, uint32_t n) {
    uint32_t o = 0;
    return idesc_mxf4nvf4(st, m, n, o) ? o : 0xFFFFFFFFu;
}
constexpr uint64_t sdesc(uint32_t s, uint32_t l, uint32_t b, uint32_t z) {
    uint64_t o = 0;
    return smem_desc(s, l, b, z, o) ? o : ~0ull;
}
}  // namespace detail
static_assert(detail::idesc_f8(0, 1, 1, 128, 128) == 0x08200410u, "F8f6f4 known answer");
static_assert(detail::idesc_nv(0, 128, 64) == 0x08100480u, "Mxf4nvf4 ue4m3 known answer");
static_assert(detail::idesc_nv(1, 128, 64) == 0x08900480u, "Mxf4nvf4 ue8m0 known answer");
static_assert(detail::sdesc(0x1230, 16, 1024, 2) == 0x4000404000010123ull, "smem known answer");
static_assert(smem_desc_k128(0x1230) == 0x4000404000010123ull, "fast K128 form");

#if defined(__CUDACC__)
// ---- device instructions -----------------------------------------------------------------
// alloc / relinquish / dealloc (src/tcgen05/alloc.rs:48, :136, :101): warp-collective.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// fence::before_thread_sync / after_thread_sync (src/tcgen05/sync.rs:22, :39).
__device__ __forceinline__ void fence_before_thread_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_thread_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// commit (src/tcgen05/sync.rs:70-80): the mbarrier arrives once all prior async tcgen05
// operations of this thread have completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

// mma kind::f8f6f4 (src/tcgen05/mma.rs:434-453): D[tmem] (+)= A[smem] * B[smem]^T.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// mma kind::f16 (bf16 operands, f32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// mma_block_scaled kind::mxf4nvf4 .block16 (= .scale_vec::4X) (src/tcgen05/mma.rs:698-724).
__device__ __forceinline__ void mma_mxf4nvf4_block16(uint32_t d_tmem, uint64_t a_desc,
                                                     uint64_t b_desc, uint32_t idesc,
                                                     uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], "
        "[%5], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
        : "memory");
}
// mma_block_scaled kind::mxf8f6f4 .block32 (= .scale_vec::1X).
__device__ __forceinline__ void mma_mxf8f6f4_block32(uint32_t d_tmem, uint64_t a_desc,
                                                     uint64_t b_desc, uint32_t idesc,
                                                     uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale.block32 [%0], %1, %2, %3, [%4], "
        "[%5], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
        : "memory");
}

// copy with CopyShape::S32x128bWarpx4 (src/tcgen05/copy.rs:29-30, :76-116): 32 rows x 16 bytes
// of smem -> 4 columns of every 32-lane quarter of TMEM.
__device__ __forceinline__ void cp_32x128b_warpx4(uint32_t taddr, uint64_t src_desc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc)
                 : "memory");
}

// ---- CtaGroup::Two forms: one thread of the CTA pair issues for both CTAs ------------------
// (src/tcgen05/mod.rs:40-57). A kernel uses either these or the cta_group::1 forms, never both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// commit::<Two> to an mbarrier given as a .shared::cluster address (own or peer CTA).
__device__ __forceinline__ void commit_pair(uint32_t cluster_bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            cluster_bar)
        : "memory");
}
// mma::<Two> kind::f8f6f4: M = 256 rows over the pair (128 from each CTA's smem), B's N rows split
// across the two CTAs' smem, D in both CTAs' TMEM at the same address.
__device__ __forceinline__ void mma_f8f6f4_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void mma_mxf4nvf4_block16_pair(uint32_t d_tmem, uint64_t a_desc,
                                                          uint64_t b_desc, uint32_t idesc,
                                                          uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %6, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%4], "
        "[%5], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
        : "memory");
}
// copy::<Two, S32x128bWarpx4>: each CTA of the pair copies from its own smem to its own TMEM.
__device__ __forceinline__ void cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t src_desc) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(src_desc)
                 : "memory");
}
// copy::<Two, S128x128b> (src/tcgen05/copy.rs): 128 rows x 16 bytes of each CTA's smem -> 4
// columns of that CTA's 128 lanes (row i to lane i).
__device__ __forceinline__ void cp_128x128b_pair(uint32_t taddr, uint64_t src_desc) {
    asm volatile("tcgen05.cp.cta_group::2.128x128b [%0], %1;" ::"r"(taddr), "l"(src_desc)
                 : "memory");
}
// mma_block_scaled_sparse::<Two, _, Block32, Mxf8f6f4> (src/tcgen05/mma.rs:725-777): A is 2:4
// sparse (the descriptor addresses the compressed K/2 values), its metadata at [meta] in TMEM;
// one MMA covers K = 64 logical elements and takes one scale byte of each operand.
__device__ __forceinline__ void mma_sp_mxf8f6f4_block32_pair(uint32_t d_tmem, uint64_t a_desc,
                                                             uint64_t b_desc, uint32_t meta_tmem,
                                                             uint32_t idesc, uint32_t sfa_tmem,
                                                             uint32_t sfb_tmem,
                                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %7, 0;\n\t"
        "tcgen05.mma.sp.cta_group::2.kind::mxf8f6f4.block_scale.block32 [%0], %1, %2, [%3], %4, "
        "[%5], [%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(meta_tmem), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem),
        "r"(accumulate)
        : "memory");
}

// load::<S32x32b, x32> (src/tcgen05/ld_st.rs:252-300): lane (32 * (warp % 4) + laneid), 32
// consecutive columns -> 32 registers.
__device__ __forceinline__ void ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
// load::<S32x32b, x8>.
__device__ __forceinline__ void ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7])
        : "r"(taddr)
        : "memory");
}
// copy::<S128x256b, B6x16P32> / <S128x256b, B4x16P64> (src/tcgen05/copy.rs:32-46, :76-116):
// 128 rows x 32 bytes of packed 6-bit (4-bit) elements, 16 per 16-byte group, into 128 lanes x
// 256 bits of 8-bit containers.
__device__ __forceinline__ void cp_128x256b_b6x16_p32(uint32_t taddr, uint64_t src_desc) {
    asm volatile("tcgen05.cp.cta_group::1.128x256b.b8x16.b6x16_p32 [%0], %1;" ::"r"(taddr),
                 "l"(src_desc)
                 : "memory");
}
__device__ __forceinline__ void cp_128x256b_b4x16_p64(uint32_t taddr, uint64_t src_desc) {
    asm volatile("tcgen05.cp.cta_group::1.128x256b.b8x16.b4x16_p64 [%0], %1;" ::"r"(taddr),
                 "l"(src_desc)
                 : "memory");
}
// load::<S32x32b, x16>.
__device__ __forceinline__ void ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
// wait_load (src/tcgen05/ld_st.rs:648).
__device__ __forceinline__ void wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
#endif  // __CUDACC__

}  // namespace ptxstd::tcgen05

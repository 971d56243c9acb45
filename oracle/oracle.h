/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of caelunshun/ptx-std's narrow-float semantics, of the block-scale
 * recipes built on them, of its tcgen05 descriptor encodings, and an f64 GEMM over decoded
 * values. Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it, and
 * only as the checker (or as the timed CPU baseline). Nothing in the product links it.
 *
 * Parity pins:
 *   - descriptor encoders: the reference's compile-time known answers
 *     (examples/tcgen05_ptxas/descriptor.rs:22-234), extracted to tests/golden/;
 *   - decode: the reference's named bit-pattern constants (src/data_types/float8.rs:22-41,
 *     :80-103, :153-162; src/data_types/float4.rs:26-42);
 *   - encode: the reference's encoders are the hardware `cvt` instructions (the core::arch::nvptx
 *     intrinsics of the rustc fork `nvptx-ext`, src/data_types/narrow.rs:156-182, :600-646), so
 *     they are pinned by running those same instructions over all 2^32 f32 inputs on a B200 and
 *     committing per-chunk digests of the outputs (tests/golden/cvt_sweep_digests.json).
 */
#ifndef PTXSTD_ORACLE_H
#define PTXSTD_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- formats ------------------------------------------------------------------------------ */
enum ptxo_format {
    PTXO_E4M3 = 0, /* FP8 E4M3, NaN-only specials, max 448 (src/data_types/float8.rs:13-42) */
    PTXO_E5M2 = 1, /* FP8 E5M2, IEEE specials, max 57344 (src/data_types/float8.rs:70-133) */
    PTXO_E2M1 = 2, /* FP4 E2M1, no specials, max 6 (src/data_types/float4.rs:14-43) */
    PTXO_E2M3 = 3, /* FP6 E2M3, no specials, max 7.5, one value per byte (src/data_types/float6.rs) */
    PTXO_E3M2 = 4, /* FP6 E3M2, no specials, max 28, one value per byte (src/data_types/float6.rs) */
};

/* Exact soft decode (src/data_types/vector.rs:61-95). specials: 0 none, 1 IEEE, 2 NaN-only. */
float ptxo_minifloat_to_f32(uint8_t bits, uint32_t exp_bits, uint32_t man_bits, int32_t bias,
                            int specials);
float ptxo_e4m3_to_f32(uint8_t bits);
float ptxo_e5m2_to_f32(uint8_t bits);
float ptxo_e2m1_to_f32(uint8_t nibble);
float ptxo_e2m3_to_f32(uint8_t bits);
float ptxo_e3m2_to_f32(uint8_t bits);
/* UE8M0 decode, 2^(b-127), 0xff NaN (src/data_types/float8.rs:148-152). */
float ptxo_ue8m0_to_f32(uint8_t bits);

/* Decode as the device `to_f32` does it: through f16 (or bf16 for ue8m0), then widened
 * (src/data_types/narrow.rs:292-299, :683-690). Differs from the soft decode only in NaN bits. */
float ptxo_to_f32_via_half(int format, uint8_t bits);
float ptxo_ue8m0_to_f32_via_bf16(uint8_t bits);

/* Round-to-nearest-even, .satfinite, optional .relu encode of one f32
 * (src/data_types/narrow.rs:125-130 for the semantics). */
uint8_t ptxo_f32_to_e4m3(float x, int relu);
uint8_t ptxo_f32_to_e5m2(float x, int relu);
uint8_t ptxo_f32_to_e2m1(float x, int relu); /* returns a nibble */
uint8_t ptxo_f32_to_narrow(int format, float x, int relu);
/* UE8M0 encode, rounding toward zero (rnd_up = 0) or toward +inf (rnd_up = 1), with or without
 * .satfinite (src/data_types/narrow.rs:585-593, :600-617). */
uint8_t ptxo_f32_to_ue8m0(float x, int rnd_up, int satfinite);

/* bf16 helpers (src/data_types/bfloat16.rs:76-86): RNE f32 -> bf16 and the exact widening. */
uint16_t ptxo_f32_to_bf16(float x);
/* cvt.rn{.relu}{.satfinite}.bf16x2.f32 of one value (bfloat16.rs:446-454): RN; every NaN becomes
 * 0x7FFF; relu maps negative results and -0 to +0; satfinite clamps overflow to 0x7F7F / 0xFF7F. */
uint16_t ptxo_f32_to_bf16_mode(float x, int relu, int satfinite);
/* Exact f16 bit pattern of a narrow code (format PTXO_E4M3 .. PTXO_E3M2; E2M1 as a nibble); NaN
 * codes give 0x7FFF. */
uint16_t ptxo_narrow_to_f16(int format, uint8_t code);
float ptxo_bf16_to_f32(uint16_t h);

/* to_bf16_scaled::<RELU, OVERFLOW> (src/data_types/narrow.rs:314-330, :444-465): the exact
 * value of a narrow code (format PTXO_E4M3 .. PTXO_E3M2; E2M1 as a nibble) times 2^(scale-127),
 * rounded to bf16 (RN, subnormals kept); relu maps negative results (and -0) to +0; satfinite
 * clamps results past the finite range to the largest finite bf16 of matching sign, otherwise
 * they become infinity; a NaN code or the NaN scale 0xff gives 0x7FFF. */
uint16_t ptxo_to_bf16_scaled(int format, uint8_t code, uint8_t scale, int relu, int satfinite);
/* Element i of codes (E2M1: nibble i % 2 of byte i / 2) with scales[i / block]. */
void ptxo_to_bf16_scaled_array(int format, const uint8_t* codes, const uint8_t* scales,
                               uint16_t* out, size_t n, size_t block, int relu, int satfinite,
                               int threads);

/* ---- stochastic rounding (cvt.rs; src/data_types/narrow.rs:217-229, :494-505; bf16
 * src/data_types/bfloat16.rs:456-462, :572-598; f16 src/data_types/float16.rs:589-595, :740-766).
 * One rbits word serves a group of four elements (FP8, FP6, E2M1) or a pair (bf16, f16). Element
 * k of the group takes a random value r of w bits (w = 13 for f16, else 16), assembled from
 * rbits as ptxo_rs_random states. The magnitude is truncated to the target's quantum at its
 * binade (or the subnormal quantum); the discarded part of a quantum, truncated to w bits, plus
 * r carries out of w bits exactly when the magnitude rounds up by one quantum. NaN, infinity,
 * .satfinite and .relu then follow the round-to-nearest path (bf16/f16: every NaN becomes
 * 0x7FFF, and .relu maps any negative result, -0 included, to +0). The reference documents only
 * the carry rule and which half-word feeds which elements; the bit order inside a half and the
 * rule for the discarded bits are fitted to the B200's cvt.rs and pinned over all 2^32 inputs
 * (tests/golden/cvt_sweep_digests.json, variants *_rs*). */
enum ptxo_rs_kind { PTXO_RS_X4 = 0, PTXO_RS_E2M1 = 1, PTXO_RS_BF16 = 2, PTXO_RS_F16 = 3 };
uint32_t ptxo_rs_random(int kind, uint32_t rbits, int k);
/* format: PTXO_E4M3 .. PTXO_E3M2; r: element's random value (ptxo_rs_random). */
uint8_t ptxo_f32_to_narrow_rs(int format, float x, uint32_t r, int relu);
uint16_t ptxo_f32_to_bf16_rs(float x, uint32_t r, int relu, int satfinite);
uint16_t ptxo_f32_to_f16_rs(float x, uint32_t r, int relu, int satfinite);
/* Element i of x with rbits[i / 4] (packed E2M1: n even, element 0 in the low nibble). */
void ptxo_encode_rs_array(int format, const float* x, const uint32_t* rbits, uint8_t* out,
                          size_t n, int relu, int threads);
/* Element i of x with rbits[i / 2]. */
void ptxo_bf16_rs_array(const float* x, const uint32_t* rbits, uint16_t* out, size_t n, int relu,
                        int satfinite, int threads);
void ptxo_f16_rs_array(const float* x, const uint32_t* rbits, uint16_t* out, size_t n, int relu,
                       int satfinite, int threads);
/* Counter-based random bits of the seeded stochastic-rounding quantisers: output i of SplitMix64
 * (Steele, Lea and Flood, OOPSLA 2014) started at `seed`; group g (four consecutive elements of
 * the flat row-major input) takes the low (g even) or high (g odd) word of output g / 2. */
uint64_t ptxo_splitmix64(uint64_t seed, uint64_t i);
uint32_t ptxo_sr_rbits(uint64_t seed, uint64_t group);

/* ---- bulk conversions (multithreaded; threads <= 0 means all hardware threads) ------------- */
/* Element i of x -> out[i] (one code per byte for FP8; packed 2 per byte, element 0 in the low
 * nibble, for E2M1 when format == PTXO_E2M1 and n is even). */
void ptxo_encode_array(int format, const float* x, uint8_t* out, size_t n, int relu, int threads);
void ptxo_decode_array(int format, const uint8_t* codes, float* out, size_t n, int threads);
void ptxo_ue8m0_encode_array(const float* x, uint8_t* out, size_t n, int rnd_up, int satfinite,
                             int threads);

/* Sweep of the f32 bit patterns [base, base + n): encodes every pattern (variant selects
 * format/relu, the ue8m0 rounding, or a stochastic-rounding form) and compares with
 * `device_out`, the device's codes for the same inputs (ptxo_sweep_width bytes per input,
 * little-endian; E2M1 nibbles unpacked). The stochastic variants give input pattern p the random
 * bits ptxo_sr_rbits(PTXO_SWEEP_SEED, p / 4) (p / 2 for bf16/f16), element p % 4 (p % 2) of its
 * group. Returns the number of mismatches and stores up to max_report of them as (input bits,
 * device code, oracle code) triples. base must be a multiple of 4. */
enum ptxo_variant {
    PTXO_V_E4M3 = 0, PTXO_V_E5M2 = 1, PTXO_V_E2M1 = 2,
    PTXO_V_E4M3_RELU = 3, PTXO_V_E5M2_RELU = 4, PTXO_V_E2M1_RELU = 5,
    PTXO_V_UE8M0_RZ = 6, PTXO_V_UE8M0_RP = 7,
    PTXO_V_E2M3 = 8, PTXO_V_E3M2 = 9, PTXO_V_E2M3_RELU = 10, PTXO_V_E3M2_RELU = 11,
    /* stochastic rounding: x4 formats, then with .relu */
    PTXO_V_E4M3_RS = 12, PTXO_V_E5M2_RS = 13, PTXO_V_E2M3_RS = 14, PTXO_V_E3M2_RS = 15,
    PTXO_V_E2M1_RS = 16, PTXO_V_E4M3_RS_RELU = 17, PTXO_V_E5M2_RS_RELU = 18,
    PTXO_V_E2M3_RS_RELU = 19, PTXO_V_E3M2_RS_RELU = 20, PTXO_V_E2M1_RS_RELU = 21,
    /* stochastic rounding to bf16 / f16 (two bytes per input): plain, .relu, .satfinite, both */
    PTXO_V_BF16_RS = 22, PTXO_V_BF16_RS_RELU = 23, PTXO_V_BF16_RS_SAT = 24,
    PTXO_V_BF16_RS_RELU_SAT = 25, PTXO_V_F16_RS = 26, PTXO_V_F16_RS_RELU = 27,
    PTXO_V_F16_RS_SAT = 28, PTXO_V_F16_RS_RELU_SAT = 29,
    /* bf16 round-to-nearest (two bytes per input): plain, .relu, .satfinite, both */
    PTXO_V_BF16_RN = 30, PTXO_V_BF16_RN_RELU = 31, PTXO_V_BF16_RN_SAT = 32,
    PTXO_V_BF16_RN_RELU_SAT = 33,
    PTXO_NUM_VARIANTS = 34,
};
#define PTXO_SWEEP_SEED 0x2545F4914F6CDD1Dull
uint8_t ptxo_encode_variant(int variant, float x); /* the round-to-nearest variants 0..11 */
/* Code of input pattern p (0 <= p < 2^32) under any variant; bytes per input of a variant. */
uint32_t ptxo_sweep_code(int variant, uint64_t p);
int ptxo_sweep_width(int variant);
uint64_t ptxo_sweep_compare(int variant, uint64_t base, uint64_t n, const uint8_t* device_out,
                            uint32_t* report, uint64_t max_report, int threads);
/* FNV-1a 64 digest of the oracle's codes for inputs [base, base + n) of a variant (width bytes
 * per input, in input order): FNV-1a 64 of every 2^16-byte piece, then over those digests.
 * Used to check the oracle against digests of the hardware's codes. */
uint64_t ptxo_sweep_digest(int variant, uint64_t base, uint64_t n, int threads);
uint64_t ptxo_fnv1a64(const uint8_t* data, size_t n, uint64_t seed);
/* The same digest scheme over given bytes (n a multiple of 2^16). */
uint64_t ptxo_digest_bytes(const uint8_t* data, uint64_t n, int threads);

/* ---- block-scale recipes ------------------------------------------------------------------ */
/* MXFP8: bf16 [rows, cols] row-major, cols % 32 == 0 -> E4M3 [rows, cols] and one UE8M0 scale
 * per 32 contiguous elements [rows, cols / 32]. Scale = floor-pow2 of the block amax minus E4M3's
 * emax (8), from the reference's f8e8m0::from_f32::<TowardZero, SaturateFinite>; elements are
 * x * 2^-(scale - 127) encoded RN .satfinite. */
void ptxo_quantize_mxfp8(const uint16_t* x, int64_t rows, int64_t cols, uint8_t* q, uint8_t* sf,
                         int threads);
/* NVFP4: bf16 [rows, cols], cols % 16 == 0, decode global scale g -> E2M1 [rows, cols / 2]
 * (element 0 in the low nibble) and one E4M3 scale per 16 contiguous elements [rows, cols / 16]:
 * sf = e4m3(amax / (6 g)), elements e2m1(x * (1 / (sf * g))). Returns -1 on a bad g. */
int ptxo_quantize_nvfp4(const uint16_t* x, int64_t rows, int64_t cols, float g, uint8_t* q,
                        uint8_t* sf, int threads);
/* One MXFP8 block / one NVFP4 block (used by the decode GEMM reference). */
uint8_t ptxo_mxfp8_block(const float* x32, uint8_t* q32);
uint8_t ptxo_nvfp4_block(const float* x16, float g, uint8_t* q16 /* one nibble per byte */);
/* The same recipes with stochastic rounding of the elements (the scales are unchanged): element
 * i of the flat input uses ptxo_rs_random(.., ptxo_sr_rbits(seed, i / 4), i % 4). */
void ptxo_quantize_mxfp8_rs(const uint16_t* x, int64_t rows, int64_t cols, uint64_t seed,
                            uint8_t* q, uint8_t* sf, int threads);
int ptxo_quantize_nvfp4_rs(const uint16_t* x, int64_t rows, int64_t cols, float g, uint64_t seed,
                           uint8_t* q, uint8_t* sf, int threads);

/* MX formats in the tcgen05 operand layout (kind::f8f6f4 / mxf8f6f4, dense K = 32; the
 * reference's F8f6f4ElementType, src/tcgen05/descriptor.rs:306-327). Every format takes one byte
 * per element in memory: FP8 codes as they are; FP6 (E2M3/E3M2) as groups of 16 six-bit codes
 * packed little-endian (element i at bits 6i .. 6i+5 of the group's 96 bits, 12 bytes) followed
 * by 4 zero bytes; FP4 (E2M1) as groups of 16 nibbles (element 2j in the low nibble of byte j, 8
 * bytes) followed by 8 zero bytes. n % 16 == 0. `codes` holds one code per byte (format PTXO_*). */
void ptxo_mx_pack(int format, const uint8_t* codes, uint8_t* packed, size_t n);
void ptxo_mx_unpack(int format, const uint8_t* packed, uint8_t* codes, size_t n);
/* The 8-bit containers that tcgen05.cp's .b8x16.b6x16_p32 / .b8x16.b4x16_p64 decompression
 * writes for n elements of packed FP6 / FP4 groups (copy.rs:32-46), one per element: an FP6 code
 * in bits 5..0; an FP4 code in bits 5..2 (E2M3-aligned, two zero mantissa bits below). */
void ptxo_cp_unpack(int format, const uint8_t* packed, uint8_t* containers, size_t n);
/* OCP MX quantisation to any of the five element formats: one UE8M0 scale per 32 contiguous
 * elements, floor-pow2 of the block amax (f8e8m0::from_f32::<TowardZero, SaturateFinite>) minus
 * the format's emax (E4M3 8, E5M2 15, E2M3 2, E3M2 4, E2M1 2), clamped at 0; elements
 * x * 2^-(scale - 127) encoded RN .satfinite. q [rows, cols] in the packed layout above,
 * sf [rows, cols / 32] row-major. For PTXO_E4M3 this is ptxo_quantize_mxfp8. */
void ptxo_quantize_mx(const uint16_t* x, int64_t rows, int64_t cols, int format, uint8_t* q,
                      uint8_t* sf, int threads);

/* ---- GEMM references (f64 over decoded values) at sampled outputs ------------------------- */
/* FP8: C[i,j] = sa * sb * sum_k A[i,k] B[j,k]; A [M,K], B [N,K] E4M3 (K contiguous). For each
 * sample s: ref[s] = exact-ish f64 value, mag[s] = sa*sb*sum_k |A B|. */
void ptxo_gemm_fp8_ref(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K,
                       float sa, float sb, const int64_t* rows, const int64_t* cols,
                       int64_t n_samples, double* ref, double* mag, int threads);
/* NVFP4: A [M,K/2], sfA [M,K/16] E4M3, ga; B [N,K/2], sfB [N,K/16], gb. */
void ptxo_gemm_nvfp4_ref(const uint8_t* A, const uint8_t* sfA, float ga, const uint8_t* B,
                         const uint8_t* sfB, float gb, int64_t M, int64_t N, int64_t K,
                         const int64_t* rows, const int64_t* cols, int64_t n_samples, double* ref,
                         double* mag, int threads);
/* MXFP8 (OCP MX): A [M,K], B [N,K] E4M3 (K contiguous), sfA [M,K/32], sfB [N,K/32] UE8M0
 * (row-major); C[i,j] = sum_k A[i,k] 2^(sfA-127) * B[j,k] 2^(sfB-127). */
void ptxo_gemm_mxfp8_ref(const uint8_t* A, const uint8_t* sfA, const uint8_t* B,
                         const uint8_t* sfB, int64_t M, int64_t N, int64_t K,
                         const int64_t* rows, const int64_t* cols, int64_t n_samples, double* ref,
                         double* mag, int threads);
/* MX GEMM with any pair of element formats: A [M,K] and B [N,K] in the packed layout of
 * ptxo_mx_pack (formats fa, fb), sfA [M,K/32], sfB [N,K/32] UE8M0 row-major. */
void ptxo_gemm_mx_ref(const uint8_t* A, int fa, const uint8_t* sfA, const uint8_t* B, int fb,
                      const uint8_t* sfB, int64_t M, int64_t N, int64_t K, const int64_t* rows,
                      const int64_t* cols, int64_t n_samples, double* ref, double* mag,
                      int threads);
/* 2:4 structured sparsity of E4M3 codes [rows, cols] (cols % 8 == 0): in every group of four
 * consecutive elements of a row, the two with the largest magnitude (code & 0x7F; ties go to the
 * lower index) are kept, in index order, in vals [rows, cols/2]; meta [rows, cols/8] holds one
 * nibble per group, i0 | i1 << 2 (i0 < i1, the kept positions), group g in the low nibble of byte
 * g/2 when g is even. This is the metadata of tcgen05.mma.sp for 8-bit kinds
 * (src/tcgen05/mma.rs:725-777): a row's nibbles in order are its lane's bits in Tensor Memory. */
void ptxo_prune_24(const uint8_t* codes, int64_t rows, int64_t cols, uint8_t* vals, uint8_t* meta,
                   int threads);
/* The dense E4M3 matrix [rows, cols] of (vals, meta): kept codes at their positions, 0 elsewhere. */
void ptxo_decompress_24(const uint8_t* vals, const uint8_t* meta, int64_t rows, int64_t cols,
                        uint8_t* codes, int threads);
/* 2:4-sparse MXFP8 GEMM (tcgen05.mma.sp kind::mxf8f6f4 .block_scale): A given as (vals [M,K/2],
 * meta [M,K/8]), B [N,K] E4M3, and ONE UE8M0 scale per 64 logical K for both operands (the
 * sparse MMA of K = 64 takes a single scale of each operand: 32 stored A elements), sfA [M,K/64],
 * sfB [N,K/64] row-major; C[i,j] = sum_k A[i,k] 2^(sfA[i,k/64]-127) B[j,k] 2^(sfB[j,k/64]-127). */
void ptxo_gemm_mxfp8_sparse_ref(const uint8_t* vals, const uint8_t* meta, const uint8_t* sfA,
                                const uint8_t* B, const uint8_t* sfB, int64_t M, int64_t N,
                                int64_t K, const int64_t* rows, const int64_t* cols,
                                int64_t n_samples, double* ref, double* mag, int threads);
/* Decode: x bf16 [M,K] is MXFP8-quantised (32-blocks) by the recipe above, W NVFP4 [N,K/2] with
 * sfW [N,K/16] and gw; C[i,j] = sum_k xq[i,k] 2^(sx-127) * w[j,k] sfW gw. */
void ptxo_gemm_decode_ref(const uint16_t* x, const uint8_t* W, const uint8_t* sfW, float gw,
                          int64_t M, int64_t N, int64_t K, const int64_t* rows,
                          const int64_t* cols, int64_t n_samples, double* ref, double* mag,
                          int threads);
/* Timed CPU baseline: C[M,N] (f32) = sum_k A[i,k] B[j,k] over f32 matrices, cache-blocked and
 * multithreaded (B given K-contiguous, like the device operands). */
void ptxo_sgemm_nt(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                   int threads);

/* ---- tcgen05 descriptor encodings (src/tcgen05/descriptor.rs) ----------------------------- */
/* All return 0 and write *out on success, -1 where the reference asserts. */
int ptxo_idesc_f16(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out);
int ptxo_idesc_tf32(uint32_t m, uint32_t n, uint32_t* out);
int ptxo_idesc_f8f6f4(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out);
int ptxo_idesc_i8(int a, int b, uint32_t m, uint32_t n, uint32_t* out);
int ptxo_idesc_mxf8f6f4(int a, int b, uint32_t m, uint32_t n, uint32_t* out);
int ptxo_idesc_mxf4(uint32_t m, uint32_t n, uint32_t* out);
int ptxo_idesc_mxf4nvf4(int scale_type, uint32_t m, uint32_t n, uint32_t* out);
/* Generic field setter: replaces the width-bit field at shift (descriptor.rs:494-498). */
int ptxo_idesc_with_field(uint32_t desc, uint32_t shift, uint32_t width, uint32_t value,
                          uint32_t* out);
int ptxo_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo, int swizzle, uint64_t* out);
int ptxo_smem_desc_with_base_offset(uint64_t desc, uint32_t base_offset, uint64_t* out);
int ptxo_smem_desc_add_start_bytes(uint64_t desc, uint32_t bytes, uint64_t* out);
int ptxo_zero_mask_new(uint32_t zeroed, uint32_t used, uint64_t* out);
int ptxo_zero_mask_with_sub_mask_start(uint64_t mask, uint32_t sub, int first_span,
                                       uint32_t start_count, uint64_t* out);
int ptxo_zero_mask_with_column_shift(uint64_t mask, uint32_t shift, uint64_t* out);

int ptxo_hardware_threads(void);

#ifdef __cplusplus
}
#endif
#endif

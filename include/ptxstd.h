/*
 * ptxstd — B200 (sm_100a) narrow-float quantisation and block-scaled tcgen05 GEMM, C ABI.
 *
 * caelunshun/ptx-std is a device-only Rust crate: its "interface" is the set of device functions a
 * user kernel calls (conversions of src/data_types/, the tcgen05 descriptors and instructions of
 * src/tcgen05/, TMA of src/tma/, mbarriers of src/mbarrier.rs). This header is the host-callable
 * boundary that a binding of that crate (Rust `extern "C"`, ctypes, cgo ...) links against: each
 * entry point names the reference API whose semantics it implements, file:line in the reference.
 *
 * Conventions
 *   - Every function returns a ptxstd_status; no C++ exception or abort crosses the boundary.
 *   - Pointers named d_* are device pointers owned by the caller (16-byte aligned unless noted);
 *     h_* are host pointers. Kernels are asynchronous on `stream` (a cudaStream_t, 0 = legacy).
 *     The quantisers use programmatic dependent launch and touch caller memory only after
 *     griddepcontrol.wait, so stream order holds as for any launch. The decode GEMM is launched
 *     the same way behind its own prep kernel, which is an ordinary launch.
 *   - Narrow codes are stored as in the reference: element 0 in the least significant bits
 *     (src/data_types/vector.rs:1-11); two E2M1 values per byte, element 0 in the low nibble
 *     (src/data_types/float4.rs:5-6).
 *   - bf16 is passed as uint16_t bit patterns.
 *   - Device-side waits are bounded; a kernel that gives up records PTXSTD_ETIMEOUT in a
 *     per-device error word read by ptxstd_last_device_error.
 */
#ifndef PTXSTD_H
#define PTXSTD_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum ptxstd_status {
    PTXSTD_OK = 0,
    PTXSTD_EINVAL = 1,      /* bad argument: shape, alignment, null pointer, unencodable value */
    PTXSTD_ECUDA = 2,       /* a CUDA runtime or driver call failed */
    PTXSTD_ENCCL = 3,       /* an NCCL call failed */
    PTXSTD_ETIMEOUT = 4,    /* a bounded device-side wait gave up */
    PTXSTD_EUNSUPPORTED = 5 /* not supported on this device (needs sm_100a) */
} ptxstd_status;

typedef void* ptxstd_stream; /* a cudaStream_t */

#if defined(__GNUC__)
#define PTXSTD_API __attribute__((visibility("default")))
#else
#define PTXSTD_API
#endif

/* ---- library ------------------------------------------------------------------------------- */
PTXSTD_API const char* ptxstd_status_string(int status);
/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
PTXSTD_API int ptxstd_version(void);
/* PTXSTD_OK when `device` is an sm_100 part this library's cubins run on. */
PTXSTD_API int ptxstd_device_supported(int device);
/* Reads (and, if clear != 0, resets) the calling device's error word after synchronising
 * `stream`. *code receives 0 or a ptxstd_status; *detail a kernel-specific location code. */
PTXSTD_API int ptxstd_last_device_error(ptxstd_stream stream, int clear, int* code, uint32_t* detail);

/* ---- data_types: element-wise conversions on device arrays --------------------------------- */
/* Vector<f8e4m3, N>::from_f32::<RELU> (src/data_types/narrow.rs:354-361, pair form :156-162):
 * RN, .satfinite, NaN -> 0x7f, optional .relu. One code per byte. n any size. */
PTXSTD_API int ptxstd_cvt_f32_to_e4m3(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream);
/* Vector<f8e5m2, N>::from_f32::<RELU> (same macro, src/data_types/float8.rs:111-126). */
PTXSTD_API int ptxstd_cvt_f32_to_e5m2(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream);
/* Vector<f4e2m1, N>::from_f32::<RELU> (src/data_types/float4.rs:52-69): n even, n/2 bytes out,
 * element 2i in the low nibble of byte i; NaN -> +6. */
PTXSTD_API int ptxstd_cvt_f32_to_e2m1x2(const float* d_x, uint8_t* d_out, size_t n, int relu,
                             ptxstd_stream stream);
/* f8e8m0::from_f32::<RND, OVERFLOW> (src/data_types/narrow.rs:600-617, semantics :585-593):
 * round_up = 0 -> Rounding::TowardZero, 1 -> Rounding::Up; satfinite selects .satfinite. */
PTXSTD_API int ptxstd_cvt_f32_to_ue8m0(const float* d_x, uint8_t* d_out, size_t n, int round_up,
                            int satfinite, ptxstd_stream stream);
/* to_f32 of each format: exact, via f16 for FP8/FP4 (src/data_types/narrow.rs:292-299) and via
 * bf16 for ue8m0 (src/data_types/narrow.rs:683-690). e2m1x2 decodes 2*n_bytes values. */
PTXSTD_API int ptxstd_cvt_e4m3_to_f32(const uint8_t* d_codes, float* d_out, size_t n, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e5m2_to_f32(const uint8_t* d_codes, float* d_out, size_t n, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e2m1x2_to_f32(const uint8_t* d_codes, float* d_out, size_t n_bytes,
                             ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_ue8m0_to_f32(const uint8_t* d_codes, float* d_out, size_t n, ptxstd_stream stream);
/* Vector<f6e2m3, N> / Vector<f6e3m2, N>::from_f32::<RELU> (src/data_types/float6.rs, narrow_cvt!
 * core from_f32 = cvt.rn.satfinite{.relu}.{e2m3,e3m2}x2.f32): RN, .satfinite, one value in the
 * low 6 bits of each output byte. E2M3: bias 1, max 7.5; E3M2: bias 3, max 28; no infinities or
 * NaNs (a NaN input becomes the code the hardware writes, pinned by the sweep). n any size. */
PTXSTD_API int ptxstd_cvt_f32_to_e2m3(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f32_to_e3m2(const float* d_x, uint8_t* d_out, size_t n, int relu,
                           ptxstd_stream stream);
/* FP6 to_f32: exact, via cvt.rn.f16x2.{e2m3,e3m2}x2 (float6.rs core to_f16x2). Only the low 6 bits
 * of each code byte are significant (float6.rs:1-8: the two top bits must be zero). */
PTXSTD_API int ptxstd_cvt_e2m3_to_f32(const uint8_t* d_codes, float* d_out, size_t n, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e3m2_to_f32(const uint8_t* d_codes, float* d_out, size_t n, ptxstd_stream stream);
/* Vector<E, N>::from_f16::<RELU> (src/data_types/narrow.rs:164-172, :363-395): f16 bit patterns ->
 * narrow codes, RN .satfinite, the same rules as from_f32 (f16 widens to f32 exactly). FP8 uses
 * cvt.rn.satfinite{.relu}.<fmt>x2.f16x2; FP6 and FP4, whose f16x2 forms this toolchain's ptxas
 * does not accept, convert the exactly widened f32. E2M1 output packed two per byte (n even). */
PTXSTD_API int ptxstd_cvt_f16_to_e4m3(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f16_to_e5m2(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f16_to_e2m1x2(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f16_to_e2m3(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f16_to_e3m2(const uint16_t* d_x, uint8_t* d_out, size_t n, int relu, ptxstd_stream stream);
/* Vector<E, N>::to_f16 (narrow.rs:275-291): exact f16 bit patterns via cvt.rn.f16x2.<fmt>x2 (e2m1x2
 * decodes 2 * n_bytes values). */
PTXSTD_API int ptxstd_cvt_e4m3_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e5m2_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e2m1x2_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n_bytes, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e2m3_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e3m2_to_f16(const uint8_t* d_codes, uint16_t* d_out, size_t n, ptxstd_stream stream);
/* bf16xN::from_f32::<R, O> (src/data_types/bfloat16.rs:104-118, :446-454): RN, relu clamps negative
 * results (and -0) to +0, satfinite clamps overflow to the largest finite bf16 (else infinity);
 * every NaN becomes 0x7FFF. */
PTXSTD_API int ptxstd_cvt_f32_to_bf16(const float* d_x, uint16_t* d_out, size_t n, int relu, int satfinite,
                           ptxstd_stream stream);
/* Vector<E, N>::to_bf16_scaled::<RELU, OVERFLOW> (src/data_types/narrow.rs:314-330, :444-465):
 * element i times the UE8M0 scale d_scales[i / block] (2^(s-127); 0xff is NaN), rounded to bf16
 * (RN). relu clamps negative results to +0; satfinite clamps results outside the finite range to
 * the largest finite bf16 of matching sign, otherwise they become infinity. block = 1 is the
 * reference's form (one scale per element); block = 32 dequantises MXFP8 rows. The reference
 * lowers this to cvt.rn...bf16x2.<fmt>x2.scale::n2::ue8m0, which the CUDA 12.9 ptxas of this
 * build does not accept; the result is computed exactly instead (exact decode, exact f32 product,
 * one cvt.rn{.relu}{.satfinite}.bf16x2.f32). e2m1x2 codes are packed two per byte (n even). */
PTXSTD_API int ptxstd_cvt_e4m3_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e5m2_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e2m1x2_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                     uint16_t* d_out, size_t n, size_t block, int relu,
                                     int satfinite, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e2m3_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_e3m2_to_bf16_scaled(const uint8_t* d_codes, const uint8_t* d_scales,
                                   uint16_t* d_out, size_t n, size_t block, int relu,
                                   int satfinite, ptxstd_stream stream);
/* Stochastic rounding: Vector<E, N>::from_f32_stochastic::<RELU> (src/data_types/narrow.rs:494-505;
 * core quad_from_f32_stochastic = cvt.rs.satfinite{.relu}.<fmt>x4.f32, :217-229). Elements
 * 4g .. 4g+3 are converted together with the random bits d_rbits[g] (ceil(n/4) words); a last
 * group of fewer than four is padded with zeros whose results are dropped (:483-486). Each value
 * is rounded toward zero unless the discarded mantissa bits plus its random bits carry. Which
 * rbits bits serve which element: FP8/FP6 "the lower 16 bits for elements 0 and 1, the upper 16
 * for elements 2 and 3" (src/data_types/float8.rs:59, float6.rs:61); E2M1 "the lower 8 bits of
 * both 16-bit halves for elements 0 and 1, the upper 8 bits of both halves for elements 2 and 3"
 * (float4.rs:60). Needs sm_100a. E2M1 output is packed two per byte (n even). d_x 16-byte
 * aligned; d_rbits 4-byte aligned. */
PTXSTD_API int ptxstd_cvt_f32_to_e4m3_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out,
                              size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f32_to_e5m2_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out,
                              size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f32_to_e2m3_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out,
                              size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f32_to_e3m2_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out,
                              size_t n, int relu, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f32_to_e2m1x2_rs(const float* d_x, const uint32_t* d_rbits, uint8_t* d_out,
                                size_t n, int relu, ptxstd_stream stream);
/* bf16xN / f16xN::from_f32_stochastic::<R, O> (src/data_types/bfloat16.rs:572-598,
 * src/data_types/float16.rs:740-766; cvt.rs{.relu}{.satfinite}.{bf16x2,f16x2}.f32): elements 2p,
 * 2p+1 with d_rbits[p] (ceil(n/2) words), the lower 16 bits for the even element (bf16: all 16;
 * f16: the 13 least significant), the upper for the odd one. satfinite = 0 lets overflow become
 * infinity. d_x 8-byte aligned; d_out 4-byte aligned. */
PTXSTD_API int ptxstd_cvt_f32_to_bf16_rs(const float* d_x, const uint32_t* d_rbits, uint16_t* d_out,
                              size_t n, int relu, int satfinite, ptxstd_stream stream);
PTXSTD_API int ptxstd_cvt_f32_to_f16_rs(const float* d_x, const uint32_t* d_rbits, uint16_t* d_out,
                             size_t n, int relu, int satfinite, ptxstd_stream stream);
/* Exhaustive-sweep helper: encodes the n f32 bit patterns base, base+1, ... (no input array) with
 * one of the variants 0 e4m3, 1 e5m2, 2 e2m1 (one nibble per byte), 3-5 the same with .relu,
 * 6 ue8m0 RZ satfinite, 7 ue8m0 RP satfinite, 8 e2m3, 9 e3m2, 10-11 the same with .relu;
 * stochastic rounding: 12 e4m3, 13 e5m2, 14 e2m3, 15 e3m2, 16 e2m1 (nibble per byte), 17-21 the
 * same with .relu, then two bytes per input: 22 bf16, 23 .relu, 24 .satfinite, 25 both, 26-29
 * the same for f16; 30-33 bf16 round-to-nearest: plain, .relu, .satfinite, both (two bytes per
 * input). Pattern p of a stochastic variant takes the random bits of group p / 4
 * (p / 2 for bf16/f16): word (group % 2) of SplitMix64 output group / 2 from the seed
 * 0x2545F4914F6CDD1D (the generator of ptxstd_quantize_mxfp8_rs). base + n <= 2^32; base % 4 == 0
 * for the stochastic variants. */
PTXSTD_API int ptxstd_cvt_sweep(int variant, uint64_t base, uint64_t n, uint8_t* d_out,
                     ptxstd_stream stream);

/* ---- quantisation kernels ------------------------------------------------------------------- */
/* MXFP8: bf16 [rows, cols] row-major (cols % 32 == 0) -> E4M3 [rows, cols] and one UE8M0 scale
 * per 32 contiguous elements, [rows, cols/32] row-major. Scale = f8e8m0::from_f32::<TowardZero,
 * SaturateFinite>(block amax) - 8 (E4M3's emax), clamped at 0, NaN kept; elements
 * f8e4m3::from_f32(x * 2^-(scale-127)) (src/data_types/narrow.rs:156-162, :600-617; block amax
 * as reduce_f32::<Max, Absolute> with NaN, src/warp_collectives.rs:864). */
PTXSTD_API int ptxstd_quantize_mxfp8(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                          uint8_t* d_sf, ptxstd_stream stream);
/* NVFP4: bf16 [rows, cols] (cols % 16 == 0) with decode global scale g (finite, > 0) ->
 * E2M1x2 [rows, cols/2] and one E4M3 scale per 16 elements [rows, cols/16]:
 * sf = f8e4m3::from_f32(amax / (6 g)), q = f4e2m1::from_f32(x * (1 / (sf * g))), each f32
 * operation one IEEE rounding (src/data_types/float4.rs:52-69, float8.rs:51-68). */
PTXSTD_API int ptxstd_quantize_nvfp4(const uint16_t* d_x, int64_t rows, int64_t cols, float global_scale,
                          uint8_t* d_q, uint8_t* d_sf, ptxstd_stream stream);
/* The same two kernels with a choice of scale layout: sf_layout 0 = row-major [rows, cols/B]
 * (B = 32 or 16); 1 = the blocked layout the block-scaled GEMMs read: tiles of 128 rows x 4
 * scale columns, 512 contiguous bytes each, row-tile major, scale (r, s) of a tile at byte
 * (r % 32) * 16 + ((r / 32) % 4) * 4 + s % 4 (the source of one tcgen05.cp.32x128b.warpx4,
 * src/tcgen05/copy.rs:29-30). Layout 1 needs rows % 128 == 0 and cols % (4 B) == 0. */
PTXSTD_API int ptxstd_quantize_mxfp8_layout(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                                 uint8_t* d_sf, int sf_layout, ptxstd_stream stream);
PTXSTD_API int ptxstd_quantize_nvfp4_layout(const uint16_t* d_x, int64_t rows, int64_t cols,
                                 float global_scale, uint8_t* d_q, uint8_t* d_sf, int sf_layout,
                                 ptxstd_stream stream);
/* Stochastic-rounding quantise (the from_f32_stochastic element conversion of
 * src/data_types/narrow.rs:494-505 inside the same recipes; scales unchanged). Element i of the
 * flat row-major input belongs to group i / 4, whose random bits are word (group % 2) of
 * SplitMix64 output group / 2 started at `seed`: z = seed + (k + 1) * 0x9E3779B97F4A7C15;
 * z = (z ^ z >> 30) * 0xBF58476D1CE4E5B9; z = (z ^ z >> 27) * 0x94D049BB133111EB; z ^ z >> 31.
 * The same seed gives the same codes on every call and every launch shape. */
PTXSTD_API int ptxstd_quantize_mxfp8_rs(const uint16_t* d_x, int64_t rows, int64_t cols, uint8_t* d_q,
                             uint8_t* d_sf, int sf_layout, uint64_t seed, ptxstd_stream stream);
PTXSTD_API int ptxstd_quantize_nvfp4_rs(const uint16_t* d_x, int64_t rows, int64_t cols,
                             float global_scale, uint8_t* d_q, uint8_t* d_sf, int sf_layout,
                             uint64_t seed, ptxstd_stream stream);

/* ---- block-scaled / narrow GEMMs on tcgen05 --------------------------------------------------- */
/* FP8 GEMM: C[M,N] bf16 row-major = sa * sb * A[M,K] * B[N,K]^T with E4M3 A and B (K contiguous),
 * fp32 accumulation, bf16 RN output. The tcgen05.mma.kind::f8f6f4 + TMA + mbarrier pipeline of
 * src/tcgen05/mod.rs:105-162 (mma :434-453 of src/tcgen05/mma.rs; InstrDescriptor::<F8f6f4>::new,
 * src/tcgen05/descriptor.rs:555-564). M % 128 == 0, N % 256 == 0, K % 128 == 0. */
PTXSTD_API int ptxstd_gemm_fp8(const uint8_t* d_a, const uint8_t* d_b, float sa, float sb,
                               uint16_t* d_c, int64_t M, int64_t N, int64_t K,
                               ptxstd_stream stream);
/* NVFP4 GEMM: C[M,N] bf16 = ga * gb * sum_k (A[m,k] sfA[m,k/16]) (B[n,k] sfB[n,k/16]).
 * A [M,K/2], B [N,K/2]: E2M1 two per byte, element 0 in the low nibble, K contiguous.
 * sfA, sfB: E4M3 scales per 16 K elements in the blocked layout of
 * ptxstd_quantize_nvfp4_layout(sf_layout = 1). tcgen05.mma.kind::mxf4nvf4.block_scale.block16
 * (mma_block_scaled, src/tcgen05/mma.rs:698-724; InstrDescriptor::<Mxf4nvf4>::new,
 * src/tcgen05/descriptor.rs:644-653; scale copy, src/tcgen05/copy.rs:76-116).
 * M % 128 == 0, N % 256 == 0, K % 256 == 0. */
PTXSTD_API int ptxstd_gemm_nvfp4(const uint8_t* d_a, const uint8_t* d_sfa, float ga,
                                 const uint8_t* d_b, const uint8_t* d_sfb, float gb,
                                 uint16_t* d_c, int64_t M, int64_t N, int64_t K,
                                 ptxstd_stream stream);
/* Tile schedule of the CTA-pair NVFP4 GEMM (process-wide; later launches use it).
 * PTXSTD_SCHEDULE_PERSISTENT (default): one resident CTA pair per two SMs walks a fixed raster
 *   of tiles; fastest when the GEMM has the GPU to itself.
 * PTXSTD_SCHEDULE_DYNAMIC: one cluster per tile; running pairs take over the tiles of clusters
 *   that have not started (cluster launch control: try_cancel_launch, src/launch.rs:154-176), so
 *   work moves to whichever SMs are free when other kernels hold some of them.
 * Returns PTXSTD_EINVAL for any other value. */
#define PTXSTD_SCHEDULE_PERSISTENT 0
#define PTXSTD_SCHEDULE_DYNAMIC 1
PTXSTD_API int ptxstd_set_gemm_schedule(int schedule);
PTXSTD_API int ptxstd_get_gemm_schedule(void);
/* MXFP8 GEMM (OCP MX): C[M,N] bf16 = sum_k (A[m,k] 2^(sfA[m,k/32]-127)) (B[n,k] 2^(sfB[n,k/32]-127)).
 * A [M,K], B [N,K]: E4M3, K contiguous. sfA, sfB: UE8M0 scales per 32 K elements in the blocked
 * layout of ptxstd_quantize_mxfp8_layout(sf_layout = 1), so quantised activations feed it as they
 * are. tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale.block32 (mma_block_scaled with
 * MmaKind::Mxf8f6f4 and ScaleVectorSize::Block32, src/tcgen05/mma.rs:58-97, :698-724;
 * InstrDescriptor::<Mxf8f6f4>::new and its scale ids, src/tcgen05/descriptor.rs:601-611).
 * M % 256 == 0, N % 256 == 0, K % 128 == 0. */
PTXSTD_API int ptxstd_gemm_mxfp8(const uint8_t* d_a, const uint8_t* d_sfa, const uint8_t* d_b,
                                 const uint8_t* d_sfb, uint16_t* d_c, int64_t M, int64_t N,
                                 int64_t K, ptxstd_stream stream);
/* MX element types of kind::f8f6f4 / mxf8f6f4, with the values of the reference's
 * F8f6f4ElementType (src/tcgen05/descriptor.rs:316-327). */
enum ptxstd_mx_type {
    PTXSTD_MX_E4M3 = 0,
    PTXSTD_MX_E5M2 = 1,
    PTXSTD_MX_E2M3 = 3,
    PTXSTD_MX_E3M2 = 4,
    PTXSTD_MX_E2M1 = 5,
};
/* OCP MX quantisation of bf16 [rows, cols] (cols % 32 == 0) to any MX element type: one UE8M0
 * scale per 32 contiguous elements (floor-pow2 of the block amax, f8e8m0::from_f32::<TowardZero,
 * SaturateFinite>, minus the format's emax: E4M3 8, E5M2 15, E2M3 2, E3M2 4, E2M1 2, clamped at 0),
 * elements x * 2^-(scale-127) RN .satfinite (narrow.rs:125-130). q [rows, cols] bytes in the
 * tensor cores' operand layout for K = 32 MMAs (descriptor.rs:306-315): FP8 one code per byte;
 * FP6 16 six-bit codes packed little-endian in 12 bytes + 4 zero bytes per 16 elements; FP4 16
 * nibbles in 8 bytes + 8 zero bytes. sf_layout as ptxstd_quantize_mxfp8_layout. For E4M3 the
 * result equals ptxstd_quantize_mxfp8_layout's. */
PTXSTD_API int ptxstd_quantize_mx(const uint16_t* d_x, int64_t rows, int64_t cols, int elem_type,
                                  uint8_t* d_q, uint8_t* d_sf, int sf_layout,
                                  ptxstd_stream stream);
/* MX GEMM with any pair of element types (mma_block_scaled with MmaKind::Mxf8f6f4,
 * InstrDescriptor::<Mxf8f6f4>::new(a_type, b_type, 256, 256), src/tcgen05/descriptor.rs:601-611):
 * C[M,N] bf16 = sum_k (A[m,k] 2^(sfA-127)) (B[n,k] 2^(sfB-127)); A [M,K] and B [N,K] in the
 * operand layout of ptxstd_quantize_mx, scales blocked (sf_layout 1). ptxstd_gemm_mxfp8 is
 * a_type = b_type = PTXSTD_MX_E4M3. M % 256 == 0, N % 256 == 0, K % 128 == 0. */
PTXSTD_API int ptxstd_gemm_mx(const uint8_t* d_a, int a_type, const uint8_t* d_sfa,
                              const uint8_t* d_b, int b_type, const uint8_t* d_sfb, uint16_t* d_c,
                              int64_t M, int64_t N, int64_t K, ptxstd_stream stream);
/* The decompressing shared-memory -> Tensor Memory copy (copy::<S128x256b, B6x16P32 | B4x16P64>,
 * src/tcgen05/copy.rs:32-46, :76-116), run over n_tiles tiles of 128 rows x 32 bytes: packed FP6
 * (elem_type PTXSTD_MX_E2M3 / E3M2: .b8x16.b6x16_p32) or FP4 (PTXSTD_MX_E2M1: .b8x16.b4x16_p64)
 * groups in the layout of ptxstd_quantize_mx go through tcgen05.cp into TMEM and come back with
 * tcgen05.ld as one 8-bit container per element, [n_tiles * 128, 32] bytes. */
PTXSTD_API int ptxstd_tcgen05_cp_unpack(const uint8_t* d_packed, uint8_t* d_out, int64_t n_tiles,
                                        int elem_type, ptxstd_stream stream);
/* 2:4 structured sparsity (the A operand of tcgen05.mma.sp, src/tcgen05/mma.rs:725-777): in each
 * group of four consecutive elements of a row of E4M3 codes [rows, cols], the two of largest
 * magnitude (code & 0x7F, ties to the lower index) are kept, in index order, in vals
 * [rows, cols/2]; meta [rows, cols/8] holds one nibble per group, i0 | i1 << 2 (i0 < i1 the kept
 * positions), group g in the low nibble of byte g/2 for even g. cols % 8 == 0; d_codes 8-byte
 * and d_vals 4-byte aligned. */
PTXSTD_API int ptxstd_prune_24_e4m3(const uint8_t* d_codes, int64_t rows, int64_t cols, uint8_t* d_vals,
                         uint8_t* d_meta, ptxstd_stream stream);
/* 2:4-sparse MXFP8 GEMM: C[M,N] bf16 = sum_k A[m,k] 2^(sfa[m,k/64]-127) * B[n,k] 2^(sfb[n,k/64]-127)
 * with A given as (vals [M,K/2], meta [M,K/8]) of ptxstd_prune_24_e4m3, B [N,K] E4M3 (K
 * contiguous), and ONE UE8M0 scale per 64 logical K for each operand (the sparse K = 64 MMA takes
 * a single scale: 32 stored elements of A), in the blocked 128x4 layout (one 512-byte tile per
 * 128 rows and 256 K). tcgen05.mma.sp.cta_group::2.kind::mxf8f6f4.block_scale.block32, metadata
 * moved to Tensor Memory with tcgen05.cp.128x128b (mma_block_scaled_sparse, src/tcgen05/mma.rs:
 * 725-777; InstrDescriptor::with_sparsity, src/tcgen05/descriptor.rs:500-506). M % 256 == 0,
 * N % 256 == 0, K % 256 == 0; all pointers 16-byte aligned. */
PTXSTD_API int ptxstd_gemm_mxfp8_sparse(const uint8_t* d_vals, const uint8_t* d_meta, const uint8_t* d_sfa,
                             const uint8_t* d_b, const uint8_t* d_sfb, uint16_t* d_c, int64_t M,
                             int64_t N, int64_t K, ptxstd_stream stream);

/* Decode-shape GEMM: y[M,N] bf16 = MXFP8(x)[M,K] * NVFP4(W)[N,K]^T * gw, M <= 16 tokens.
 * x: bf16 [M,K] row-major, quantised inside the call with the recipe of ptxstd_quantize_mxfp8
 * (f8e8m0::from_f32::<TowardZero, SaturateFinite>, src/data_types/narrow.rs:600-617; f8e4m3
 * ::from_f32, :156-162). W: [N,K/2] E2M1x2 with E4M3 scales per 16 in the blocked layout
 * (ptxstd_quantize_nvfp4_layout, sf_layout 1) and f32 global scale gw. Both operands are brought
 * to f16 exactly and multiplied with tcgen05.mma.kind::f16 with the A operand in TMEM
 * (src/tcgen05/mma.rs:434-453), fp32 accumulation. N % 128 == 0, K % 256 == 0.
 * workspace: device scratch of ptxstd_gemm_decode_workspace_bytes(M, N, K) bytes, 1024-byte
 * aligned, owned by the caller; the call initialises it itself (no zeroing needed). Calls that
 * share a workspace must be stream-ordered. The size depends on the current device's SM count
 * (two 8 KiB partial-sum slots per SM, plus the quantised x and N/128 counters), so query it
 * with the device current that will run the calls. The result is bitwise reproducible: a weight
 * block split between CTAs is summed from their partials in a fixed order. */
PTXSTD_API size_t ptxstd_gemm_decode_workspace_bytes(int64_t M, int64_t N, int64_t K);
PTXSTD_API int ptxstd_gemm_decode(const uint16_t* d_x, const uint8_t* d_w, const uint8_t* d_sfw,
                                  float gw, uint16_t* d_y, int64_t M, int64_t N, int64_t K,
                                  void* d_workspace, size_t workspace_bytes,
                                  ptxstd_stream stream);

/* Size of the fixed device scratch array behind ptxstd_gemm_decode_noalloc (4 MiB). */
#define PTXSTD_DECODE_NOALLOC_SCRATCH_BYTES (4u << 20)
/* The decode GEMM for callers that cannot allocate device memory; this entry point has no
 * counterpart in the reference (ptx-std has no host code at all). It computes what
 * ptxstd_gemm_decode computes, with the same arguments minus the workspace, and allocates
 * nothing: no cudaMalloc, no cudaFree, no allocating library call. It is meant for callers such
 * as a serving loop whose device-memory plan is fixed at start-up (cudaMalloc / cudaFree can
 * synchronise the device and fragment a sized pool, so they are not allowed per request), or a
 * thin C / Rust binding that owns only its input and output buffers and has no allocator of its
 * own for a workspace. Its scratch is a file-scope device array of
 * PTXSTD_DECODE_NOALLOC_SCRATCH_BYTES (1024-byte aligned); shapes whose scratch
 * (ptxstd_gemm_decode_workspace_bytes) would exceed it are rejected with PTXSTD_EINVAL (the
 * 16 x 57344 x 8192 decode shape fits). A device reserves the array when the decode code is first
 * used on it (the CUDA runtime loads device code lazily by default), i.e. at the first call of
 * this entry point or of ptxstd_gemm_decode there, and holds it until the process exits; the
 * regular ptxstd_gemm_decode therefore carries the same 4 MiB. The first call on a device also
 * looks up the array's device address for that device. So make one warm-up call per device at
 * start-up, before serving and before any stream capture. The address is kept for the life of
 * the process: calls across a device reset (cudaDeviceReset) are not supported. All calls on a
 * device share the array (each call clears what must start at zero); calls that overlap on the
 * GPU, e.g. on two streams, race on it and must be serialised by the caller. */
PTXSTD_API int ptxstd_gemm_decode_noalloc(const uint16_t* d_x, const uint8_t* d_w,
                                          const uint8_t* d_sfw, float gw, uint16_t* d_y,
                                          int64_t M, int64_t N, int64_t K, ptxstd_stream stream);

/* ---- multi-GPU: N-sharded weights over NCCL ---------------------------------------------------
 * No counterpart in the reference (it has no host-side communication). One rank per GPU; ranks
 * share an NCCL unique id (e.g. broadcast over torch.distributed or MPI) and create a
 * communicator on their current device. NCCL is loaded at run time (PTXSTD_ENCCL if missing). */
typedef struct ptxstd_dist ptxstd_dist;
PTXSTD_API int ptxstd_dist_unique_id(uint8_t* out_128);
PTXSTD_API int ptxstd_dist_init(const uint8_t* unique_id_128, int nranks, int rank,
                                ptxstd_dist** out);
PTXSTD_API int ptxstd_dist_free(ptxstd_dist* dist);
PTXSTD_API int ptxstd_dist_size(const ptxstd_dist* dist, int* nranks, int* rank);
/* NVFP4 GEMM with B split along N: this rank holds B rows [rank*N/world, (rank+1)*N/world) (and
 * their scales) and computes C_shard [M, N/world]. No communication. */
PTXSTD_API int ptxstd_gemm_nvfp4_sharded(const ptxstd_dist* dist, const uint8_t* d_a,
                                         const uint8_t* d_sfa, float ga, const uint8_t* d_b_shard,
                                         const uint8_t* d_sfb_shard, float gb, uint16_t* d_c_shard,
                                         int64_t M, int64_t N, int64_t K, ptxstd_stream stream);
/* Decode GEMM with W split along N: each rank computes its [M, N/world] block, NCCL all-gathers
 * the blocks in place over NVLink, and y [M, N] (row-major, every rank) is assembled on the
 * device. workspace: ptxstd_gemm_decode_sharded_workspace_bytes bytes, 1024-byte aligned. */
PTXSTD_API size_t ptxstd_gemm_decode_sharded_workspace_bytes(const ptxstd_dist* dist, int64_t M,
                                                             int64_t N, int64_t K);
PTXSTD_API int ptxstd_gemm_decode_sharded(const ptxstd_dist* dist, const uint16_t* d_x,
                                          const uint8_t* d_w_shard, const uint8_t* d_sfw_shard,
                                          float gw, uint16_t* d_y, int64_t M, int64_t N,
                                          int64_t K, void* d_workspace, size_t workspace_bytes,
                                          ptxstd_stream stream);

/* The decode GEMM with the all-gather fused into it: every rank's epilogue stores each finished
 * [M, 128] output block straight into every rank's y over NVLink (CUDA IPC peer mappings), with
 * monotonic counters and bounded waits in place of a collective, so a step is two kernels plus a
 * one-block completion wait and can be captured in a CUDA graph. Setup, once per communicator
 * and N (collective: every rank calls it): this rank's y [16, N] bf16 row-major, owned by the
 * library until ptxstd_dist_free, is returned in *d_y. A step (collective): rows 0..M-1 of that y
 * hold the full product when the stream reaches the end of the call; with d_y_copy non-null they
 * are also copied there. Steps of one communicator must be issued in the same order on every
 * rank, with the communicator's GPU current (else EINVAL). N % (128 * world) == 0; at most 8
 * ranks, each on a GPU of its own (the step's kernels
 * wait on the other ranks' kernels; ranks that share a GPU get PTXSTD_EUNSUPPORTED from the
 * setup); workspace as ptxstd_gemm_decode_workspace_bytes(M, N / world, K). */
PTXSTD_API int ptxstd_dist_decode_p2p_init(ptxstd_dist* dist, int64_t N, uint16_t** d_y);
PTXSTD_API int ptxstd_gemm_decode_sharded_p2p(const ptxstd_dist* dist, const uint16_t* d_x,
                                              const uint8_t* d_w_shard, const uint8_t* d_sfw_shard,
                                              float gw, uint16_t* d_y_copy, int64_t M, int64_t N,
                                              int64_t K, void* d_workspace, size_t workspace_bytes,
                                              ptxstd_stream stream);

/* ---- tcgen05 descriptors (src/tcgen05/descriptor.rs) ---------------------------------------- */
/* InstrDescriptor::<KIND>::new for each kind. Element types use the reference's discriminants:
 * F16ElementType F16 0 / Bf16 1; FloatAccumulator F16 0 / F32 1; F8f6f4ElementType E4m3 0,
 * E5m2 1, E2m3 3, E3m2 4, E2m1 5; I8ElementType U8 0 / S8 1; Nvf4ScaleType Ue4m3 0, Ue8m0 1,
 * Ue5m3 2 (descriptor.rs:285-392). PTXSTD_EINVAL where the reference asserts. */
PTXSTD_API int ptxstd_idesc_f16(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out);   /* :520-527 */
PTXSTD_API int ptxstd_idesc_tf32(uint32_t m, uint32_t n, uint32_t* out);                       /* :537-541 */
PTXSTD_API int ptxstd_idesc_f8f6f4(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out); /* :555-564 */
PTXSTD_API int ptxstd_idesc_i8(int a, int b, uint32_t m, uint32_t n, uint32_t* out);           /* :575-578 */
PTXSTD_API int ptxstd_idesc_mxf8f6f4(int a, int b, uint32_t m, uint32_t n, uint32_t* out);     /* :601-611 */
PTXSTD_API int ptxstd_idesc_mxf4(uint32_t m, uint32_t n, uint32_t* out);                       /* :625-628 */
PTXSTD_API int ptxstd_idesc_mxf4nvf4(int scale_type, uint32_t m, uint32_t n, uint32_t* out);   /* :644-653 */
/* The with_* setters (descriptor.rs:400-411, :660-813). kind: MmaKind F16 0, Tf32 1, F8f6f4 2,
 * I8 3, Mxf8f6f4 4, Mxf4 5, Mxf4nvf4 6 (src/tcgen05/mod.rs:322-337). field: 0 sparsity,
 * 1 sparsity_selector, 2 saturate, 3 negate_a, 4 negate_b, 5 major_a, 6 major_b, 7 max_b_shift,
 * 8 scale_a_id, 9 scale_b_id, 10 k. PTXSTD_EINVAL when the kind has no such setter (a compile
 * error in the reference) or the value does not fit. */
PTXSTD_API int ptxstd_idesc_set(uint32_t desc, int kind, int field, uint32_t value, uint32_t* out);
/* SmemDescriptor::from_shared_address (:152-162); swizzle is the Swizzle discriminant 0, 1, 2, 4
 * or 6 (:31-45). with_base_offset (:176-183); add_start_bytes (:231-237). */
PTXSTD_API int ptxstd_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo, int swizzle, uint64_t* out);
PTXSTD_API int ptxstd_smem_desc_with_base_offset(uint64_t desc, uint32_t base_offset, uint64_t* out);
PTXSTD_API int ptxstd_smem_desc_add_start_bytes(uint64_t desc, uint32_t bytes, uint64_t* out);
/* ZeroColumnMask::new / with_sub_mask_start / with_column_shift (:870-921); first_span is
 * ColumnSpan Used 0 / Zeroed 1. */
PTXSTD_API int ptxstd_zero_mask_new(uint32_t zeroed, uint32_t used, uint64_t* out);
PTXSTD_API int ptxstd_zero_mask_with_sub_mask_start(uint64_t mask, uint32_t sub_mask, int first_span,
                                                    uint32_t start_count, uint64_t* out);
PTXSTD_API int ptxstd_zero_mask_with_column_shift(uint64_t mask, uint32_t shift, uint64_t* out);

#ifdef __cplusplus
}
#endif
#endif /* PTXSTD_H */

/*
 * CPU ORACLE — test infrastructure only (see oracle.h for what pins each part).
 *
 * Every function restates the reference's documented semantics in plain C; the file:line cited
 * beside each is the reference code it follows. Built by oracle/Makefile into
 * oracle/_build/liboracle.so; loaded by tests/ and bench.py's CPU-baseline leg through ctypes.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------------------------ */
/* small helpers                                                                              */
/* ------------------------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

int ptxo_hardware_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

/* Runs fn(ctx, lo, hi) over [0, n) split into contiguous ranges on `threads` threads. */
typedef void (*range_fn)(void* ctx, uint64_t lo, uint64_t hi);
typedef struct { range_fn fn; void* ctx; uint64_t lo, hi; } range_job;

static void* range_tramp(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->ctx, j->lo, j->hi);
    return NULL;
}

static void parallel_for(uint64_t n, int threads, range_fn fn, void* ctx) {
    if (threads <= 0) threads = ptxo_hardware_threads();
    if ((uint64_t)threads > n) threads = n ? (int)n : 1;
    if (threads <= 1) { fn(ctx, 0, n); return; }
    pthread_t* tid = (pthread_t*)malloc(sizeof(pthread_t) * threads);
    range_job* jobs = (range_job*)malloc(sizeof(range_job) * threads);
    uint64_t per = n / threads, extra = n % threads, lo = 0;
    for (int t = 0; t < threads; ++t) {
        uint64_t len = per + ((uint64_t)t < extra ? 1 : 0);
        jobs[t].fn = fn; jobs[t].ctx = ctx; jobs[t].lo = lo; jobs[t].hi = lo + len;
        lo += len;
        pthread_create(&tid[t], NULL, range_tramp, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(tid[t], NULL);
    free(tid); free(jobs);
}

/* ------------------------------------------------------------------------------------------ */
/* decode                                                                                     */
/* ------------------------------------------------------------------------------------------ */

/* Restates minifloat_to_f32 (src/data_types/vector.rs:61-95): sign at bit exp+man, the largest
 * exponent encodes specials for IEEE formats (and only with all mantissa bits set for NaN-only
 * formats), exponent 0 is subnormal with scale 2^(1-bias). */
float ptxo_minifloat_to_f32(uint8_t bits8, uint32_t exp_bits, uint32_t man_bits, int32_t bias,
                            int specials) {
    uint32_t bits = bits8;
    int negative = (bits >> (exp_bits + man_bits)) & 1;
    uint32_t e = (bits >> man_bits) & ((1u << exp_bits) - 1);
    uint32_t m = bits & ((1u << man_bits) - 1);
    uint32_t max_e = (1u << exp_bits) - 1, max_m = (1u << man_bits) - 1;
    int special = 0;
    if (e == max_e) {
        if (specials == 1) special = 1;              /* IEEE */
        else if (specials == 2) special = (m == max_m); /* NaN only */
    }
    float mag;
    if (special) {
        mag = (m == 0) ? INFINITY : NAN;
    } else {
        float frac = (e == 0) ? 0.0f : 1.0f;
        int32_t se = (e == 0) ? (1 - bias) : ((int32_t)e - bias);
        float scale = u2f((uint32_t)(se + 127) << 23);
        mag = (frac + (float)m / (float)(1u << man_bits)) * scale;
    }
    return negative ? -mag : mag;
}

/* f8e4m3 decode: minifloat_to_f32(bits, 4, 3, 7, NanOnly) (src/data_types/float8.rs:20). */
float ptxo_e4m3_to_f32(uint8_t b) { return ptxo_minifloat_to_f32(b, 4, 3, 7, 2); }
/* f8e5m2 decode: minifloat_to_f32(bits, 5, 2, 15, Ieee) (src/data_types/float8.rs:79). */
float ptxo_e5m2_to_f32(uint8_t b) { return ptxo_minifloat_to_f32(b, 5, 2, 15, 1); }
/* f4e2m1 decode: minifloat_to_f32(bits, 2, 1, 1, None) (src/data_types/float4.rs:24). */
float ptxo_e2m1_to_f32(uint8_t b) { return ptxo_minifloat_to_f32(b & 0xF, 2, 1, 1, 0); }
/* FP6 (src/data_types/float6.rs: f6e2m3 decode minifloat_to_f32(bits, 2, 3, 1, Specials::None),
 * f6e3m2 decode (bits, 3, 2, 3, Specials::None)); the value is in the low 6 bits. */
float ptxo_e2m3_to_f32(uint8_t b) { return ptxo_minifloat_to_f32(b & 0x3F, 2, 3, 1, 0); }
float ptxo_e3m2_to_f32(uint8_t b) { return ptxo_minifloat_to_f32(b & 0x3F, 3, 2, 3, 0); }

/* f8e8m0 decode (src/data_types/float8.rs:148-152): 0xff NaN, 0 -> 2^-127, else bits << 23. */
float ptxo_ue8m0_to_f32(uint8_t b) {
    if (b == 0xFF) return NAN;
    if (b == 0) return u2f(0x00400000u);
    return u2f((uint32_t)b << 23);
}

/* The device's `to_f32` is to_f16 (`cvt.rn.f16x2.<fmt>x2`) followed by f16::to_f32, which is
 * `self.prim() as f32` (src/data_types/narrow.rs:292-299, src/data_types/float16.rs:90-92), the
 * hardware cvt.f32.f16: finite values are exact, and every NaN becomes the canonical f32 NaN
 * 0x7fffffff whatever its sign or payload (observed on B200 for codes 0x7f and 0xff). */
float ptxo_to_f32_via_half(int format, uint8_t bits) {
    float v;
    switch (format) {
    case PTXO_E4M3: v = ptxo_e4m3_to_f32(bits); break;
    case PTXO_E5M2: v = ptxo_e5m2_to_f32(bits); break;
    case PTXO_E2M3: v = ptxo_e2m3_to_f32(bits); break;
    case PTXO_E3M2: v = ptxo_e3m2_to_f32(bits); break;
    default: v = ptxo_e2m1_to_f32(bits); break;
    }
    if (v != v) return u2f(0x7FFFFFFFu);
    return v;
}

/* ue8m0 `to_f32` goes through bf16 (`cvt.rn.bf16x2.ue8m0x2`, src/data_types/narrow.rs:683-690):
 * NaN becomes the bf16 canonical NaN 0x7fff, widened to 0x7fff0000. */
float ptxo_ue8m0_to_f32_via_bf16(uint8_t bits) {
    if (bits == 0xFF) return u2f(0x7FFF0000u);
    return ptxo_ue8m0_to_f32(bits);
}

/* ------------------------------------------------------------------------------------------ */
/* encode                                                                                     */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    int exp_bits, man_bits, bias;
    uint32_t max_mag;  /* largest finite magnitude code */
    uint8_t nan_code;  /* code written for a NaN input */
    uint8_t sign_bit;
} narrow_fmt;

/* E4M3: max 0x7E = 448, NaN 0x7F (src/data_types/float8.rs:32-35). */
static const narrow_fmt FMT_E4M3 = {4, 3, 7, 0x7E, 0x7F, 0x80};
/* E5M2: max 0x7B = 57344 (src/data_types/float8.rs:96-99); NaN written as 0x7F. */
static const narrow_fmt FMT_E5M2 = {5, 2, 15, 0x7B, 0x7F, 0x80};
/* E2M1: max 0x7 = 6 (src/data_types/float4.rs:35-36); no NaN, so NaN becomes +max
 * (src/data_types/narrow.rs:125-130). */
static const narrow_fmt FMT_E2M1 = {2, 1, 1, 0x7, 0x7, 0x8};
/* E2M3: max 0x1F = 7.5, E3M2: max 0x1F = 28 (src/data_types/float6.rs consts MAX); sign bit 0x20;
 * no NaN, so, as for E2M1, NaN becomes +max. */
static const narrow_fmt FMT_E2M3 = {2, 3, 1, 0x1F, 0x1F, 0x20};
static const narrow_fmt FMT_E3M2 = {3, 2, 3, 0x1F, 0x1F, 0x20};

static inline const narrow_fmt* fmt_of(int format) {
    switch (format) {
    case PTXO_E4M3: return &FMT_E4M3;
    case PTXO_E5M2: return &FMT_E5M2;
    case PTXO_E2M3: return &FMT_E2M3;
    case PTXO_E3M2: return &FMT_E3M2;
    default: return &FMT_E2M1;
    }
}

/* Round-to-nearest-even of a finite, non-negative f32 (given as bits) to the magnitude code of
 * the format, saturating to the largest finite code (.satfinite). Integer formulation: the
 * 24-bit significand is shifted to the quantum of the target binade (or of the subnormal range),
 * with ties to even, then re-encoded. */
static inline uint32_t encode_mag(const narrow_fmt* f, uint32_t a) {
    uint32_t e32 = a >> 23;
    if (e32 == 0) return 0; /* zero or f32 subnormal: far below half the smallest subnormal */
    uint32_t sig = (a & 0x7FFFFFu) | 0x800000u;
    int e = (int)e32 - 127;
    int emin = 1 - f->bias;
    int te = e < emin ? emin : e;
    int shift = 23 - f->man_bits + (te - e);
    uint32_t n;
    if (shift >= 26) {
        n = 0; /* sig < 2^24 <= half a quantum */
    } else {
        n = sig >> shift;
        uint32_t rem = sig & ((1u << shift) - 1);
        uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (n & 1))) n++;
    }
    uint32_t one = 1u << f->man_bits;
    if (n >= (one << 1)) { te++; n >>= 1; }
    uint32_t code;
    if (te == emin && n < one) code = n;
    else code = ((uint32_t)(te + f->bias) << f->man_bits) | (n - one);
    if (code > f->max_mag) code = f->max_mag;
    return code;
}

/* RN .satfinite [.relu] conversion of one f32 (src/data_types/narrow.rs:125-130): out-of-range
 * values and infinities clamp to the largest finite value of matching sign; NaN becomes the
 * format's NaN (FP8) or the largest positive value (FP4); RELU clamps negative results to +0. */
static inline uint8_t encode_narrow(const narrow_fmt* f, float x, int relu) {
    uint32_t u = f2u(x);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return f->nan_code;
    uint8_t sign = (u >> 31) ? f->sign_bit : 0;
    if (relu && sign) return 0;
    uint32_t mag = (a == 0x7F800000u) ? f->max_mag : encode_mag(f, a);
    return (uint8_t)(mag | sign);
}

uint8_t ptxo_f32_to_e4m3(float x, int relu) { return encode_narrow(&FMT_E4M3, x, relu); }
uint8_t ptxo_f32_to_e5m2(float x, int relu) { return encode_narrow(&FMT_E5M2, x, relu); }
uint8_t ptxo_f32_to_e2m1(float x, int relu) { return encode_narrow(&FMT_E2M1, x, relu); }
uint8_t ptxo_f32_to_narrow(int format, float x, int relu) {
    return encode_narrow(fmt_of(format), x, relu);
}

/* ue8m0 encode (src/data_types/narrow.rs:585-593, :600-617): the format holds only powers of
 * two, so RZ keeps the f32 exponent and RP bumps it when any mantissa bit is set; NaN -> 0xff;
 * with .satfinite, overflow (and infinity) clamp to 0xfe = 2^127, without it they give 0xff.
 * Values below 2^-127 (including zero) give the smallest code 0 under RZ; under RP everything in
 * (0, 2^-127] gives 0 and (2^-127, 2^-126) gives 1. The sign is ignored (unsigned format). */
uint8_t ptxo_f32_to_ue8m0(float x, int rnd_up, int satfinite) {
    uint32_t a = f2u(x) & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0xFF;
    if (a == 0x7F800000u) return satfinite ? 0xFE : 0xFF;
    uint32_t e = a >> 23, m = a & 0x7FFFFFu;
    if (e == 0) {
        if (!rnd_up) return 0;
        return (m > 0x400000u) ? 1 : 0;
    }
    uint32_t code = e + ((rnd_up && m) ? 1u : 0u);
    if (code >= 0xFF) return satfinite ? 0xFE : 0xFF;
    return (uint8_t)code;
}

/* bf16 RNE from f32 (src/data_types/bfloat16.rs:104-118); NaN keeps its sign and becomes quiet. */
uint16_t ptxo_f32_to_bf16(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x40);
    uint32_t lsb = (u >> 16) & 1;
    u += 0x7FFFu + lsb;
    return (uint16_t)(u >> 16);
}
float ptxo_bf16_to_f32(uint16_t h) { return u2f((uint32_t)h << 16); }

uint16_t ptxo_f32_to_bf16_mode(float x, int relu, int satfinite) {
    uint32_t u = f2u(x);
    if ((u & 0x7FFFFFFFu) > 0x7F800000u) return 0x7FFF;
    if (relu && (u >> 31)) return 0;
    uint32_t lsb = (u >> 16) & 1;
    uint32_t r = (u & 0x7FFFFFFFu) == 0x7F800000u ? u : u + 0x7FFFu + lsb;
    uint16_t h = (uint16_t)(r >> 16);
    if (satfinite && (h & 0x7FFF) == 0x7F80) h = (uint16_t)((h & 0x8000) | 0x7F7F);
    return h;
}

/* ------------------------------------------------------------------------------------------ */
/* scaled up-conversion to bf16                                                               */
/* ------------------------------------------------------------------------------------------ */

static float narrow_value(int format, uint8_t code) {
    switch (format) {
    case PTXO_E4M3: return ptxo_e4m3_to_f32(code);
    case PTXO_E5M2: return ptxo_e5m2_to_f32(code);
    case PTXO_E2M3: return ptxo_e2m3_to_f32(code);
    case PTXO_E3M2: return ptxo_e3m2_to_f32(code);
    default: return ptxo_e2m1_to_f32(code);
    }
}

uint16_t ptxo_narrow_to_f16(int format, uint8_t code) {
    float v = narrow_value(format, code);
    if (v != v) return 0x7FFF;
    uint32_t u = f2u(v), sign = (u >> 16) & 0x8000u, a = u & 0x7FFFFFFFu;
    if (a == 0) return (uint16_t)sign;
    if (a == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
    int e = (int)(a >> 23) - 127;
    uint32_t m = (a & 0x7FFFFFu) | 0x800000u;
    if (e >= -14) /* normal f16: the narrow value has at most 4 significant bits, exact */
        return (uint16_t)(sign | ((uint32_t)(e + 15) << 10) | ((m >> 13) & 0x3FFu));
    return (uint16_t)(sign | (m >> (13 + (-14 - e)))); /* subnormal f16, exact (>= 2^-24) */
}

uint16_t ptxo_to_bf16_scaled(int format, uint8_t code, uint8_t scale, int relu, int satfinite) {
    float v = narrow_value(format, code);
    if (v != v || scale == 0xFF) return 0x7FFF;
    double p = (double)v * ldexp(1.0, (int)scale - 127); /* exact: <= 4 significant bits */
    int neg = signbit(p) != 0;
    if (relu && neg) return 0;
    double a = fabs(p);
    uint16_t sign = neg ? 0x8000 : 0;
    if (isinf(a)) return (uint16_t)(sign | (satfinite ? 0x7F7F : 0x7F80));
    if (a == 0.0) return sign;
    /* quantum: 2^(e-7) in the normal range, 2^-133 below 2^-126 */
    int e;
    frexp(a, &e);
    e -= 1;
    double q = ldexp(1.0, e < -126 ? -133 : e - 7);
    double m = a / q, r = nearbyint(m); /* round half to even (default rounding mode) */
    double b = r * q;
    if (b >= ldexp(1.0, 128)) return (uint16_t)(sign | (satfinite ? 0x7F7F : 0x7F80));
    return (uint16_t)(sign | (f2u((float)b) >> 16));
}

typedef struct {
    int format, relu, sat; const uint8_t *codes, *scales; uint16_t* out; size_t block;
} scaled_ctx;

static void scaled_range(void* p, uint64_t lo, uint64_t hi) {
    scaled_ctx* c = (scaled_ctx*)p;
    for (uint64_t i = lo; i < hi; ++i) {
        uint8_t code = c->format == PTXO_E2M1 ? (uint8_t)((c->codes[i / 2] >> (4 * (i % 2))) & 0xF)
                                              : c->codes[i];
        c->out[i] = ptxo_to_bf16_scaled(c->format, code, c->scales[i / c->block], c->relu, c->sat);
    }
}

void ptxo_to_bf16_scaled_array(int format, const uint8_t* codes, const uint8_t* scales,
                               uint16_t* out, size_t n, size_t block, int relu, int satfinite,
                               int threads) {
    scaled_ctx c = {format, relu, satfinite, codes, scales, out, block};
    parallel_for(n, threads, scaled_range, &c);
}

/* ------------------------------------------------------------------------------------------ */
/* stochastic rounding                                                                        */
/* ------------------------------------------------------------------------------------------ */

static inline uint32_t bitrev8(uint32_t v) {
    uint32_t r = 0;
    for (int i = 0; i < 8; ++i) r |= ((v >> i) & 1u) << (7 - i);
    return r;
}
static inline uint32_t bitrev16(uint32_t v) { return (bitrev8(v & 0xFFu) << 8) | bitrev8(v >> 8); }

/* Element k's random value. FP8/FP6 (narrow.rs quad_from_f32_stochastic, float8.rs:59: "the lower
 * 16 bits are used for elements 0 and 1 and the upper 16 bits for elements 2 and 3"): the even
 * element reads its half most significant bit first, the odd element reads it bit-reversed (bit
 * 0 or 16 most significant). E2M1 (float4.rs:60: "the lower 8 bits of both 16-bit halves are used
 * for elements 0 and 1 and the upper 8 bits of both halves for elements 2 and 3"): a 16-bit value
 * from two bytes, the byte of the upper half first for the even element; the odd element reads
 * both bytes bit-reversed, the lower half's first. bf16 (bfloat16.rs:572-579): the low 16 bits
 * for element 0, the high 16 for element 1; f16 (float16.rs:740-745): the 13 low bits of each
 * half. */
uint32_t ptxo_rs_random(int kind, uint32_t rb, int k) {
    switch (kind) {
    case PTXO_RS_X4: {
        uint32_t half = (k < 2) ? (rb & 0xFFFFu) : (rb >> 16);
        return (k & 1) ? bitrev16(half) : half;
    }
    case PTXO_RS_E2M1:
        switch (k) {
        case 0: return (((rb >> 16) & 0xFFu) << 8) | (rb & 0xFFu);
        case 1: return (bitrev8(rb & 0xFFu) << 8) | bitrev8((rb >> 16) & 0xFFu);
        case 2: return ((rb >> 24) << 8) | ((rb >> 8) & 0xFFu);
        default: return (bitrev8((rb >> 8) & 0xFFu) << 8) | bitrev8(rb >> 24);
        }
    case PTXO_RS_BF16: return k ? (rb >> 16) : (rb & 0xFFFFu);
    default: return (k ? (rb >> 16) : rb) & 0x1FFFu;
    }
}

/* |x| (finite, bits a, a normal f32) split at the quantum of the target binade: the number n of
 * whole quanta and the carry of (discarded part, truncated to w bits) + r out of w bits.
 * shift = number of significand bits below the quantum. */
static inline uint32_t rs_quanta(uint32_t a, int man_bits, int emin, uint32_t r, int w, int* te) {
    uint64_t sig = (uint64_t)((a & 0x7FFFFFu) | 0x800000u);
    int e = (int)(a >> 23) - 127;
    *te = e < emin ? emin : e;
    int shift = 23 - man_bits + (*te - e);
    uint64_t n = 0, fw = 0;
    if (shift < 64) {
        n = sig >> shift;
        fw = ((sig & ((1ull << shift) - 1)) << w) >> shift;
    }
    if (fw + r >= (1ull << w)) n++;
    return (uint32_t)n;
}

/* Stochastic rounding of a finite, non-negative f32 (bits a) to a narrow magnitude code with
 * .satfinite. f32 subnormals lie below 2^-126, where every format's discarded fraction has no
 * set bit among its top 16, so they give 0. */
static inline uint32_t encode_mag_rs(const narrow_fmt* f, uint32_t a, uint32_t r) {
    if ((a >> 23) == 0) return 0;
    int emin = 1 - f->bias, te;
    uint32_t n = rs_quanta(a, f->man_bits, emin, r, 16, &te);
    uint32_t one = 1u << f->man_bits;
    if (n >= (one << 1)) { te++; n >>= 1; }
    uint32_t code;
    if (te == emin && n < one) code = n;
    else code = ((uint32_t)(te + f->bias) << f->man_bits) | (n - one);
    if (code > f->max_mag) code = f->max_mag;
    return code;
}

uint8_t ptxo_f32_to_narrow_rs(int format, float x, uint32_t r, int relu) {
    const narrow_fmt* f = fmt_of(format);
    uint32_t u = f2u(x);
    uint32_t a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return f->nan_code;
    uint8_t sign = (u >> 31) ? f->sign_bit : 0;
    if (relu && sign) return 0;
    uint32_t mag = (a == 0x7F800000u) ? f->max_mag : encode_mag_rs(f, a, r);
    return (uint8_t)(mag | sign);
}

/* bf16 keeps the f32 exponent, so the discarded part is the low 16 bits of the pattern (for f32
 * subnormals too: bf16's subnormal quantum is 2^-133, bit 16 of the f32 subnormal). */
uint16_t ptxo_f32_to_bf16_rs(float x, uint32_t r, int relu, int satfinite) {
    uint32_t u = f2u(x), a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7FFF;
    uint32_t m;
    if (a == 0x7F800000u) {
        m = satfinite ? 0x7F7Fu : 0x7F80u;
    } else {
        m = a >> 16;
        if ((a & 0xFFFFu) + (r & 0xFFFFu) >= 0x10000u) m++;
        if (m >= 0x7F80u) m = satfinite ? 0x7F7Fu : 0x7F80u;
    }
    if (relu && (u >> 31)) return 0;
    return (uint16_t)(((u >> 16) & 0x8000u) | m);
}

uint16_t ptxo_f32_to_f16_rs(float x, uint32_t r, int relu, int satfinite) {
    uint32_t u = f2u(x), a = u & 0x7FFFFFFFu;
    if (a > 0x7F800000u) return 0x7FFF;
    uint32_t m;
    if (a == 0x7F800000u) {
        m = satfinite ? 0x7BFFu : 0x7C00u;
    } else if ((a >> 23) == 0) {
        m = 0; /* below 2^-126: nothing within the top 13 bits of a 2^-24 quantum */
    } else {
        int te;
        uint32_t n = rs_quanta(a, 10, -14, r & 0x1FFFu, 13, &te);
        if (te == -14) {
            m = n; /* subnormal, or the first normal binade reached by the carry */
        } else {
            if (n == 2048) { te++; n = 1024; }
            m = ((uint32_t)(te + 15) << 10) | (n - 1024);
        }
        if (m >= 0x7C00u) m = satfinite ? 0x7BFFu : 0x7C00u;
    }
    if (relu && (u >> 31)) return 0;
    return (uint16_t)(((u >> 16) & 0x8000u) | m);
}

uint64_t ptxo_splitmix64(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint32_t ptxo_sr_rbits(uint64_t seed, uint64_t group) {
    uint64_t h = ptxo_splitmix64(seed, group >> 1);
    return (group & 1) ? (uint32_t)(h >> 32) : (uint32_t)h;
}

/* ------------------------------------------------------------------------------------------ */
/* bulk conversions                                                                           */
/* ------------------------------------------------------------------------------------------ */

typedef struct { int format, relu; const float* x; uint8_t* out; } enc_ctx;

static void enc_range(void* p, uint64_t lo, uint64_t hi) {
    enc_ctx* c = (enc_ctx*)p;
    const narrow_fmt* f = fmt_of(c->format);
    if (c->format == PTXO_E2M1) {
        /* lo/hi count bytes (pairs); element 0 in the low nibble (src/data_types/float4.rs:5-6). */
        for (uint64_t i = lo; i < hi; ++i) {
            uint8_t l = encode_narrow(f, c->x[2 * i], c->relu);
            uint8_t h = encode_narrow(f, c->x[2 * i + 1], c->relu);
            c->out[i] = (uint8_t)(l | (h << 4));
        }
    } else {
        for (uint64_t i = lo; i < hi; ++i) c->out[i] = encode_narrow(f, c->x[i], c->relu);
    }
}

void ptxo_encode_array(int format, const float* x, uint8_t* out, size_t n, int relu,
                       int threads) {
    enc_ctx c = {format, relu, x, out};
    parallel_for(format == PTXO_E2M1 ? n / 2 : n, threads, enc_range, &c);
}

typedef struct { int format; const uint8_t* codes; float* out; } dec_ctx;

static void dec_range(void* p, uint64_t lo, uint64_t hi) {
    dec_ctx* c = (dec_ctx*)p;
    if (c->format == PTXO_E2M1) {
        for (uint64_t i = lo; i < hi; ++i) {
            c->out[2 * i] = ptxo_to_f32_via_half(PTXO_E2M1, c->codes[i] & 0xF);
            c->out[2 * i + 1] = ptxo_to_f32_via_half(PTXO_E2M1, c->codes[i] >> 4);
        }
    } else {
        for (uint64_t i = lo; i < hi; ++i) c->out[i] = ptxo_to_f32_via_half(c->format, c->codes[i]);
    }
}

void ptxo_decode_array(int format, const uint8_t* codes, float* out, size_t n, int threads) {
    dec_ctx c = {format, codes, out};
    parallel_for(format == PTXO_E2M1 ? n / 2 : n, threads, dec_range, &c);
}

typedef struct { const float* x; uint8_t* out; int up, sat; } ue_ctx;

static void ue_range(void* p, uint64_t lo, uint64_t hi) {
    ue_ctx* c = (ue_ctx*)p;
    for (uint64_t i = lo; i < hi; ++i) c->out[i] = ptxo_f32_to_ue8m0(c->x[i], c->up, c->sat);
}

void ptxo_ue8m0_encode_array(const float* x, uint8_t* out, size_t n, int rnd_up, int satfinite,
                             int threads) {
    ue_ctx c = {x, out, rnd_up, satfinite};
    parallel_for(n, threads, ue_range, &c);
}

typedef struct {
    int format, relu, sat; const float* x; const uint32_t* rb; uint8_t* out8; uint16_t* out16;
} rs_ctx;

static void rs_range(void* p, uint64_t lo, uint64_t hi) {
    rs_ctx* c = (rs_ctx*)p;
    if (c->format == PTXO_E2M1) {
        for (uint64_t i = lo; i < hi; ++i) { /* i indexes output bytes: elements 2i, 2i + 1 */
            uint8_t b = 0;
            for (int h = 0; h < 2; ++h) {
                uint64_t e = 2 * i + h;
                uint32_t r = ptxo_rs_random(PTXO_RS_E2M1, c->rb[e / 4], (int)(e % 4));
                b |= (uint8_t)(ptxo_f32_to_narrow_rs(PTXO_E2M1, c->x[e], r, c->relu) << (4 * h));
            }
            c->out8[i] = b;
        }
    } else if (c->format >= 0) {
        for (uint64_t i = lo; i < hi; ++i) {
            uint32_t r = ptxo_rs_random(PTXO_RS_X4, c->rb[i / 4], (int)(i % 4));
            c->out8[i] = ptxo_f32_to_narrow_rs(c->format, c->x[i], r, c->relu);
        }
    } else {
        int bf = c->format == -1;
        for (uint64_t i = lo; i < hi; ++i) {
            uint32_t r = ptxo_rs_random(bf ? PTXO_RS_BF16 : PTXO_RS_F16, c->rb[i / 2], (int)(i % 2));
            c->out16[i] = bf ? ptxo_f32_to_bf16_rs(c->x[i], r, c->relu, c->sat)
                             : ptxo_f32_to_f16_rs(c->x[i], r, c->relu, c->sat);
        }
    }
}

void ptxo_encode_rs_array(int format, const float* x, const uint32_t* rbits, uint8_t* out,
                          size_t n, int relu, int threads) {
    rs_ctx c = {format, relu, 1, x, rbits, out, NULL};
    parallel_for(format == PTXO_E2M1 ? n / 2 : n, threads, rs_range, &c);
}

void ptxo_bf16_rs_array(const float* x, const uint32_t* rbits, uint16_t* out, size_t n, int relu,
                        int satfinite, int threads) {
    rs_ctx c = {-1, relu, satfinite, x, rbits, NULL, out};
    parallel_for(n, threads, rs_range, &c);
}

void ptxo_f16_rs_array(const float* x, const uint32_t* rbits, uint16_t* out, size_t n, int relu,
                       int satfinite, int threads) {
    rs_ctx c = {-2, relu, satfinite, x, rbits, NULL, out};
    parallel_for(n, threads, rs_range, &c);
}

/* ------------------------------------------------------------------------------------------ */
/* exhaustive sweep support                                                                   */
/* ------------------------------------------------------------------------------------------ */

uint8_t ptxo_encode_variant(int variant, float x) {
    switch (variant) {
    case PTXO_V_E4M3: return encode_narrow(&FMT_E4M3, x, 0);
    case PTXO_V_E5M2: return encode_narrow(&FMT_E5M2, x, 0);
    case PTXO_V_E2M1: return encode_narrow(&FMT_E2M1, x, 0);
    case PTXO_V_E4M3_RELU: return encode_narrow(&FMT_E4M3, x, 1);
    case PTXO_V_E5M2_RELU: return encode_narrow(&FMT_E5M2, x, 1);
    case PTXO_V_E2M1_RELU: return encode_narrow(&FMT_E2M1, x, 1);
    case PTXO_V_UE8M0_RZ: return ptxo_f32_to_ue8m0(x, 0, 1);
    case PTXO_V_UE8M0_RP: return ptxo_f32_to_ue8m0(x, 1, 1);
    case PTXO_V_E2M3: return encode_narrow(&FMT_E2M3, x, 0);
    case PTXO_V_E3M2: return encode_narrow(&FMT_E3M2, x, 0);
    case PTXO_V_E2M3_RELU: return encode_narrow(&FMT_E2M3, x, 1);
    default: return encode_narrow(&FMT_E3M2, x, 1);
    }
}

int ptxo_sweep_width(int variant) { return variant >= PTXO_V_BF16_RS ? 2 : 1; }

uint32_t ptxo_sweep_code(int variant, uint64_t p) {
    float x = u2f((uint32_t)p);
    if (variant < PTXO_V_E4M3_RS) return ptxo_encode_variant(variant, x);
    if (variant < PTXO_V_BF16_RS) {
        static const int fmts[5] = {PTXO_E4M3, PTXO_E5M2, PTXO_E2M3, PTXO_E3M2, PTXO_E2M1};
        int v = variant - PTXO_V_E4M3_RS;
        int fmt = fmts[v % 5], relu = v >= 5;
        uint32_t rb = ptxo_sr_rbits(PTXO_SWEEP_SEED, p >> 2);
        uint32_t r = ptxo_rs_random(fmt == PTXO_E2M1 ? PTXO_RS_E2M1 : PTXO_RS_X4, rb, (int)(p & 3));
        return ptxo_f32_to_narrow_rs(fmt, x, r, relu);
    }
    if (variant >= PTXO_V_BF16_RN) {
        int w = variant - PTXO_V_BF16_RN;
        return ptxo_f32_to_bf16_mode(x, w & 1, (w >> 1) & 1);
    }
    int v = variant - PTXO_V_BF16_RS;
    int bf = v < 4, relu = v & 1, sat = (v >> 1) & 1;
    uint32_t rb = ptxo_sr_rbits(PTXO_SWEEP_SEED, p >> 1);
    uint32_t r = ptxo_rs_random(bf ? PTXO_RS_BF16 : PTXO_RS_F16, rb, (int)(p & 1));
    return bf ? ptxo_f32_to_bf16_rs(x, r, relu, sat) : ptxo_f32_to_f16_rs(x, r, relu, sat);
}

typedef struct {
    int variant; uint64_t base; const uint8_t* dev;
    uint32_t* report; uint64_t max_report;
    uint64_t mismatches; pthread_mutex_t mu;
} sweep_ctx;

static void sweep_range(void* p, uint64_t lo, uint64_t hi) {
    sweep_ctx* c = (sweep_ctx*)p;
    uint64_t local = 0;
    const int w = ptxo_sweep_width(c->variant);
    for (uint64_t i = lo; i < hi; ++i) {
        uint32_t bits = (uint32_t)(c->base + i);
        uint32_t want = ptxo_sweep_code(c->variant, c->base + i);
        uint32_t got = c->dev[w * i];
        if (w == 2) got |= (uint32_t)c->dev[w * i + 1] << 8;
        if (want != got) {
            pthread_mutex_lock(&c->mu);
            if (c->mismatches < c->max_report && c->report) {
                c->report[3 * c->mismatches] = bits;
                c->report[3 * c->mismatches + 1] = got;
                c->report[3 * c->mismatches + 2] = want;
            }
            c->mismatches++;
            pthread_mutex_unlock(&c->mu);
            local++;
        }
    }
    (void)local;
}

uint64_t ptxo_sweep_compare(int variant, uint64_t base, uint64_t n, const uint8_t* device_out,
                            uint32_t* report, uint64_t max_report, int threads) {
    sweep_ctx c;
    c.variant = variant; c.base = base; c.dev = device_out; c.report = report;
    c.max_report = max_report; c.mismatches = 0;
    pthread_mutex_init(&c.mu, NULL);
    parallel_for(n, threads, sweep_range, &c);
    pthread_mutex_destroy(&c.mu);
    return c.mismatches;
}

#define FNV_OFFSET 0xcbf29ce484222325ull
#define FNV_PRIME 0x100000001b3ull

uint64_t ptxo_fnv1a64(const uint8_t* data, size_t n, uint64_t seed) {
    uint64_t h = seed ? seed : FNV_OFFSET;
    for (size_t i = 0; i < n; ++i) { h ^= data[i]; h *= FNV_PRIME; }
    return h;
}

typedef struct { int variant; uint64_t base; uint64_t* part; uint64_t chunk; } dig_ctx;

static void dig_range(void* p, uint64_t lo, uint64_t hi) {
    dig_ctx* c = (dig_ctx*)p;
    const int w = ptxo_sweep_width(c->variant);
    for (uint64_t k = lo; k < hi; ++k) {
        uint64_t h = FNV_OFFSET;
        uint64_t b0 = c->base + k * c->chunk;
        for (uint64_t i = 0; i < c->chunk; ++i) {
            uint32_t code = ptxo_sweep_code(c->variant, b0 + i);
            for (int j = 0; j < w; ++j) {
                h ^= (code >> (8 * j)) & 0xFFu;
                h *= FNV_PRIME;
            }
        }
        c->part[k] = h;
    }
}

/* Digest of [base, base + n): FNV-1a 64 of each 2^16-byte piece of the codes (width bytes per
 * input, little-endian), then FNV-1a 64 over those digests' little-endian bytes (so that the
 * pieces can be hashed in parallel). n * width must be a multiple of 2^16. */
uint64_t ptxo_sweep_digest(int variant, uint64_t base, uint64_t n, int threads) {
    const uint64_t chunk = (1u << 16) / (uint64_t)ptxo_sweep_width(variant);
    uint64_t parts = n / chunk;
    uint64_t* part = (uint64_t*)malloc(sizeof(uint64_t) * (parts ? parts : 1));
    dig_ctx c = {variant, base, part, chunk};
    parallel_for(parts, threads, dig_range, &c);
    uint64_t h = ptxo_fnv1a64((const uint8_t*)part, parts * 8, 0);
    free(part);
    return h;
}

typedef struct { const uint8_t* data; uint64_t* part; uint64_t chunk; } digb_ctx;

static void digb_range(void* p, uint64_t lo, uint64_t hi) {
    digb_ctx* c = (digb_ctx*)p;
    for (uint64_t k = lo; k < hi; ++k) c->part[k] = ptxo_fnv1a64(c->data + k * c->chunk, c->chunk, 0);
}

/* The same digest scheme as ptxo_sweep_digest, over given bytes (n a multiple of 2^16). */
uint64_t ptxo_digest_bytes(const uint8_t* data, uint64_t n, int threads) {
    const uint64_t chunk = 1u << 16;
    uint64_t parts = n / chunk;
    uint64_t* part = (uint64_t*)malloc(sizeof(uint64_t) * (parts ? parts : 1));
    digb_ctx c = {data, part, chunk};
    parallel_for(parts, threads, digb_range, &c);
    uint64_t h = ptxo_fnv1a64((const uint8_t*)part, parts * 8, 0);
    free(part);
    return h;
}

/* ------------------------------------------------------------------------------------------ */
/* block-scale recipes                                                                        */
/* ------------------------------------------------------------------------------------------ */

/* NaN-propagating max of |x| over a block (the `.NaN` form of redux.sync.max.abs.f32,
 * src/warp_collectives.rs:679-700). */
static inline float block_amax(const float* x, int n) {
    float m = 0.0f;
    for (int i = 0; i < n; ++i) {
        float a = fabsf(x[i]);
        if (a != a) return a;
        if (a > m) m = a;
    }
    return m;
}

/* 2^-(code-127) as an f32 (exact: 2^127 .. 2^-127, the last an f32 subnormal). */
static inline float ue8m0_inverse(uint8_t code) {
    if (code == 0xFF) return NAN;
    int e = 127 - (int)code; /* -127 .. 127 */
    if (e >= -126) return u2f((uint32_t)(e + 127) << 23);
    return u2f(0x00400000u); /* 2^-127 */
}

/* MXFP8 scale of one 32-block: u = f8e8m0::from_f32::<TowardZero, SaturateFinite>(amax)
 * (src/data_types/narrow.rs:600-617), minus E4M3's emax 8, clamped at 0; NaN stays NaN. */
uint8_t ptxo_mxfp8_block(const float* x32, uint8_t* q32) {
    float amax = block_amax(x32, 32);
    uint8_t u = ptxo_f32_to_ue8m0(amax, 0, 1);
    uint8_t code = (u == 0xFF) ? 0xFF : (u > 8 ? (uint8_t)(u - 8) : 0);
    float inv = ue8m0_inverse(code);
    for (int i = 0; i < 32; ++i) q32[i] = encode_narrow(&FMT_E4M3, x32[i] * inv, 0);
    return code;
}

/* NVFP4 block of 16: sf = e4m3_rn_satfinite(amax / (6 g)); r = 1 / (sf g) (0 when sf g == 0);
 * q = e2m1_rn_satfinite(x r). All f32 operations are single IEEE roundings. */
uint8_t ptxo_nvfp4_block(const float* x16, float g, uint8_t* q16) {
    float amax = block_amax(x16, 16);
    float six_g = 6.0f * g;
    float s = amax / six_g;
    uint8_t sf = encode_narrow(&FMT_E4M3, s, 0);
    float t = ptxo_e4m3_to_f32(sf) * g;
    float r = (t == 0.0f) ? 0.0f : 1.0f / t;
    for (int i = 0; i < 16; ++i) q16[i] = encode_narrow(&FMT_E2M1, x16[i] * r, 0);
    return sf;
}

typedef struct {
    const uint16_t* x; int64_t cols; uint8_t* q; uint8_t* sf; float g;
} quant_ctx;

static void mxfp8_rows(void* p, uint64_t lo, uint64_t hi) {
    quant_ctx* c = (quant_ctx*)p;
    float buf[32];
    for (uint64_t r = lo; r < hi; ++r) {
        const uint16_t* xr = c->x + r * c->cols;
        for (int64_t b = 0; b < c->cols / 32; ++b) {
            for (int i = 0; i < 32; ++i) buf[i] = ptxo_bf16_to_f32(xr[b * 32 + i]);
            c->sf[r * (c->cols / 32) + b] = ptxo_mxfp8_block(buf, c->q + r * c->cols + b * 32);
        }
    }
}

void ptxo_quantize_mxfp8(const uint16_t* x, int64_t rows, int64_t cols, uint8_t* q, uint8_t* sf,
                         int threads) {
    quant_ctx c = {x, cols, q, sf, 0.0f};
    parallel_for((uint64_t)rows, threads, mxfp8_rows, &c);
}

static void nvfp4_rows(void* p, uint64_t lo, uint64_t hi) {
    quant_ctx* c = (quant_ctx*)p;
    float buf[16];
    uint8_t nib[16];
    for (uint64_t r = lo; r < hi; ++r) {
        const uint16_t* xr = c->x + r * c->cols;
        uint8_t* qr = c->q + r * (c->cols / 2);
        for (int64_t b = 0; b < c->cols / 16; ++b) {
            for (int i = 0; i < 16; ++i) buf[i] = ptxo_bf16_to_f32(xr[b * 16 + i]);
            c->sf[r * (c->cols / 16) + b] = ptxo_nvfp4_block(buf, c->g, nib);
            for (int i = 0; i < 8; ++i) qr[b * 8 + i] = (uint8_t)(nib[2 * i] | (nib[2 * i + 1] << 4));
        }
    }
}

int ptxo_quantize_nvfp4(const uint16_t* x, int64_t rows, int64_t cols, float g, uint8_t* q,
                        uint8_t* sf, int threads) {
    if (!(g > 0.0f) || isinf(g)) return -1;
    quant_ctx c = {x, cols, q, sf, g};
    parallel_for((uint64_t)rows, threads, nvfp4_rows, &c);
    return 0;
}

typedef struct {
    const uint16_t* x; int64_t cols; uint8_t* q; uint8_t* sf; float g; uint64_t seed;
} quant_rs_ctx;

/* Element i of the flat input: rs_random(kind, sr_rbits(seed, i / 4), i % 4). */
static inline uint32_t quant_rs_random(uint64_t seed, uint64_t i, int kind) {
    return ptxo_rs_random(kind, ptxo_sr_rbits(seed, i >> 2), (int)(i & 3));
}

static void mxfp8_rs_rows(void* p, uint64_t lo, uint64_t hi) {
    quant_rs_ctx* c = (quant_rs_ctx*)p;
    float buf[32];
    for (uint64_t r = lo; r < hi; ++r) {
        const uint16_t* xr = c->x + r * c->cols;
        for (int64_t b = 0; b < c->cols / 32; ++b) {
            for (int i = 0; i < 32; ++i) buf[i] = ptxo_bf16_to_f32(xr[b * 32 + i]);
            uint8_t qtmp[32];
            uint8_t code = ptxo_mxfp8_block(buf, qtmp); /* the scale; elements redone below */
            float inv = ue8m0_inverse(code);
            uint64_t e0 = r * (uint64_t)c->cols + (uint64_t)b * 32;
            for (int i = 0; i < 32; ++i)
                c->q[e0 + i] = ptxo_f32_to_narrow_rs(PTXO_E4M3, buf[i] * inv,
                                                     quant_rs_random(c->seed, e0 + i, PTXO_RS_X4), 0);
            c->sf[r * (c->cols / 32) + b] = code;
        }
    }
}

void ptxo_quantize_mxfp8_rs(const uint16_t* x, int64_t rows, int64_t cols, uint64_t seed,
                            uint8_t* q, uint8_t* sf, int threads) {
    quant_rs_ctx c = {x, cols, q, sf, 0.0f, seed};
    parallel_for((uint64_t)rows, threads, mxfp8_rs_rows, &c);
}

static void nvfp4_rs_rows(void* p, uint64_t lo, uint64_t hi) {
    quant_rs_ctx* c = (quant_rs_ctx*)p;
    float buf[16];
    uint8_t nib[16];
    for (uint64_t r = lo; r < hi; ++r) {
        const uint16_t* xr = c->x + r * c->cols;
        uint8_t* qr = c->q + r * (c->cols / 2);
        for (int64_t b = 0; b < c->cols / 16; ++b) {
            for (int i = 0; i < 16; ++i) buf[i] = ptxo_bf16_to_f32(xr[b * 16 + i]);
            uint8_t sf = ptxo_nvfp4_block(buf, c->g, nib); /* the scale; elements redone below */
            float t = ptxo_e4m3_to_f32(sf) * c->g;
            float rcp = (t == 0.0f) ? 0.0f : 1.0f / t;
            uint64_t e0 = r * (uint64_t)c->cols + (uint64_t)b * 16;
            for (int i = 0; i < 16; ++i)
                nib[i] = ptxo_f32_to_narrow_rs(PTXO_E2M1, buf[i] * rcp,
                                               quant_rs_random(c->seed, e0 + i, PTXO_RS_E2M1), 0);
            c->sf[r * (c->cols / 16) + b] = sf;
            for (int i = 0; i < 8; ++i) qr[b * 8 + i] = (uint8_t)(nib[2 * i] | (nib[2 * i + 1] << 4));
        }
    }
}

int ptxo_quantize_nvfp4_rs(const uint16_t* x, int64_t rows, int64_t cols, float g, uint64_t seed,
                           uint8_t* q, uint8_t* sf, int threads) {
    if (!(g > 0.0f) || isinf(g)) return -1;
    quant_rs_ctx c = {x, cols, q, sf, g, seed};
    parallel_for((uint64_t)rows, threads, nvfp4_rs_rows, &c);
    return 0;
}

/* ------------------------------------------------------------------------------------------ */
/* GEMM references                                                                            */
/* ------------------------------------------------------------------------------------------ */

typedef struct {
    const uint8_t *A, *B, *sfA, *sfB, *W, *sfW;
    const uint16_t* x;
    float sa, sb, ga, gb, gw;
    int64_t M, N, K;
    const int64_t *rows, *cols;
    double *ref, *mag;
} gemm_ctx;

static void fp8_samples(void* p, uint64_t lo, uint64_t hi) {
    gemm_ctx* c = (gemm_ctx*)p;
    double lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = ptxo_e4m3_to_f32((uint8_t)i);
    for (uint64_t s = lo; s < hi; ++s) {
        const uint8_t* a = c->A + c->rows[s] * c->K;
        const uint8_t* b = c->B + c->cols[s] * c->K;
        double acc = 0, mag = 0;
        for (int64_t k = 0; k < c->K; ++k) {
            double t = lut[a[k]] * lut[b[k]];
            acc += t; mag += fabs(t);
        }
        double sc = (double)c->sa * (double)c->sb;
        c->ref[s] = acc * sc; c->mag[s] = mag * fabs(sc);
    }
}

void ptxo_gemm_fp8_ref(const uint8_t* A, const uint8_t* B, int64_t M, int64_t N, int64_t K,
                       float sa, float sb, const int64_t* rows, const int64_t* cols,
                       int64_t n_samples, double* ref, double* mag, int threads) {
    gemm_ctx c; memset(&c, 0, sizeof c);
    c.A = A; c.B = B; c.M = M; c.N = N; c.K = K; c.sa = sa; c.sb = sb;
    c.rows = rows; c.cols = cols; c.ref = ref; c.mag = mag;
    parallel_for((uint64_t)n_samples, threads, fp8_samples, &c);
}

static inline double nvfp4_elem(const uint8_t* q, const uint8_t* sf, int64_t k) {
    uint8_t byte = q[k >> 1];
    uint8_t nib = (k & 1) ? (byte >> 4) : (byte & 0xF);
    return (double)ptxo_e2m1_to_f32(nib) * (double)ptxo_e4m3_to_f32(sf[k >> 4]);
}

static void nvfp4_samples(void* p, uint64_t lo, uint64_t hi) {
    gemm_ctx* c = (gemm_ctx*)p;
    for (uint64_t s = lo; s < hi; ++s) {
        const uint8_t* a = c->A + c->rows[s] * (c->K / 2);
        const uint8_t* sa = c->sfA + c->rows[s] * (c->K / 16);
        const uint8_t* b = c->B + c->cols[s] * (c->K / 2);
        const uint8_t* sb = c->sfB + c->cols[s] * (c->K / 16);
        double acc = 0, mag = 0;
        for (int64_t k = 0; k < c->K; ++k) {
            double t = nvfp4_elem(a, sa, k) * nvfp4_elem(b, sb, k);
            acc += t; mag += fabs(t);
        }
        double g = (double)c->ga * (double)c->gb;
        c->ref[s] = acc * g; c->mag[s] = mag * fabs(g);
    }
}

void ptxo_gemm_nvfp4_ref(const uint8_t* A, const uint8_t* sfA, float ga, const uint8_t* B,
                         const uint8_t* sfB, float gb, int64_t M, int64_t N, int64_t K,
                         const int64_t* rows, const int64_t* cols, int64_t n_samples, double* ref,
                         double* mag, int threads) {
    gemm_ctx c; memset(&c, 0, sizeof c);
    c.A = A; c.sfA = sfA; c.ga = ga; c.B = B; c.sfB = sfB; c.gb = gb;
    c.M = M; c.N = N; c.K = K; c.rows = rows; c.cols = cols; c.ref = ref; c.mag = mag;
    parallel_for((uint64_t)n_samples, threads, nvfp4_samples, &c);
}

/* MXFP8 element: E4M3 code times its UE8M0 block scale (OCP MX; f8e8m0 decode 2^(b-127),
 * src/data_types/float8.rs:148-152; f8e4m3 decode, vector.rs:61-95). */
static inline double mxfp8_elem(const uint8_t* q, const uint8_t* sf, int64_t k, const double* lut) {
    return lut[q[k]] * (double)ptxo_ue8m0_to_f32(sf[k >> 5]);
}

static void mxfp8_samples(void* p, uint64_t lo, uint64_t hi) {
    gemm_ctx* c = (gemm_ctx*)p;
    double lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = ptxo_e4m3_to_f32((uint8_t)i);
    for (uint64_t s = lo; s < hi; ++s) {
        const uint8_t* a = c->A + c->rows[s] * c->K;
        const uint8_t* sa = c->sfA + c->rows[s] * (c->K / 32);
        const uint8_t* b = c->B + c->cols[s] * c->K;
        const uint8_t* sb = c->sfB + c->cols[s] * (c->K / 32);
        double acc = 0, mag = 0;
        for (int64_t k = 0; k < c->K; ++k) {
            double t = mxfp8_elem(a, sa, k, lut) * mxfp8_elem(b, sb, k, lut);
            acc += t; mag += fabs(t);
        }
        c->ref[s] = acc; c->mag[s] = mag;
    }
}

void ptxo_gemm_mxfp8_ref(const uint8_t* A, const uint8_t* sfA, const uint8_t* B,
                         const uint8_t* sfB, int64_t M, int64_t N, int64_t K,
                         const int64_t* rows, const int64_t* cols, int64_t n_samples, double* ref,
                         double* mag, int threads) {
    gemm_ctx c; memset(&c, 0, sizeof c);
    c.A = A; c.sfA = sfA; c.B = B; c.sfB = sfB;
    c.M = M; c.N = N; c.K = K; c.rows = rows; c.cols = cols; c.ref = ref; c.mag = mag;
    parallel_for((uint64_t)n_samples, threads, mxfp8_samples, &c);
}

/* ---- MX formats in the tcgen05 operand layout --------------------------------------------- */
/* Packing of 4- and 6-bit elements for kind::f8f6f4 / mxf8f6f4 operands in shared memory
 * (documented beside F8f6f4ElementType, src/tcgen05/descriptor.rs:306-315): groups of 16 elements
 * padded to 16 bytes. */
void ptxo_mx_pack(int format, const uint8_t* codes, uint8_t* packed, size_t n) {
    for (size_t g = 0; g < n / 16; ++g) {
        const uint8_t* c = codes + 16 * g;
        uint8_t* o = packed + 16 * g;
        memset(o, 0, 16);
        if (format == PTXO_E4M3 || format == PTXO_E5M2) {
            memcpy(o, c, 16);
        } else if (format == PTXO_E2M3 || format == PTXO_E3M2) {
            for (int i = 0; i < 16; ++i) {
                const uint32_t v = c[i] & 0x3Fu, bit = 6u * (uint32_t)i;
                o[bit / 8] |= (uint8_t)(v << (bit % 8));
                if (bit % 8 > 2) o[bit / 8 + 1] |= (uint8_t)(v >> (8 - bit % 8));
            }
        } else {
            for (int j = 0; j < 8; ++j)
                o[j] = (uint8_t)((c[2 * j] & 0xF) | ((c[2 * j + 1] & 0xF) << 4));
        }
    }
}

void ptxo_mx_unpack(int format, const uint8_t* packed, uint8_t* codes, size_t n) {
    for (size_t g = 0; g < n / 16; ++g) {
        const uint8_t* p = packed + 16 * g;
        uint8_t* c = codes + 16 * g;
        if (format == PTXO_E4M3 || format == PTXO_E5M2) {
            memcpy(c, p, 16);
        } else if (format == PTXO_E2M3 || format == PTXO_E3M2) {
            for (int i = 0; i < 16; ++i) {
                const uint32_t bit = 6u * (uint32_t)i;
                uint32_t v = (uint32_t)p[bit / 8] >> (bit % 8);
                if (bit % 8 > 2) v |= (uint32_t)p[bit / 8 + 1] << (8 - bit % 8);
                c[i] = (uint8_t)(v & 0x3Fu);
            }
        } else {
            for (int j = 0; j < 8; ++j) {
                c[2 * j] = p[j] & 0xF;
                c[2 * j + 1] = p[j] >> 4;
            }
        }
    }
}

void ptxo_cp_unpack(int format, const uint8_t* packed, uint8_t* containers, size_t n) {
    /* FP6: the 6-bit code in bits 5..0 of its container. FP4: the nibble in bits 5..2, i.e. at
     * the sign / exponent / mantissa positions of an E2M3 value with two zero mantissa bits
     * below (pinned on the B200). The other bits are zero. */
    ptxo_mx_unpack(format, packed, containers, n);
    if (format == PTXO_E2M1)
        for (size_t i = 0; i < n; ++i) containers[i] = (uint8_t)(containers[i] << 2);
}

static int mx_emax(int format) {
    switch (format) {
    case PTXO_E4M3: return 8;
    case PTXO_E5M2: return 15;
    case PTXO_E3M2: return 4;
    default: return 2;  /* E2M3, E2M1 */
    }
}

static float mx_decode(int format, uint8_t code) {
    switch (format) {
    case PTXO_E4M3: return ptxo_e4m3_to_f32(code);
    case PTXO_E5M2: return ptxo_e5m2_to_f32(code);
    case PTXO_E2M3: return ptxo_e2m3_to_f32(code);
    case PTXO_E3M2: return ptxo_e3m2_to_f32(code);
    default: return ptxo_e2m1_to_f32(code);
    }
}

typedef struct { const uint16_t* x; int64_t cols; int format; uint8_t *q, *sf; } mx_ctx;

static void mx_rows(void* p, uint64_t lo, uint64_t hi) {
    mx_ctx* c = (mx_ctx*)p;
    float buf[32];
    uint8_t codes[32];
    const int emax = mx_emax(c->format);
    for (uint64_t r = lo; r < hi; ++r) {
        const uint16_t* xr = c->x + r * c->cols;
        for (int64_t b = 0; b < c->cols / 32; ++b) {
            for (int i = 0; i < 32; ++i) buf[i] = ptxo_bf16_to_f32(xr[b * 32 + i]);
            const uint8_t u = ptxo_f32_to_ue8m0(block_amax(buf, 32), 0, 1);
            const uint8_t code = (u == 0xFF) ? 0xFF : (u > emax ? (uint8_t)(u - emax) : 0);
            const float inv = ue8m0_inverse(code);
            for (int i = 0; i < 32; ++i) codes[i] = ptxo_f32_to_narrow(c->format, buf[i] * inv, 0);
            c->sf[r * (c->cols / 32) + b] = code;
            ptxo_mx_pack(c->format, codes, c->q + r * c->cols + b * 32, 32);
        }
    }
}

void ptxo_quantize_mx(const uint16_t* x, int64_t rows, int64_t cols, int format, uint8_t* q,
                      uint8_t* sf, int threads) {
    mx_ctx c = {x, cols, format, q, sf};
    parallel_for((uint64_t)rows, threads, mx_rows, &c);
}

typedef struct {
    const uint8_t *A, *B, *sfA, *sfB;
    int fa, fb;
    int64_t K;
    const int64_t *rows, *cols;
    double *ref, *mag;
} mx_gemm_ctx;

static void mx_samples(void* p, uint64_t lo, uint64_t hi) {
    mx_gemm_ctx* c = (mx_gemm_ctx*)p;
    double la[256], lb[256];
    for (int i = 0; i < 256; ++i) {
        la[i] = mx_decode(c->fa, (uint8_t)i);
        lb[i] = mx_decode(c->fb, (uint8_t)i);
    }
    uint8_t* ca = (uint8_t*)malloc((size_t)c->K);
    uint8_t* cb = (uint8_t*)malloc((size_t)c->K);
    if (!ca || !cb) { free(ca); free(cb); return; }
    for (uint64_t s = lo; s < hi; ++s) {
        ptxo_mx_unpack(c->fa, c->A + c->rows[s] * c->K, ca, (size_t)c->K);
        ptxo_mx_unpack(c->fb, c->B + c->cols[s] * c->K, cb, (size_t)c->K);
        const uint8_t* sa = c->sfA + c->rows[s] * (c->K / 32);
        const uint8_t* sb = c->sfB + c->cols[s] * (c->K / 32);
        double acc = 0, mag = 0;
        for (int64_t k = 0; k < c->K; ++k) {
            const double t = la[ca[k]] * (double)ptxo_ue8m0_to_f32(sa[k >> 5]) * lb[cb[k]] *
                             (double)ptxo_ue8m0_to_f32(sb[k >> 5]);
            acc += t; mag += fabs(t);
        }
        c->ref[s] = acc; c->mag[s] = mag;
    }
    free(ca); free(cb);
}

void ptxo_gemm_mx_ref(const uint8_t* A, int fa, const uint8_t* sfA, const uint8_t* B, int fb,
                      const uint8_t* sfB, int64_t M, int64_t N, int64_t K, const int64_t* rows,
                      const int64_t* cols, int64_t n_samples, double* ref, double* mag,
                      int threads) {
    (void)M; (void)N;
    mx_gemm_ctx c = {A, B, sfA, sfB, fa, fb, K, rows, cols, ref, mag};
    parallel_for((uint64_t)n_samples, threads, mx_samples, &c);
}

/* 2:4 pruning (one row per job step): magnitude = code & 0x7F (E4M3 codes order like their
 * magnitudes; the NaN code 0x7F sorts highest), ties to the lower index. */
typedef struct { const uint8_t* codes; int64_t cols; uint8_t *vals, *meta; } prune_ctx;

static void prune_rows(void* p, uint64_t lo, uint64_t hi) {
    prune_ctx* c = (prune_ctx*)p;
    for (uint64_t r = lo; r < hi; ++r) {
        const uint8_t* x = c->codes + r * c->cols;
        uint8_t* v = c->vals + r * (c->cols / 2);
        uint8_t* m = c->meta + r * (c->cols / 8);
        for (int64_t g = 0; g < c->cols / 4; ++g) {
            const uint8_t* q = x + 4 * g;
            int best = 0;
            for (int i = 1; i < 4; ++i) if ((q[i] & 0x7F) > (q[best] & 0x7F)) best = i;
            int second = -1;
            for (int i = 0; i < 4; ++i) {
                if (i == best) continue;
                if (second < 0 || (q[i] & 0x7F) > (q[second] & 0x7F)) second = i;
            }
            int i0 = best < second ? best : second, i1 = best < second ? second : best;
            v[2 * g] = q[i0];
            v[2 * g + 1] = q[i1];
            uint8_t nib = (uint8_t)(i0 | (i1 << 2));
            if (g % 2 == 0) m[g / 2] = nib;
            else m[g / 2] |= (uint8_t)(nib << 4);
        }
    }
}

void ptxo_prune_24(const uint8_t* codes, int64_t rows, int64_t cols, uint8_t* vals, uint8_t* meta,
                   int threads) {
    prune_ctx c = {codes, cols, vals, meta};
    parallel_for((uint64_t)rows, threads, prune_rows, &c);
}

typedef struct { const uint8_t *vals, *meta; int64_t cols; uint8_t* codes; } dec24_ctx;

static void decompress_rows(void* p, uint64_t lo, uint64_t hi) {
    dec24_ctx* c = (dec24_ctx*)p;
    for (uint64_t r = lo; r < hi; ++r) {
        uint8_t* x = c->codes + r * c->cols;
        const uint8_t* v = c->vals + r * (c->cols / 2);
        const uint8_t* m = c->meta + r * (c->cols / 8);
        memset(x, 0, (size_t)c->cols);
        for (int64_t g = 0; g < c->cols / 4; ++g) {
            uint8_t nib = (uint8_t)((m[g / 2] >> (4 * (g % 2))) & 0xF);
            x[4 * g + (nib & 3)] = v[2 * g];
            x[4 * g + (nib >> 2)] = v[2 * g + 1];
        }
    }
}

void ptxo_decompress_24(const uint8_t* vals, const uint8_t* meta, int64_t rows, int64_t cols,
                        uint8_t* codes, int threads) {
    dec24_ctx c = {vals, meta, cols, codes};
    parallel_for((uint64_t)rows, threads, decompress_rows, &c);
}

static void mxfp8_sparse_samples(void* p, uint64_t lo, uint64_t hi) {
    gemm_ctx* c = (gemm_ctx*)p;
    double lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = ptxo_e4m3_to_f32((uint8_t)i);
    const int64_t K = c->K;
    for (uint64_t s = lo; s < hi; ++s) {
        /* c->A holds vals, c->W holds meta */
        const uint8_t* v = c->A + c->rows[s] * (K / 2);
        const uint8_t* m = c->W + c->rows[s] * (K / 8);
        const uint8_t* sa = c->sfA + c->rows[s] * (K / 64);
        const uint8_t* b = c->B + c->cols[s] * K;
        const uint8_t* sb = c->sfB + c->cols[s] * (K / 64);
        double acc = 0, mag = 0;
        for (int64_t g = 0; g < K / 4; ++g) {
            uint8_t nib = (uint8_t)((m[g / 2] >> (4 * (g % 2))) & 0xF);
            double scale = (double)ptxo_ue8m0_to_f32(sa[(4 * g) >> 6]) *
                           (double)ptxo_ue8m0_to_f32(sb[(4 * g) >> 6]);
            for (int h = 0; h < 2; ++h) {
                int64_t k = 4 * g + (h ? (nib >> 2) : (nib & 3));
                double t = lut[v[2 * g + h]] * lut[b[k]] * scale;
                acc += t; mag += fabs(t);
            }
        }
        c->ref[s] = acc; c->mag[s] = mag;
    }
}

void ptxo_gemm_mxfp8_sparse_ref(const uint8_t* vals, const uint8_t* meta, const uint8_t* sfA,
                                const uint8_t* B, const uint8_t* sfB, int64_t M, int64_t N,
                                int64_t K, const int64_t* rows, const int64_t* cols,
                                int64_t n_samples, double* ref, double* mag, int threads) {
    gemm_ctx c; memset(&c, 0, sizeof c);
    c.A = vals; c.W = meta; c.sfA = sfA; c.B = B; c.sfB = sfB;
    c.M = M; c.N = N; c.K = K; c.rows = rows; c.cols = cols; c.ref = ref; c.mag = mag;
    parallel_for((uint64_t)n_samples, threads, mxfp8_sparse_samples, &c);
}

static void decode_samples(void* p, uint64_t lo, uint64_t hi) {
    gemm_ctx* c = (gemm_ctx*)p;
    int64_t K = c->K;
    float* xf = (float*)malloc(sizeof(float) * K);
    double* xv = (double*)malloc(sizeof(double) * K);
    uint8_t q32[32];
    int64_t cur_row = -1;
    for (uint64_t s = lo; s < hi; ++s) {
        int64_t i = c->rows[s];
        if (i != cur_row) {
            for (int64_t k = 0; k < K; ++k) xf[k] = ptxo_bf16_to_f32(c->x[i * K + k]);
            for (int64_t b = 0; b < K / 32; ++b) {
                uint8_t code = ptxo_mxfp8_block(xf + b * 32, q32);
                double scale = (double)ptxo_ue8m0_to_f32(code);
                for (int j = 0; j < 32; ++j) xv[b * 32 + j] = (double)ptxo_e4m3_to_f32(q32[j]) * scale;
            }
            cur_row = i;
        }
        const uint8_t* w = c->W + c->cols[s] * (K / 2);
        const uint8_t* sw = c->sfW + c->cols[s] * (K / 16);
        double acc = 0, mag = 0;
        for (int64_t k = 0; k < K; ++k) {
            double t = xv[k] * nvfp4_elem(w, sw, k);
            acc += t; mag += fabs(t);
        }
        c->ref[s] = acc * (double)c->gw; c->mag[s] = mag * fabs((double)c->gw);
    }
    free(xf); free(xv);
}

void ptxo_gemm_decode_ref(const uint16_t* x, const uint8_t* W, const uint8_t* sfW, float gw,
                          int64_t M, int64_t N, int64_t K, const int64_t* rows,
                          const int64_t* cols, int64_t n_samples, double* ref, double* mag,
                          int threads) {
    gemm_ctx c; memset(&c, 0, sizeof c);
    c.x = x; c.W = W; c.sfW = sfW; c.gw = gw; c.M = M; c.N = N; c.K = K;
    c.rows = rows; c.cols = cols; c.ref = ref; c.mag = mag;
    parallel_for((uint64_t)n_samples, threads, decode_samples, &c);
}

/* Cache-blocked C = A * B^T in f32 for the timed CPU baseline. Rows of C are split across
 * threads; within a thread, blocks of 64 columns x 256 K keep B's panel in cache and 4 rows of A
 * are processed per pass. */
typedef struct { const float *A, *B; float* C; int64_t M, N, K; } sg_ctx;

static void sgemm_rows(void* p, uint64_t lo, uint64_t hi) {
    sg_ctx* c = (sg_ctx*)p;
    const int64_t NB = 64, KB = 256;
    for (uint64_t i = lo; i < hi; ++i)
        for (int64_t j = 0; j < c->N; ++j) c->C[i * c->N + j] = 0.0f;
    for (int64_t j0 = 0; j0 < c->N; j0 += NB) {
        int64_t j1 = j0 + NB < c->N ? j0 + NB : c->N;
        for (int64_t k0 = 0; k0 < c->K; k0 += KB) {
            int64_t k1 = k0 + KB < c->K ? k0 + KB : c->K;
            for (uint64_t i = lo; i < hi; ++i) {
                const float* a = c->A + i * c->K;
                for (int64_t j = j0; j < j1; ++j) {
                    const float* b = c->B + j * c->K;
                    float acc = 0.0f;
                    for (int64_t k = k0; k < k1; ++k) acc += a[k] * b[k];
                    c->C[i * c->N + j] += acc;
                }
            }
        }
    }
}

void ptxo_sgemm_nt(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                   int threads) {
    sg_ctx c = {A, B, C, M, N, K};
    parallel_for((uint64_t)M, threads, sgemm_rows, &c);
}

/* ------------------------------------------------------------------------------------------ */
/* tcgen05 descriptors (src/tcgen05/descriptor.rs)                                            */
/* ------------------------------------------------------------------------------------------ */

/* encode_n: N a multiple of 8 in [8, 256], at bits 17..23 as N >> 3 (descriptor.rs:450-457). */
static int enc_n(uint32_t n, uint32_t* f) {
    if (n % 8 || n < 8 || n > 256) return -1;
    *f = (n >> 3) << 17; return 0;
}
/* encode_m: M a multiple of 16 in [16, 256], at bits 24..29 as M >> 4 (descriptor.rs:460-467). */
static int enc_m(uint32_t m, uint32_t* f) {
    if (m % 16 || m < 16 || m > 256) return -1;
    *f = (m >> 4) << 24; return 0;
}
/* encode_m_block_scaled: M 128 or 256, at bits 27..29 as M >> 7 (descriptor.rs:470-476). */
static int enc_m_bs(uint32_t m, uint32_t* f) {
    if (m != 128 && m != 256) return -1;
    *f = (m >> 7) << 27; return 0;
}

/* F16 / F8f6f4: d << 4 | a << 7 | b << 10 | N | M (descriptor.rs:520-527, :555-564). */
int ptxo_idesc_f16(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out) {
    uint32_t fm, fn;
    if (enc_m(m, &fm) || enc_n(n, &fn)) return -1;
    *out = ((uint32_t)d << 4) | ((uint32_t)a << 7) | ((uint32_t)b << 10) | fn | fm;
    return 0;
}
int ptxo_idesc_f8f6f4(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out) {
    return ptxo_idesc_f16(a, b, d, m, n, out);
}
/* Tf32: D f32 (1 << 4), A and B tf32 (2 << 7, 2 << 10) (descriptor.rs:537-541). */
int ptxo_idesc_tf32(uint32_t m, uint32_t n, uint32_t* out) {
    return ptxo_idesc_f16(2, 2, 1, m, n, out);
}
/* I8: D s32 (2 << 4) (descriptor.rs:575-578). */
int ptxo_idesc_i8(int a, int b, uint32_t m, uint32_t n, uint32_t* out) {
    return ptxo_idesc_f16(a, b, 2, m, n, out);
}
/* Mxf8f6f4: a << 7 | b << 10 | ue8m0 scales (1 << 23) | N | M>>7<<27 (descriptor.rs:601-611). */
int ptxo_idesc_mxf8f6f4(int a, int b, uint32_t m, uint32_t n, uint32_t* out) {
    uint32_t fm, fn;
    if (enc_m_bs(m, &fm) || enc_n(n, &fn)) return -1;
    *out = ((uint32_t)a << 7) | ((uint32_t)b << 10) | (1u << 23) | fn | fm;
    return 0;
}
/* Mxf4: e2m1 A and B (1 << 7, 1 << 10), ue8m0 scales (1 << 23) (descriptor.rs:625-628). */
int ptxo_idesc_mxf4(uint32_t m, uint32_t n, uint32_t* out) {
    return ptxo_idesc_mxf8f6f4(1, 1, m, n, out);
}
/* Mxf4nvf4: e2m1 A and B, scale type << 23 (ue4m3 0, ue8m0 1, ue5m3 2) (descriptor.rs:644-653). */
int ptxo_idesc_mxf4nvf4(int scale_type, uint32_t m, uint32_t n, uint32_t* out) {
    uint32_t fm, fn;
    if (scale_type < 0 || scale_type > 2) return -1;
    if (enc_m_bs(m, &fm) || enc_n(n, &fn)) return -1;
    *out = (1u << 7) | (1u << 10) | ((uint32_t)scale_type << 23) | fn | fm;
    return 0;
}
/* with_field (descriptor.rs:494-498): the value must fit in the field. */
int ptxo_idesc_with_field(uint32_t desc, uint32_t shift, uint32_t width, uint32_t value,
                          uint32_t* out) {
    if (width == 0 || width > 31 || shift + width > 32) return -1;
    if (value >= (1u << width)) return -1;
    uint32_t mask = ((1u << width) - 1) << shift;
    *out = (desc & ~mask) | (value << shift);
    return 0;
}

/* encode_smem_offset: multiple of 16, at most 0x3FFFF, stored >> 4 (descriptor.rs:100-108). */
static int enc_off(uint32_t bytes, uint64_t* f) {
    if (bytes % 16 || bytes > 0x3FFFF) return -1;
    *f = bytes >> 4; return 0;
}

/* from_shared_address (descriptor.rs:152-162): start bits 4..17 at 0, LBO >> 4 at 16, SBO >> 4
 * at 32, the constant 0b001 at 46, swizzle code at 61 (Swizzle codes 0, 1, 2, 4, 6). */
int ptxo_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo, int swizzle, uint64_t* out) {
    uint64_t l, s;
    if (!(swizzle == 0 || swizzle == 1 || swizzle == 2 || swizzle == 4 || swizzle == 6)) return -1;
    if (enc_off(lbo, &l) || enc_off(sbo, &s)) return -1;
    uint64_t st = (uint64_t)((start & 0x3FFFFu) >> 4);
    *out = st | (l << 16) | (s << 32) | (1ull << 46) | ((uint64_t)swizzle << 61);
    return 0;
}
/* with_base_offset (descriptor.rs:176-183): 3 bits at 49; not with the absolute LBO mode. */
int ptxo_smem_desc_with_base_offset(uint64_t desc, uint32_t base_offset, uint64_t* out) {
    if (base_offset >= 8) return -1;
    if (base_offset != 0 && (desc & (1ull << 52))) return -1;
    *out = (desc & ~(7ull << 49)) | ((uint64_t)base_offset << 49);
    return 0;
}
/* add_start_bytes (descriptor.rs:231-237): a 64-bit add of bytes >> 4. */
int ptxo_smem_desc_add_start_bytes(uint64_t desc, uint32_t bytes, uint64_t* out) {
    if (bytes % 16) return -1;
    *out = desc + (uint64_t)(bytes >> 4);
    return 0;
}

/* ZeroColumnMask::new (descriptor.rs:870-883): enable bit 39, zeroed-1 at 40, used-1 at 48. */
int ptxo_zero_mask_new(uint32_t zeroed, uint32_t used, uint64_t* out) {
    if (zeroed < 1 || zeroed > 256 || used < 1 || used > 256) return -1;
    *out = (1ull << 39) | ((uint64_t)(zeroed - 1) << 40) | ((uint64_t)(used - 1) << 48);
    return 0;
}
/* with_sub_mask_start (descriptor.rs:891-909): count at 8*sub, first span at 32+sub. */
int ptxo_zero_mask_with_sub_mask_start(uint64_t mask, uint32_t sub, int first_span,
                                       uint32_t start_count, uint64_t* out) {
    if (sub >= 4 || start_count >= 256 || (first_span != 0 && first_span != 1)) return -1;
    uint32_t cs = 8 * sub, ss = 32 + sub;
    *out = (mask & ~((0xFFull << cs) | (1ull << ss))) | ((uint64_t)start_count << cs) |
           ((uint64_t)first_span << ss);
    return 0;
}
/* with_column_shift (descriptor.rs:917-921): 6 bits at 56, at most 32. */
int ptxo_zero_mask_with_column_shift(uint64_t mask, uint32_t shift, uint64_t* out) {
    if (shift > 32) return -1;
    *out = (mask & ~(0x3Full << 56)) | ((uint64_t)shift << 56);
    return 0;
}

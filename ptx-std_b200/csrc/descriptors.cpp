// C ABI of the tcgen05 descriptor builders (ptx-std src/tcgen05/descriptor.rs). Pure integer
// host functions over the same constexpr encoders the kernels use; every case where the
// reference's builder asserts returns PTXSTD_EINVAL instead.
#include "tcgen05.cuh"

namespace t5 = ptxstd::tcgen05;

extern "C" {

int ptxstd_idesc_f16(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out) {
    if (!out || a < 0 || a > 1 || b < 0 || b > 1 || d < 0 || d > 1) return PTXSTD_EINVAL;
    uint32_t v = 0;
    if (!t5::idesc_dense(a, b, d, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_idesc_tf32(uint32_t m, uint32_t n, uint32_t* out) {
    uint32_t v = 0;
    if (!out || !t5::idesc_dense(2, 2, 1, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

static bool f8f6f4_type(int t) { return t == 0 || t == 1 || t == 3 || t == 4 || t == 5; }

int ptxstd_idesc_f8f6f4(int a, int b, int d, uint32_t m, uint32_t n, uint32_t* out) {
    if (!out || !f8f6f4_type(a) || !f8f6f4_type(b) || d < 0 || d > 1) return PTXSTD_EINVAL;
    uint32_t v = 0;
    if (!t5::idesc_dense(a, b, d, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_idesc_i8(int a, int b, uint32_t m, uint32_t n, uint32_t* out) {
    if (!out || a < 0 || a > 1 || b < 0 || b > 1) return PTXSTD_EINVAL;
    uint32_t v = 0;
    if (!t5::idesc_dense(a, b, 2, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_idesc_mxf8f6f4(int a, int b, uint32_t m, uint32_t n, uint32_t* out) {
    if (!out || !f8f6f4_type(a) || !f8f6f4_type(b)) return PTXSTD_EINVAL;
    uint32_t v = 0;
    if (!t5::idesc_mxf8f6f4(a, b, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_idesc_mxf4(uint32_t m, uint32_t n, uint32_t* out) {
    // Mxf4: A and B e2m1 encoded as 1 in this kind's layout (descriptor.rs:625-628).
    uint32_t v = 0;
    if (!out || !t5::idesc_mxf8f6f4(1, 1, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_idesc_mxf4nvf4(int scale_type, uint32_t m, uint32_t n, uint32_t* out) {
    uint32_t v = 0;
    if (!out || scale_type < 0 || !t5::idesc_mxf4nvf4(scale_type, m, n, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_idesc_set(uint32_t desc, int kind, int field, uint32_t value, uint32_t* out) {
    if (!out || kind < 0 || kind > 6 || field < 0 || field > 10) return PTXSTD_EINVAL;
    uint32_t shift = 0, width = 0;
    if (!t5::idesc_field_of(static_cast<t5::MmaKind>(kind), static_cast<t5::IdescField>(field),
                            shift, width))
        return PTXSTD_EINVAL;
    uint32_t v = 0;
    if (!t5::idesc_with_field(desc, shift, width, value, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_smem_desc(uint32_t start, uint32_t lbo, uint32_t sbo, int swizzle, uint64_t* out) {
    uint64_t v = 0;
    if (!out || swizzle < 0 || !t5::smem_desc(start, lbo, sbo, swizzle, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_smem_desc_with_base_offset(uint64_t desc, uint32_t base_offset, uint64_t* out) {
    uint64_t v = 0;
    if (!out || !t5::smem_desc_with_base_offset(desc, base_offset, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_smem_desc_add_start_bytes(uint64_t desc, uint32_t bytes, uint64_t* out) {
    uint64_t v = 0;
    if (!out || !t5::smem_desc_add_start_bytes(desc, bytes, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_zero_mask_new(uint32_t zeroed, uint32_t used, uint64_t* out) {
    uint64_t v = 0;
    if (!out || !t5::zero_mask_new(zeroed, used, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_zero_mask_with_sub_mask_start(uint64_t mask, uint32_t sub_mask, int first_span,
                                         uint32_t start_count, uint64_t* out) {
    uint64_t v = 0;
    if (!out || first_span < 0 ||
        !t5::zero_mask_with_sub_mask_start(mask, sub_mask, first_span, start_count, v))
        return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

int ptxstd_zero_mask_with_column_shift(uint64_t mask, uint32_t shift, uint64_t* out) {
    uint64_t v = 0;
    if (!out || !t5::zero_mask_with_column_shift(mask, shift, v)) return PTXSTD_EINVAL;
    *out = v;
    return PTXSTD_OK;
}

}  // extern "C"

/* A plain C99 consumer of the C ABI: it compiles against include/ptxstd.h alone and links
 * libptxstd.so, as a binding in another language would. It makes only calls that need no GPU
 * (status strings, version, descriptor encoders with their known answers, argument checks) and
 * prints "ok" or the first failing check. */
#include <stdio.h>
#include <string.h>

#include "ptxstd.h"

#define CHECK(c)                                                  \
    do {                                                          \
        if (!(c)) {                                               \
            printf("fail at line %d: %s\n", __LINE__, #c);        \
            return 1;                                             \
        }                                                         \
    } while (0)

int main(void) {
    uint64_t d = 0;
    uint32_t i = 0;
    uint16_t* y = NULL;
    CHECK(ptxstd_version() > 0);
    CHECK(strlen(ptxstd_status_string(PTXSTD_EINVAL)) > 0);
    /* SmemDescriptor: K-major, 128-byte swizzle, SBO 1024 (descriptor.rs:152-162) */
    CHECK(ptxstd_smem_desc(0x1230, 16, 1024, 2, &d) == PTXSTD_OK);
    CHECK(d == 0x4000404000010123ull);
    CHECK(ptxstd_smem_desc(0x1230, 16, 1024, 3, &d) == PTXSTD_EINVAL); /* no swizzle mode 3 */
    /* InstrDescriptor::<Mxf4nvf4>::new(Ue4m3, 128, 64) */
    CHECK(ptxstd_idesc_mxf4nvf4(0, 128, 64, &i) == PTXSTD_OK);
    CHECK(i == 0x08100480u);
    /* argument checks answer before any CUDA call */
    CHECK(ptxstd_quantize_mx(NULL, 128, 128, PTXSTD_MX_E2M3, NULL, NULL, 0, NULL) ==
          PTXSTD_EINVAL);
    CHECK(ptxstd_gemm_mx(NULL, 2, NULL, NULL, PTXSTD_MX_E4M3, NULL, NULL, 256, 256, 128, NULL) ==
          PTXSTD_EINVAL);
    CHECK(ptxstd_gemm_decode(NULL, NULL, NULL, 1.0f, NULL, 17, 128, 256, NULL, 0, NULL) ==
          PTXSTD_EINVAL);
    CHECK(ptxstd_dist_free(NULL) == PTXSTD_OK);
    CHECK(ptxstd_dist_decode_p2p_init(NULL, 1024, &y) == PTXSTD_EINVAL);
    printf("ok\n");
    return 0;
}

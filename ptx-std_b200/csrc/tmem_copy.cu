// The decompressing shared-memory -> Tensor Memory copy, exposed for parity: the reference's
// copy::<S128x256b, B6x16P32 | B4x16P64> (src/tcgen05/copy.rs:32-46, :76-116), which turns FP6
// (E2M3 / E3M2) or FP4 (E2M1) operands in the packed K = 32 layout (16 elements + padding per 16
// bytes, src/tcgen05/descriptor.rs:306-315) into the 8-bit containers that an MMA reads as matrix
// A from Tensor Memory.
//
// One CTA of four warps per 4 KiB tile (128 rows x 32 bytes): the threads store row r's two
// 16-byte groups into the canonical unswizzled K-major layout (8-row x 16-byte core matrices,
// 128 bytes apart along the rows, the second group of every row 2 KiB further), thread 0 issues
// the copy into 8 TMEM columns and commits it to an mbarrier, and each warp reads its lane
// quarter back with tcgen05.ld.32x32b.x8 and writes row r's 32 containers. The shared buffer is
// 32 KiB so that the copy stays inside it under either assignment of the two strides.
#include "common.cuh"
#include "tcgen05.cuh"

namespace {

namespace t5 = ptxstd::tcgen05;
using ptxstd::mbar_wait;

constexpr uint32_t kRows = 128, kRowBytes = 32, kTileBytes = kRows * kRowBytes;
constexpr uint32_t kGroupStride = 128;   // SBO: next 8-row core matrix
constexpr uint32_t kChunkStride = 2048;  // LBO: second 16-byte group of the rows
constexpr uint32_t kTmemCols = 32;       // the allocation minimum; the copy fills 8

struct alignas(1024) Smem {
    uint8_t buf[32768];
    uint64_t bar;
    uint32_t tmem;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;

template <bool FP6>
__global__ void __launch_bounds__(128) cp_unpack_kernel(const uint8_t* __restrict__ in,
                                                        uint8_t* __restrict__ out,
                                                        uint32_t n_tiles, uint32_t* err) {
    extern __shared__ uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~static_cast<uintptr_t>(1023));
    const uint32_t r = threadIdx.x, warp = r / 32;
    if (r == 0) {
        ptxstd::mbar_init(&s.bar, 1);
        ptxstd::fence_mbarrier_init();
    }
    if (warp == 0) {
        t5::tmem_alloc(&s.tmem, kTmemCols);
        t5::tmem_relinquish();
    }
    t5::fence_before_thread_sync();
    __syncthreads();
    t5::fence_after_thread_sync();
    const uint32_t tmem = s.tmem;
    uint32_t phase = 0;
    for (uint32_t t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        const uint4* src =
            reinterpret_cast<const uint4*>(in + static_cast<size_t>(t) * kTileBytes + r * kRowBytes);
        uint8_t* row = s.buf + (r % 8) * 16 + (r / 8) * kGroupStride;
        *reinterpret_cast<uint4*>(row) = src[0];
        *reinterpret_cast<uint4*>(row + kChunkStride) = src[1];
        ptxstd::fence_proxy_async_smem();
        t5::fence_before_thread_sync();
        __syncthreads();
        t5::fence_after_thread_sync();
        if (r == 0) {
            const uint64_t desc =
                t5::smem_desc_nosw(ptxstd::smem_u32(s.buf), kChunkStride, kGroupStride);
            if constexpr (FP6)
                t5::cp_128x256b_b6x16_p32(tmem, desc);
            else
                t5::cp_128x256b_b4x16_p64(tmem, desc);
            t5::commit(&s.bar);
        }
        const bool ok = mbar_wait(&s.bar, phase);
        phase ^= 1u;
        if (__syncthreads_or(!ok)) {
            if (r == 0) ptxstd::record_error(err, PTXSTD_ETIMEOUT, 0x5100u);
            break;
        }
        t5::fence_after_thread_sync();
        uint32_t v[8];
        t5::ld_32x32b_x8(tmem + ((32u * warp) << 16), v);
        t5::wait_ld();
        uint4* dst = reinterpret_cast<uint4*>(out + static_cast<size_t>(t) * kTileBytes +
                                              r * kRowBytes);
        dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
        dst[1] = make_uint4(v[4], v[5], v[6], v[7]);
        // the next tile rewrites the shared buffer and the TMEM columns
        t5::fence_before_thread_sync();
        __syncthreads();
        t5::fence_after_thread_sync();
    }
    if (warp == 0) t5::tmem_dealloc(tmem, kTmemCols);
}

}  // namespace

extern "C" int ptxstd_tcgen05_cp_unpack(const uint8_t* d_packed, uint8_t* d_out, int64_t n_tiles,
                                        int elem_type, ptxstd_stream stream) {
    if (n_tiles <= 0 || n_tiles >= (1ll << 31) || !d_packed || !d_out ||
        !ptxstd::aligned16(d_packed) || !ptxstd::aligned16(d_out))
        return PTXSTD_EINVAL;
    if (elem_type != 3 && elem_type != 4 && elem_type != 5) return PTXSTD_EINVAL;
    const bool fp6 = elem_type != 5;
    const void* fn = fp6 ? reinterpret_cast<const void*>(cp_unpack_kernel<true>)
                         : reinterpret_cast<const void*>(cp_unpack_kernel<false>);
    int st = ptxstd::set_max_dynamic_smem(fn, static_cast<int>(kSmemBytes));
    if (st) return st;
    uint32_t* err = ptxstd::device_error_word();
    if (!err) return PTXSTD_ECUDA;
    const int sms = ptxstd::sm_count();
    const uint32_t grid = static_cast<uint32_t>(n_tiles < sms ? n_tiles : sms);
    auto s = static_cast<cudaStream_t>(stream);
    if (fp6)
        cp_unpack_kernel<true><<<grid, 128, kSmemBytes, s>>>(d_packed, d_out,
                                                             static_cast<uint32_t>(n_tiles), err);
    else
        cp_unpack_kernel<false><<<grid, 128, kSmemBytes, s>>>(d_packed, d_out,
                                                              static_cast<uint32_t>(n_tiles), err);
    return ptxstd::launch_status();
}

// Device-side foundation shared by every kernel of libptxstd: status/error word, bounded mbarrier
// waits, fences, elect, TMA copies. Each wrapper is one PTX instruction (or a short bounded loop
// around one) with the semantics of the ptx-std API named beside it.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "../../include/ptxstd.h"

namespace ptxstd {

// ---- error word ----------------------------------------------------------------------------
// Each device holds one error word pair {status, detail}. Kernels record the first failure with
// a CAS so that the earliest cause is kept; the host reads it with ptxstd_last_device_error.
__device__ __forceinline__ void record_error(uint32_t* err, uint32_t status, uint32_t detail) {
    if (err != nullptr && atomicCAS(err, 0u, status) == 0u) atomicExch(err + 1, detail);
}

// Host side: the address of this device's error word (set up once per device).
uint32_t* device_error_word();

// ---- time -----------------------------------------------------------------------------------
// %globaltimer in ns (ptx-std src/time.rs:40).
__device__ __forceinline__ uint64_t global_timer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every device-side wait gives up after this long and reports PTXSTD_ETIMEOUT.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// ---- addresses --------------------------------------------------------------------------------
// memory::to_shared_address (src/memory.rs:482): generic -> .shared::cta address.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- warp collectives ---------------------------------------------------------------------------
// warp_collectives::elect (src/warp_collectives.rs:900): true on exactly one lane of the warp.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred;
    asm volatile(
        "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(pred));
    return pred != 0;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t warp_id() {
    return __shfl_sync(0xffffffffu, threadIdx.x >> 5, 0);
}

// ---- mbarrier (src/mbarrier.rs) --------------------------------------------------------------
// MBarrier::init (:311).
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}
// MBarrier::fence_init (:345): makes the initialisation visible to the async proxy / cluster.
__device__ __forceinline__ void fence_mbarrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// MBarrier::arrive_expect_tx (:533).
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// MBarrier::arrive.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// MBarrier::try_wait (:928) on a phase parity.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// The reference's MBarrier::wait spins forever (:1011-1016); this one is bounded by
// kWaitLimitNs on %globaltimer and returns false when it gives up (try_wait_timed, :965).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity)) return true;
    const uint64_t t0 = global_timer();
    while (!mbar_try_wait(a, parity)) {
        if (global_timer() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// The same wait with acquire at cluster scope, for data that a thread of another CTA of the
// cluster wrote before its remote (release.cluster) arrive on `bar`.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait_cluster(a, parity)) return true;  // the timer only once it has to wait
    const uint64_t t0 = global_timer();
    while (!mbar_try_wait_cluster(a, parity)) {
        if (global_timer() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// ---- launch control and register allocation (src/launch.rs) ----------------------------------
// try_cancel_launch::<CancelDelivery::Block> (:154-176): asks to cancel a cluster of this grid
// that has not started yet. The 16-byte response is written to `resp` (this CTA's smem, 16-byte
// aligned) through the async proxy and completes a 16-byte transaction on `bar`, which must
// expect it. After a response that cancelled nothing, no further request may be issued.
__device__ __forceinline__ void clc_try_cancel(void* resp, uint64_t* bar) {
    asm volatile(
        "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 "
        "[%0], [%1];" ::"r"(smem_u32(resp)),
        "r"(smem_u32(bar))
        : "memory");
}
// CancelResponse::first_cta_id (:86-106): x index of the first CTA of the cancelled cluster, or
// -1 when the request cancelled nothing.
__device__ __forceinline__ int32_t clc_first_ctaid_x(const void* resp) {
    uint32_t ok, x;
    asm volatile(
        "{\n\t.reg .b128 v;\n\t.reg .pred p;\n\tld.shared.b128 v, [%2];\n\t"
        "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, v;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t"
        "clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, v;\n\t}"
        : "=r"(ok), "=r"(x)
        : "r"(smem_u32(resp))
        : "memory");
    return ok ? static_cast<int32_t>(x) : -1;
}
// increase_max_registers / decrease_max_registers (:204, :240): every warp of a warpgroup
// executes the same one; N is a multiple of 8 in 24..256. The kernel must be launched with a
// known register count (__launch_bounds__ with a minimum of one block).
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
    static_assert(N % 8 == 0 && N >= 24 && N <= 256, "register count");
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
    static_assert(N % 8 == 0 && N >= 24 && N <= 256, "register count");
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---- clusters (src/cluster.rs, src/globals.rs) -----------------------------------------------
// 32-bit store to a .shared::cluster address (a variable of any CTA of the cluster, via mapa).
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// block_rank_in_cluster (globals.rs:283).
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// map_to_cta (cluster.rs:117): this CTA's .shared::cta address -> the same variable in CTA `rank`
// of the cluster, as a .shared::cluster address.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// cluster::barrier_sync (cluster.rs:91): every thread of every CTA of the cluster.
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}
// Remote arrive on an mbarrier of another CTA of the cluster (MBarrier::arrive on a
// map_to_cta_rank barrier, mbarrier.rs:698).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// tma_load_tile_to_cluster::<2, CtaGroup::Two> without multicast (src/tma/tensor.rs:441-480): the
// tile lands in this CTA's smem and completes on an mbarrier that may live in the peer CTA of the
// pair (`bar` is a .shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar,
                                                 int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::"
        "bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// ---- fences (src/fence.rs) -------------------------------------------------------------------
// fence_proxy::<AsyncSharedCta> (:107): generic-proxy smem writes -> async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Release/acquire fences (the lighter alternative fence.rs:33-40 points to beside fence_seq_cst):
// order this thread's earlier accesses before its later ones for threads of the GPU / system,
// without joining the total order of fence.sc.
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// ---- TMA (src/tma/tensor.rs) -----------------------------------------------------------------
// tma_load_tile::<2> (:214-236): 2-D tile global -> this CTA's smem, completing on `bar`.
// Coordinates are in elements, innermost first. No multicast anywhere in this library.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int32_t c0, int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// bulk_load (src/tma/bulk.rs:60): `bytes` (a multiple of 16, both addresses 16-byte aligned)
// global -> this CTA's smem, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// L2 eviction policies for loads of data read exactly once (a weight stream): evict-first keeps
// the lines that are read again (partial sums, operand images) in L2 while the stream passes
// through. The reference applies `.L2::cache_hint` policies to its atomics (src/atomic.rs:45-46);
// its TMA wrappers have no hint form.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int32_t c0, int32_t c1, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void bulk_load_hint(void* dst, const void* src, uint32_t bytes,
                                               uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}
// tma_store_tile::<2> (:746): smem (a .shared::cta address) -> global, tracked by the bulk
// async-group. Stores never start at a negative coordinate here.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t c0,
                                             int32_t c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(src), "r"(c0), "r"(c1)
        : "memory");
}
// bulk_commit_group / bulk_wait_group::<N> read variant (src/tma/mod.rs:204, :220).
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// prefetch_tensormap (src/tma/mod.rs:239).
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 16-byte store to a .shared::cta address.
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

}  // namespace ptxstd

// ---- host-side helpers ----------------------------------------------------------------------
namespace ptxstd {
// Maps a CUDA error to a status, remembering nothing (callers check cudaGetLastError()).
inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? PTXSTD_OK : PTXSTD_ECUDA; }
// Launch-side check of the last launch.
inline int launch_status() { return cuda_status(cudaGetLastError()); }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
// Streaming-multiprocessor count of the current device (cached per device).
int sm_count();
// Raises a kernel's dynamic shared memory limit once per device; returns a ptxstd_status.
int set_max_dynamic_smem(const void* kernel, int bytes);
}  // namespace ptxstd

// Multi-GPU layer: one process (or thread) per GPU, an NCCL communicator per rank, weights sharded
// along N.
//
//   - ptxstd_gemm_nvfp4_sharded: B (and its scales) split along N into world contiguous blocks;
//     each rank computes its C columns. No communication (the path partitions).
//   - ptxstd_gemm_decode_sharded: W split along N; each rank runs the decode GEMM on its shard,
//     writing its [M, N/world] output block into its slot of a rank-major gather buffer, NCCL
//     all-gathers that buffer in place over NVLink, and a small kernel permutes the rank-major
//     blocks [world][M][N/world] into row-major y [M, N].
//   - ptxstd_gemm_decode_sharded_p2p: the same product with the gather fused into the GEMM: the
//     epilogue that finalises an output block stores it straight into every rank's y over NVLink
//     (CUDA IPC peer mappings of a buffer each rank allocates once), with the counters and bounded
//     waits of decode_out.h in place of a collective.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2; the copy a host process such as torch has
// already loaded is reused), so the library itself loads on machines without NCCL. The reference
// has no host-side communication at all; its device-side multimem primitives are not used here.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "decode_out.h"

struct ptxstd_dist {
    ncclComm_t comm;
    int nranks;
    int rank;
    int device;
    // peer-to-peer decode output (ptxstd_dist_decode_p2p_init)
    uint8_t* p2p_local = nullptr;                       // this rank's y [16][N] + signal words
    uint8_t* p2p_peer[ptxstd::decode::kMaxRanks] = {};  // every rank's buffer, mapped here
    int64_t p2p_n = 0;
};

namespace {

struct Nccl {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
};

Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        n.get_unique_id = reinterpret_cast<decltype(n.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        n.comm_init_rank =
            reinterpret_cast<decltype(n.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        n.comm_destroy = reinterpret_cast<decltype(n.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        n.all_gather = reinterpret_cast<decltype(n.all_gather)>(dlsym(h, "ncclAllGather"));
        n.error_string = reinterpret_cast<decltype(n.error_string)>(dlsym(h, "ncclGetErrorString"));
        n.ok = n.get_unique_id && n.comm_init_rank && n.comm_destroy && n.all_gather;
    });
    return n;
}

// [world][M][ns] bf16 -> [M][world * ns], 16 bytes (8 bf16) per thread; ns % 8 == 0.
__global__ void __launch_bounds__(256) unshard_columns_kernel(const uint4* __restrict__ g,
                                                              uint4* __restrict__ y, uint32_t world,
                                                              uint32_t M, uint32_t ns8) {
    const size_t total = static_cast<size_t>(world) * M * ns8;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t c = i % ns8;
        const size_t m = (i / ns8) % M;
        const size_t r = i / (static_cast<size_t>(ns8) * M);
        y[m * world * ns8 + r * ns8 + c] = g[i];
    }
}

}  // namespace

extern "C" {

int ptxstd_dist_unique_id(uint8_t* out_128) {
    if (!out_128) return PTXSTD_EINVAL;
    Nccl& n = nccl();
    if (!n.ok) return PTXSTD_ENCCL;
    ncclUniqueId id;
    if (n.get_unique_id(&id) != ncclSuccess) return PTXSTD_ENCCL;
    static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out_128, &id, 128);
    return PTXSTD_OK;
}

int ptxstd_dist_init(const uint8_t* unique_id_128, int nranks, int rank, ptxstd_dist** out) {
    if (!unique_id_128 || !out || nranks < 1 || rank < 0 || rank >= nranks) return PTXSTD_EINVAL;
    Nccl& n = nccl();
    if (!n.ok) return PTXSTD_ENCCL;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return PTXSTD_ECUDA;
    ncclUniqueId id;
    memcpy(&id, unique_id_128, 128);
    ncclComm_t comm = nullptr;
    if (n.comm_init_rank(&comm, nranks, id, rank) != ncclSuccess) return PTXSTD_ENCCL;
    *out = new ptxstd_dist{comm, nranks, rank, dev};
    return PTXSTD_OK;
}

int ptxstd_dist_free(ptxstd_dist* d) {
    if (!d) return PTXSTD_OK;
    Nccl& n = nccl();
    int st = PTXSTD_OK;
    if (d->p2p_local) {
        // every rank unmaps the peers' buffers, then all ranks meet before any buffer is freed
        if (cudaDeviceSynchronize() != cudaSuccess) st = PTXSTD_ECUDA;
        for (int r = 0; r < d->nranks; ++r)
            if (r != d->rank && d->p2p_peer[r] && cudaIpcCloseMemHandle(d->p2p_peer[r]) != cudaSuccess)
                st = PTXSTD_ECUDA;
        if (n.ok && d->comm) {
            uint8_t* tmp = nullptr;
            if (cudaMalloc(&tmp, 16 * static_cast<size_t>(d->nranks)) != cudaSuccess) {
                st = PTXSTD_ECUDA;
            } else {
                if (n.all_gather(tmp + 16 * d->rank, tmp, 16, ncclUint8, d->comm, 0) != ncclSuccess)
                    st = PTXSTD_ENCCL;
                if (cudaDeviceSynchronize() != cudaSuccess) st = PTXSTD_ECUDA;
                cudaFree(tmp);
            }
        }
        if (cudaFree(d->p2p_local) != cudaSuccess) st = PTXSTD_ECUDA;
    }
    if (n.ok && d->comm && n.comm_destroy(d->comm) != ncclSuccess) st = PTXSTD_ENCCL;
    delete d;
    return st;
}

int ptxstd_dist_size(const ptxstd_dist* d, int* nranks, int* rank) {
    if (!d || !nranks || !rank) return PTXSTD_EINVAL;
    *nranks = d->nranks;
    *rank = d->rank;
    return PTXSTD_OK;
}

int ptxstd_gemm_nvfp4_sharded(const ptxstd_dist* d, const uint8_t* d_a, const uint8_t* d_sfa,
                              float ga, const uint8_t* d_b_shard, const uint8_t* d_sfb_shard,
                              float gb, uint16_t* d_c_shard, int64_t M, int64_t N, int64_t K,
                              ptxstd_stream stream) {
    if (!d || N % d->nranks != 0) return PTXSTD_EINVAL;
    return ptxstd_gemm_nvfp4(d_a, d_sfa, ga, d_b_shard, d_sfb_shard, gb, d_c_shard, M,
                             N / d->nranks, K, stream);
}

size_t ptxstd_gemm_decode_sharded_workspace_bytes(const ptxstd_dist* d, int64_t M, int64_t N,
                                                  int64_t K) {
    if (!d || M <= 0 || N <= 0 || K <= 0 || N % d->nranks != 0) return 0;
    const int64_t ns = N / d->nranks;
    const size_t dec = ptxstd_gemm_decode_workspace_bytes(M, ns, K);
    const size_t gather = static_cast<size_t>(M) * static_cast<size_t>(N) * 2;
    return ((dec + 1023) & ~static_cast<size_t>(1023)) + gather;
}

int ptxstd_gemm_decode_sharded(const ptxstd_dist* d, const uint16_t* d_x, const uint8_t* d_w_shard,
                               const uint8_t* d_sfw_shard, float gw, uint16_t* d_y, int64_t M,
                               int64_t N, int64_t K, void* d_workspace, size_t workspace_bytes,
                               ptxstd_stream stream) {
    if (!d || !d_y || !d_workspace || M <= 0 || N <= 0 || N % d->nranks != 0) return PTXSTD_EINVAL;
    const int64_t ns = N / d->nranks;
    if (ns % 8 != 0) return PTXSTD_EINVAL;
    const size_t need = ptxstd_gemm_decode_sharded_workspace_bytes(d, M, N, K);
    if (need == 0 || workspace_bytes < need || !ptxstd::aligned16(d_y)) return PTXSTD_EINVAL;
    const size_t dec = ptxstd_gemm_decode_workspace_bytes(M, ns, K);
    uint8_t* ws = static_cast<uint8_t*>(d_workspace);
    uint16_t* gather = reinterpret_cast<uint16_t*>(ws + ((dec + 1023) & ~static_cast<size_t>(1023)));
    uint16_t* mine = gather + static_cast<size_t>(d->rank) * M * ns;
    int st = ptxstd_gemm_decode(d_x, d_w_shard, d_sfw_shard, gw, mine, M, ns, K, ws, dec, stream);
    if (st) return st;
    auto s = static_cast<cudaStream_t>(stream);
    if (d->nranks > 1) {
        Nccl& n = nccl();
        if (!n.ok) return PTXSTD_ENCCL;
        // in place: rank r's block already sits at offset r * count
        if (n.all_gather(mine, gather, static_cast<size_t>(M) * ns * 2, ncclUint8, d->comm, s) !=
            ncclSuccess)
            return PTXSTD_ENCCL;
    }
    const uint32_t ns8 = static_cast<uint32_t>(ns / 8);
    const size_t work = static_cast<size_t>(d->nranks) * M * ns8;
    const int grid = static_cast<int>(std::min<size_t>((work + 255) / 256,
                                                       static_cast<size_t>(ptxstd::sm_count()) * 4));
    unshard_columns_kernel<<<grid, 256, 0, s>>>(reinterpret_cast<const uint4*>(gather),
                                                reinterpret_cast<uint4*>(d_y),
                                                static_cast<uint32_t>(d->nranks),
                                                static_cast<uint32_t>(M), ns8);
    return ptxstd::launch_status();
}

namespace {
constexpr int64_t kP2pRows = 16;
size_t p2p_y_bytes(int64_t N) {
    return (static_cast<size_t>(kP2pRows) * static_cast<size_t>(N) * 2 + 255) &
           ~static_cast<size_t>(255);
}
}  // namespace

int ptxstd_dist_decode_p2p_init(ptxstd_dist* d, int64_t N, uint16_t** d_y) {
    namespace pd = ptxstd::decode;
    if (!d || !d_y || N <= 0 || N % (128 * static_cast<int64_t>(d->nranks)) != 0 ||
        d->nranks > static_cast<int>(pd::kMaxRanks))
        return PTXSTD_EINVAL;
    if (d->p2p_local) return PTXSTD_EINVAL;  // once per communicator
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return PTXSTD_ECUDA;
    if (cur != d->device) return PTXSTD_EINVAL;  // the communicator's GPU must be current
    Nccl& n = nccl();
    if (!n.ok) return PTXSTD_ENCCL;
    const size_t bytes = p2p_y_bytes(N) + pd::kSigWords * sizeof(uint32_t);
    uint8_t* buf = nullptr;
    if (cudaMalloc(&buf, bytes) != cudaSuccess) return PTXSTD_ECUDA;
    // zeroed (counters at 0) before any peer can learn the handle
    if (cudaMemset(buf, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(buf);
        return PTXSTD_ECUDA;
    }
    cudaIpcMemHandle_t h;
    static_assert(sizeof(h) == 64, "IPC handle size");
    if (cudaIpcGetMemHandle(&h, buf) != cudaSuccess) {
        cudaFree(buf);
        return PTXSTD_ECUDA;
    }
    // every rank's record {IPC handle, GPU UUID}, gathered with one NCCL all-gather through a
    // device staging buffer
    constexpr size_t kRec = 128;
    uint8_t mine[kRec] = {};
    memcpy(mine, &h, 64);
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, d->device) != cudaSuccess) {
        cudaFree(buf);
        return PTXSTD_ECUDA;
    }
    static_assert(sizeof(prop.uuid) == 16, "UUID size");
    memcpy(mine + 64, &prop.uuid, 16);
    uint8_t* stage = nullptr;
    std::vector<uint8_t> all(kRec * static_cast<size_t>(d->nranks));
    int st = PTXSTD_OK;
    if (cudaMalloc(&stage, all.size()) != cudaSuccess) st = PTXSTD_ECUDA;
    if (!st && cudaMemcpy(stage + kRec * d->rank, mine, kRec, cudaMemcpyHostToDevice) != cudaSuccess)
        st = PTXSTD_ECUDA;
    if (!st && n.all_gather(stage + kRec * d->rank, stage, kRec, ncclUint8, d->comm, 0) !=
                   ncclSuccess)
        st = PTXSTD_ENCCL;
    if (!st && (cudaMemcpy(all.data(), stage, all.size(), cudaMemcpyDeviceToHost) != cudaSuccess))
        st = PTXSTD_ECUDA;
    if (stage) cudaFree(stage);
    // The step's kernels wait on the other ranks' kernels, so every rank needs a GPU of its own:
    // two ranks on one GPU are refused (every rank sees the same records and decides the same).
    for (int a = 0; !st && a < d->nranks; ++a)
        for (int b = a + 1; !st && b < d->nranks; ++b)
            if (memcmp(all.data() + kRec * a + 64, all.data() + kRec * b + 64, 16) == 0)
                st = PTXSTD_EUNSUPPORTED;
    for (int r = 0; !st && r < d->nranks; ++r) {
        if (r == d->rank) {
            d->p2p_peer[r] = buf;
            continue;
        }
        cudaIpcMemHandle_t hr;
        memcpy(&hr, all.data() + kRec * r, 64);
        void* p = nullptr;
        if (cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
            st = PTXSTD_ECUDA;
        d->p2p_peer[r] = static_cast<uint8_t*>(p);
    }
    if (st) {
        for (int r = 0; r < d->nranks; ++r)
            if (r != d->rank && d->p2p_peer[r]) cudaIpcCloseMemHandle(d->p2p_peer[r]);
        memset(d->p2p_peer, 0, sizeof(d->p2p_peer));
        cudaFree(buf);
        return st;
    }
    d->p2p_local = buf;
    d->p2p_n = N;
    *d_y = reinterpret_cast<uint16_t*>(buf);
    return PTXSTD_OK;
}

int ptxstd_gemm_decode_sharded_p2p(const ptxstd_dist* d, const uint16_t* d_x,
                                   const uint8_t* d_w_shard, const uint8_t* d_sfw_shard, float gw,
                                   uint16_t* d_y, int64_t M, int64_t N, int64_t K,
                                   void* d_workspace, size_t workspace_bytes,
                                   ptxstd_stream stream) {
    namespace pd = ptxstd::decode;
    if (!d || !d->p2p_local || N != d->p2p_n || M <= 0 || M > kP2pRows || !d_workspace)
        return PTXSTD_EINVAL;
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) return PTXSTD_ECUDA;
    if (cur != d->device) return PTXSTD_EINVAL;  // the communicator's GPU must be current
    const int64_t ns = N / d->nranks;
    if (ns % 128 != 0) return PTXSTD_EINVAL;
    const size_t dec = ptxstd_gemm_decode_workspace_bytes(M, ns, K);
    if (dec == 0 || workspace_bytes < dec) return PTXSTD_EINVAL;
    pd::Out out = {};
    for (int r = 0; r < d->nranks; ++r) {
        out.y[r] = reinterpret_cast<uint16_t*>(d->p2p_peer[r]);
        out.sig[r] = reinterpret_cast<uint32_t*>(d->p2p_peer[r] + p2p_y_bytes(N));
    }
    out.nranks = static_cast<uint32_t>(d->nranks);
    out.rank = static_cast<uint32_t>(d->rank);
    out.ldy = static_cast<uint64_t>(N);
    out.col0 = static_cast<uint64_t>(d->rank) * static_cast<uint64_t>(ns);
    auto s = static_cast<cudaStream_t>(stream);
    int st = pd::launch(d_x, d_w_shard, d_sfw_shard, gw, out, M, ns, K,
                        static_cast<uint8_t*>(d_workspace), s);
    if (st || !d_y) return st;
    if (cudaMemcpyAsync(d_y, d->p2p_local, static_cast<size_t>(M) * N * 2,
                        cudaMemcpyDeviceToDevice, s) != cudaSuccess)
        return PTXSTD_ECUDA;
    return PTXSTD_OK;
}

}  // extern "C"

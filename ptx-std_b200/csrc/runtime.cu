// Library-level entry points: status strings, version, device check, and the per-device error
// word that every bounded device-side wait reports into.
#include <mutex>
#include <utility>
#include <vector>

#include "common.cuh"

namespace {

// {status, detail} of the first device-side failure since the last clear.
__device__ uint32_t g_error_word[2];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
uint32_t* g_error_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};

int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    return d;
}

}  // namespace

namespace ptxstd {

// Address of this device's error word, from cudaGetSymbolAddress on first use per device (the
// symbol's host name is not a device address).
uint32_t* device_error_word() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_error_ptr[d] == nullptr) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_error_word) != cudaSuccess) return nullptr;
        g_error_ptr[d] = static_cast<uint32_t*>(p);
    }
    return g_error_ptr[d];
}

int sm_count() {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return 148;
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_sm_count[d] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d) != cudaSuccess || n <= 0)
            n = 148;
        g_sm_count[d] = n;
    }
    return g_sm_count[d];
}

int set_max_dynamic_smem(const void* kernel, int bytes) {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return PTXSTD_ECUDA;
    static std::mutex mu;
    static std::vector<std::pair<const void*, uint64_t>> done;  // (kernel, device mask)
    std::lock_guard<std::mutex> lock(mu);
    for (auto& e : done)
        if (e.first == kernel && (e.second >> d) & 1u) return PTXSTD_OK;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
        cudaSuccess)
        return PTXSTD_ECUDA;
    for (auto& e : done)
        if (e.first == kernel) {
            e.second |= 1ull << d;
            return PTXSTD_OK;
        }
    done.emplace_back(kernel, 1ull << d);
    return PTXSTD_OK;
}

}  // namespace ptxstd

extern "C" {

const char* ptxstd_status_string(int status) {
    switch (status) {
    case PTXSTD_OK: return "ok";
    case PTXSTD_EINVAL: return "invalid argument";
    case PTXSTD_ECUDA: return "CUDA error";
    case PTXSTD_ENCCL: return "NCCL error";
    case PTXSTD_ETIMEOUT: return "device-side wait timed out";
    case PTXSTD_EUNSUPPORTED: return "unsupported device";
    default: return "unknown status";
    }
}

int ptxstd_version(void) { return 100; }

int ptxstd_device_supported(int device) {
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return PTXSTD_ECUDA;
    return (prop.major == 10 && prop.minor == 0) ? PTXSTD_OK : PTXSTD_EUNSUPPORTED;
}

int ptxstd_last_device_error(ptxstd_stream stream, int clear, int* code, uint32_t* detail) {
    if (code == nullptr) return PTXSTD_EINVAL;
    uint32_t* w = ptxstd::device_error_word();
    if (w == nullptr) return PTXSTD_ECUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t h[2] = {0, 0};
    if (cudaMemcpyAsync(h, w, sizeof h, cudaMemcpyDeviceToHost, s) != cudaSuccess)
        return PTXSTD_ECUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return PTXSTD_ECUDA;
    if (clear) {
        if (cudaMemsetAsync(w, 0, sizeof h, s) != cudaSuccess) return PTXSTD_ECUDA;
        if (cudaStreamSynchronize(s) != cudaSuccess) return PTXSTD_ECUDA;
    }
    *code = static_cast<int>(h[0]);
    if (detail) *detail = h[1];
    return PTXSTD_OK;
}

}  // extern "C"

// Output routing of the decode GEMM, shared by the single-GPU entry points (one local output) and
// the peer-to-peer sharded path of the multi-GPU layer (every rank's output over NVLink).
//
// Peer-to-peer protocol. Each rank owns one peer-shared buffer: y [16][N] bf16 followed by
// kSigWords 32-bit signal words, all counters monotonic (compared wrap-safe):
//   - [kSigReady + r]: steps rank r has started, raised by r's prep kernel on every rank;
//   - [kSigDone + r]: steps whose output rank r has finished storing here;
//   - [kSigStep]: this rank's own step count, raised by its prep kernel (in device memory, so a
//     captured CUDA graph replays correct steps).
// Per step: the prep kernel raises its step and every rank's READY[self]; the epilogue warps wait
// (bounded, before their first accumulator) until READY[r] >= step for every r, i.e. every rank's
// stream has passed its readers of the previous step, then store each finalised block's bf16
// values into every rank's y; after the GEMM kernel completes, a one-block kernel fences at system
// scope, raises DONE[self] on every rank and waits (bounded) until DONE[r] >= step for every r,
// after which y holds all N columns.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace ptxstd::decode {

constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kSigReady = 0, kSigDone = kMaxRanks, kSigStep = 2 * kMaxRanks;
constexpr uint32_t kSigWords = 2 * kMaxRanks + 1;

struct Out {
    uint16_t* y[kMaxRanks];    // output of each rank (y[0] only, and local, when nranks == 0)
    uint32_t* sig[kMaxRanks];  // signal words of each rank (nranks > 0)
    uint32_t nranks;           // 0: single GPU, plain local output
    uint32_t rank;
    uint64_t ldy;              // row stride of y in elements
    uint64_t col0;             // column of this launch's first output column in y
};

// Prep + decode kernels (+ the completion wait when out.nranks > 0) on `stream`.
int launch(const uint16_t* x, const uint8_t* W, const uint8_t* sfW, float gw, const Out& out,
           int64_t M, int64_t N, int64_t K, uint8_t* ws, cudaStream_t stream);

}  // namespace ptxstd::decode

// Host entry points of the tensor-core (tcgen05, split-bf16) path.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "m3ssd_common.cuh"

namespace m3ssd {
namespace tc {

// The tensor-core path blocks the sequence in chunks of 64 positions internally.
constexpr int kChunk = 64;

// kernels enqueued by one run_fwd call (the memset of the flag area is not a kernel)
constexpr int kFwdLaunches = 1;

// head_dim = state_dim = 64, real x, B/C with contiguous state dim and 16-byte aligned strides
bool fwd_supported(const Problem& p);
size_t fwd_workspace_bytes(const Problem& p);
int run_fwd(const Problem& p, float* y, void* states, void* ws, cudaStream_t st);

}  // namespace tc
}  // namespace m3ssd

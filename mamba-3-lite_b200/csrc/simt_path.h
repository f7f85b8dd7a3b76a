// Host entry points of the generic fp32 CUDA-core path (simt_path.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>

#include "m3ssd_common.cuh"

namespace m3ssd {
namespace simt {

// kernels enqueued by one run_fwd / run_bwd call
constexpr int kFwdLaunches = 4;
constexpr int kBwdLaunches = 9;

size_t states_bytes(const Problem& p);
size_t fwd_workspace_bytes(const Problem& p);
size_t bwd_workspace_bytes(const Problem& p);

int run_fwd(const Problem& p, float* y, void* states, void* ws, cudaStream_t st);
int run_bwd(const Problem& p, const float* dy, const long long dys[4], const void* states,
            void* dx, float2* dA, float2* dB, float2* dC, float* ddt, void* ws, cudaStream_t st);

}  // namespace simt
}  // namespace m3ssd

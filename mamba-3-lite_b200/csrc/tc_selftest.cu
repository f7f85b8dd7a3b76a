// Self-test of the bounded waits every tensor-core kernel relies on: one thread runs the same
// helpers the kernels use (mbar_wait on an mbarrier nobody arrives at, flag_wait on a hand-off flag
// nobody sets). Each must give up after its bound, record its bit in the status word and return,
// leaving the CUDA context usable: this is how a lost hand-off is reported instead of hanging the
// GPU. It faults nothing and waits on nothing that can hang (the bounds are ~1 s each).
#include <cuda_runtime.h>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"
#include "tc_path.h"

namespace m3ssd {
namespace tc {

namespace {

__global__ void k_selftest_waits(uint32_t* ws) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);  // expects one arrival that never comes
  fence_barrier_init();
  mbar_wait(&bar, 0u, ws, kErrMmaWait);
  flag_wait(ws + 1, ws);  // ws[1] is zero and nothing sets it
}

}  // namespace

int run_selftest_waits(void* ws, cudaStream_t st) {
  if (cudaMemsetAsync(ws, 0, 256, st) != cudaSuccess) return M3SSD_ERR_LAUNCH;
  k_selftest_waits<<<1, 32, 0, st>>>(static_cast<uint32_t*>(ws));
  return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace m3ssd

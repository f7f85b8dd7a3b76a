// Per-phase timestamps of the tensor-core kernels: where a chunk ticket's time goes.
//
// Compiled in only with -DM3SSD_TRACE (a separate measurement build of the library); in the
// default build every M3_TRACE is empty. In a trace build each kernel file holds a device pointer
// that m3ssd_trace_set_<kernel>() points at a caller buffer of
// kTraceCtas x kTraceIters x kTraceSlots 64-bit SM clock stamps: stamp `slot` of the `it`-th
// ticket of CTA `blockIdx.x`, taken by lane 0 of the calling warp (CTAs and tickets past the
// limits are not recorded). Stamps of one CTA share its SM's clock.
#pragma once

#include <stdint.h>

namespace m3ssd {
namespace tc {
constexpr int kTraceCtas = 16, kTraceIters = 64, kTraceSlots = 48;
}  // namespace tc
}  // namespace m3ssd

#ifdef M3SSD_TRACE
#define M3_TRACE_DEFINE(setter)                                                          \
  static __constant__ unsigned long long* g_m3_trace = nullptr;                          \
  extern "C" __attribute__((visibility("default"))) int setter(void* buf) {              \
    unsigned long long* p = static_cast<unsigned long long*>(buf);                       \
    return (int)cudaMemcpyToSymbol(g_m3_trace, &p, sizeof(p));                           \
  }
#define M3_TRACE(it, slot)                                                               \
  do {                                                                                   \
    if (g_m3_trace != nullptr && blockIdx.x < (unsigned)::m3ssd::tc::kTraceCtas &&       \
        (int)(it) < ::m3ssd::tc::kTraceIters && (threadIdx.x & 31) == 0)                 \
      g_m3_trace[((size_t)blockIdx.x * ::m3ssd::tc::kTraceIters + (it)) *               \
                     ::m3ssd::tc::kTraceSlots + (slot)] = (unsigned long long)clock64(); \
  } while (0)
#else
#define M3_TRACE_DEFINE(setter)
#define M3_TRACE(it, slot) ((void)0)
#endif

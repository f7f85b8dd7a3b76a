// Complex x on the tensor-core path, as two passes of the real-x kernels.
//
// The operator is linear in x. With x = xr + i xi, the state splits as s = s_r + i s_i, where
// s_r is driven by xr and s_i by xi (models/ssd_complex.py:17-33), so
//   y = Re(sum_n C s) = Re(sum_n C s_r) + Re(sum_n (i C) s_i) = F(xr; C) + F(xi; i C),
// F the real-x operator with the same A, B, dt. The second pass multiplies C by i as it converts
// the C tile (crot), so nothing is materialised, and adds its y into the first pass's with TMA
// reduce-add stores. Gradients in PyTorch's convention (dL/dRe + i dL/dIm): dx = dxr + i dxi,
// dB, dA, ddt are the sums of the two passes', and dC = dC_1 + conj(i) dC_2 (the second pass
// rotates its dC by conj(crot) in the epilogue and adds it with reduce-add stores).
//
// `states` holds the first pass's H tiles, then the decay records (shared: A and dt are the same),
// then the second pass's H tiles. The backward writes the two real parts of dx into its workspace
// and interleaves them into the complex dx at the end.
#include <cuda_runtime.h>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"
#include "tc_path.h"

namespace m3ssd {
namespace tc {

namespace {

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

size_t dx_part_bytes(const Problem& p) {
  return al256(sizeof(float) * 64 * (size_t)p.Bsz * p.T * p.H);
}

// dx[i] = dxr[i] + i dxi[i], four elements per thread and step (n4 = elements / 4)
__global__ void __launch_bounds__(256) k_interleave_dx(const float4* __restrict__ re,
                                                       const float4* __restrict__ im,
                                                       float4* __restrict__ out, long long n4) {
  for (long long i = blockIdx.x * 256ll + threadIdx.x; i < n4; i += (long long)gridDim.x * 256) {
    const float4 a = re[i], b = im[i];
    out[2 * i] = make_float4(a.x, b.x, a.y, b.y);
    out[2 * i + 1] = make_float4(a.z, b.z, a.w, b.w);
  }
}

}  // namespace

Problem real_part_view(const Problem& p, int part) {
  Problem q = p;
  q.x_complex = 0;
  q.x_pair = 1;
  q.x = static_cast<const float*>(p.x) + part;
  for (int i = 0; i < 4; ++i) q.xs[i] = 2 * p.xs[i];  // complex strides in floats
  return q;
}

size_t complex_states_bytes(const Problem& p) {
  return 2 * states_h_bytes(p) + chunk_prep_bytes(p);
}

size_t complex_bwd_workspace_bytes(const Problem& p) {
  return al256(bwd_workspace_bytes(real_part_view(p, 0), 1)) + 2 * dx_part_bytes(p);
}

int run_fwd_complex(const Problem& p, void* y, void* states, void* ws, cudaStream_t st) {
  const Problem q0 = real_part_view(p, 0), q1 = real_part_view(p, 1);
  char* base = static_cast<char*>(states);
  const void* recs = base + states_h_bytes(p);
  void* states1 = base + states_h_bytes(p) + chunk_prep_bytes(p);
  int rc = run_fwd(q0, y, states, ws, st);
  if (rc != M3SSD_OK) return rc;
  return run_fwd(q1, y, states1, ws, st, nullptr, nullptr, 1, /*prep=*/false,
                 /*clear_status=*/false, recs, make_float2(0.f, 1.f), /*y_accum=*/true);
}

int run_bwd_complex(const Problem& p, const void* dy, const long long dys[4], const void* states,
                    float2* dx, float2* dA, float2* dB, float2* dC, float* ddt, void* ws,
                    cudaStream_t st) {
  const Problem q0 = real_part_view(p, 0), q1 = real_part_view(p, 1);
  const char* base = static_cast<const char*>(states);
  const void* recs = base + states_h_bytes(p);
  const void* states1 = base + states_h_bytes(p) + chunk_prep_bytes(p);
  float* dxr = reinterpret_cast<float*>(static_cast<char*>(ws) +
                                        al256(bwd_workspace_bytes(q0, 1)));
  float* dxi = reinterpret_cast<float*>(reinterpret_cast<char*>(dxr) + dx_part_bytes(p));
  int rc = run_bwd(q0, dy, dys, states, contiguous_bwd_out(q0, dxr, dA, dB, dC, ddt), ws, st);
  if (rc != M3SSD_OK) return rc;
  rc = run_bwd(q1, dy, dys, states1, contiguous_bwd_out(q1, dxi, dA, dB, dC, ddt), ws, st,
               nullptr, nullptr, nullptr, 1, nullptr, /*clear_status=*/false, recs,
               make_float2(0.f, 1.f), /*accum=*/true);
  if (rc != M3SSD_OK) return rc;
  const long long n4 = 16ll * p.Bsz * p.T * p.H;  // 64 values per (b, t, h), 4 per step
  const int sms = sm_count();
  long long blocks = (n4 + 255) / 256;
  if (sms > 0 && blocks > 8ll * sms) blocks = 8ll * sms;
  k_interleave_dx<<<(unsigned)blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(dxr),
                                                    reinterpret_cast<const float4*>(dxi),
                                                    reinterpret_cast<float4*>(dx), n4);
  return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace m3ssd

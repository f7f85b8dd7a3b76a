// Per-chunk decay quantities for the tensor-core kernels (one small launch per call).
//
// For each (sequence b*H + h, chunk z) of 64 positions: a_t = softplus(dt_t) A_h
// (models/ssd_complex.py:82, a = 0 past T), the within-chunk inclusive cumsum Sigma_l (:89) as
// rho + i theta, and the factors the chunk kernels use: exp(rho_l), exp(rho_Gamma - rho_l)
// (decay_states, :90), cis(theta_l), e^Gamma and cis(theta_Gamma), plus softplus and its
// derivative for the backward. Moving this out of the chunk kernels removes a serial
// scan-and-transcendental phase (three CTA barriers) from every chunk they process.
#include <cuda_runtime.h>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"
#include "tc_path.h"

namespace m3ssd {
namespace tc {

__global__ void __launch_bounds__(128) k_chunk_prep(const float2* __restrict__ A,
                                                    const float* __restrict__ dt,
                                                    long long ds0, long long ds1, long long ds2,
                                                    int Bsz, int T, int H, int nc,
                                                    ChunkRec* __restrict__ out) {
  __shared__ float2 carry[2];
  const int rec = blockIdx.x * 2 + (threadIdx.x >> 6);  // two records per block
  const int l = threadIdx.x & 63, lane = threadIdx.x & 31;
  const int half = threadIdx.x >> 6;
  const bool valid = rec < Bsz * H * nc;
  const int z = valid ? rec % nc : 0, bh = valid ? rec / nc : 0;
  const int b = bh / H, h = bh % H, t = 64 * z + l;
  float2 a = make_float2(0.f, 0.f);
  float sp = 0.f, dsp = 0.f;
  if (valid && t < T) {
    const float v = dt[b * ds0 + (long long)t * ds1 + h * ds2];
    sp = softplus_f(v);
    dsp = softplus_grad_f(v);
    const float2 Ah = A[h];
    a = make_float2(sp * Ah.x, sp * Ah.y);
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float ux = __shfl_up_sync(0xffffffffu, a.x, o);
    const float uy = __shfl_up_sync(0xffffffffu, a.y, o);
    if (lane >= o) {
      a.x += ux;
      a.y += uy;
    }
  }
  if (l == 31) carry[half] = a;
  __syncthreads();
  if (l >= 32) {
    a.x += carry[half].x;
    a.y += carry[half].y;
  }
  __shared__ float2 gam[2];
  if (l == 63) gam[half] = a;
  __syncthreads();
  if (!valid) return;
  ChunkRec* r = out + rec;
  float sn, cs;
  sincosf(a.y, &sn, &cs);
  r->rho2[l] = a.x * 1.4426950408889634f;  // log2(e)
  r->el[l] = expf(a.x);
  r->dec[l] = expf(gam[half].x - a.x);
  r->sp[l] = sp;
  r->dsp[l] = dsp;
  r->cis[l] = make_float2(cs, sn);
  if (l == 63) {
    const float mg = expf(a.x);
    r->g = make_float2(mg * cs, mg * sn);
    r->ct = make_float2(cs, sn);
    r->pad[0] = r->pad[1] = make_float2(0.f, 0.f);
  }
}

size_t chunk_prep_bytes(const Problem& p) {
  return sizeof(ChunkRec) * (size_t)p.Bsz * p.H * ((p.T + 63) / 64);
}

int run_chunk_prep(const Problem& p, ChunkRec* out, cudaStream_t st) {
  const int nrec = p.Bsz * p.H * ((p.T + 63) / 64);
  k_chunk_prep<<<(nrec + 1) / 2, 128, 0, st>>>(p.A, p.dt, p.dts[0], p.dts[1], p.dts[2], p.Bsz,
                                                p.T, p.H, (p.T + 63) / 64, out);
  return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace m3ssd

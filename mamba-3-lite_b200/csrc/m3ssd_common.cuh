// Shared device helpers and the internal problem descriptor of the m3ssd kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "m3ssd.h"

namespace m3ssd {

// ---------------------------------------------------------------------------------------------
// complex64 helpers (float2: x = real, y = imaginary)
// ---------------------------------------------------------------------------------------------
__host__ __device__ __forceinline__ float2 cz() { return make_float2(0.f, 0.f); }
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
// acc += a * b
__device__ __forceinline__ void cfma(float2& acc, float2 a, float2 b) {
  acc.x = fmaf(a.x, b.x, fmaf(-a.y, b.y, acc.x));
  acc.y = fmaf(a.x, b.y, fmaf(a.y, b.x, acc.y));
}
// exp(z) for complex z, with the accurate libdevice expf / sincosf (phases reach ~1e2 rad).
__device__ __forceinline__ float2 cexp(float2 z) {
  float s, c;
  sincosf(z.y, &s, &c);
  const float m = expf(z.x);
  return make_float2(m * c, m * s);
}

// torch.nn.functional.softplus with beta = 1, threshold = 20 (models/ssd_complex.py:14, :82)
__device__ __forceinline__ float softplus_f(float v) { return v > 20.f ? v : log1pf(expf(v)); }
// d softplus / dv as torch computes it: e^v / (e^v + 1) below the threshold, 1 above it
__device__ __forceinline__ float softplus_grad_f(float v) {
  if (v > 20.f) return 1.f;
  const float z = expf(v);
  return z / (z + 1.f);
}

// ---------------------------------------------------------------------------------------------
// Internal problem view: raw pointers plus element strides, shared by every kernel.
// ---------------------------------------------------------------------------------------------
struct Problem {
  int Bsz, T, H, D, N, C, nc;  // nc = ceil(T / C)
  int x_complex;
  // x is one part (real or imaginary) of complex values, strides counting floats (the view a
  // complex-x pass takes): the floats between its elements belong to the same complex tensor
  int x_pair;
  const void* x;   long long xs[4];
  const float2* A;
  const float2* Bm; long long bs[4];
  const float2* Cm; long long cs[4];
  const float* dt; long long dts[3];
  // B and C in the column layout of the block's in_proj output (models/mamba_block.py:76-82):
  // planar fp32, real parts at Bm / Cm (read as float), imaginary parts H*N floats further;
  // bs / cs then count floats. Only the tensor-core kernels take this form.
  int bc_planar;
  // y (forward output) and dy (backward input) in bfloat16 (M3SSD_Y_BF16); tensor-core path only
  int y_bf16;
  __host__ __device__ __forceinline__ long long Tp() const { return (long long)nc * C; }
};

// x[b,t,h,d] as complex (imaginary part 0 for real x); 0 for padded t >= T
__device__ __forceinline__ float2 ld_x(const Problem& p, int b, int t, int h, int d) {
  if (t >= p.T) return cz();
  const long long o = b * p.xs[0] + t * p.xs[1] + h * p.xs[2] + d * p.xs[3];
  if (p.x_complex) return reinterpret_cast<const float2*>(p.x)[o];
  return make_float2(reinterpret_cast<const float*>(p.x)[o], 0.f);
}
__device__ __forceinline__ float2 ld_B(const Problem& p, int b, int t, int h, int n) {
  if (t >= p.T) return cz();
  return p.Bm[b * p.bs[0] + t * p.bs[1] + h * p.bs[2] + n * p.bs[3]];
}
__device__ __forceinline__ float2 ld_C(const Problem& p, int b, int t, int h, int n) {
  if (t >= p.T) return cz();
  return p.Cm[b * p.cs[0] + t * p.cs[1] + h * p.cs[2] + n * p.cs[3]];
}
__device__ __forceinline__ float ld_dt(const Problem& p, int b, int t, int h) {
  return p.dt[b * p.dts[0] + t * p.dts[1] + h * p.dts[2]];
}

}  // namespace m3ssd

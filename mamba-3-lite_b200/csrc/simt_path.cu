// Generic fp32 CUDA-core path of the complex chunkwise SSD operator (forward and backward).
//
// It handles every supported shape (any chunk length 1..256, any head_dim/state_dim up to 256,
// real or complex x, arbitrary input strides) and is the accurate (fp32) reference on the GPU
// for the tensor-core path. Work is chunk-parallel:
//
//   forward   k_chunk_cumsum  within-chunk cumsum of a = softplus(dt) A       (per b,h,chunk)
//             k_fwd_state     S_z = sum_s e^{Gamma-Sigma_s} B_s x_s^T            (per chunk tile)
//             k_fwd_scan      H_{z+1} = e^{Gamma_z} H_z + S_z, writes H_z in place (per b,h,n,p)
//             k_fwd_out       y = Re(sum_{s<=l} (C_l.B_s) e^{Sigma_l-Sigma_s} x_s
//                                    + e^{Sigma_l} C_l H_z)                    (per chunk tile)
//   backward  k_bwd_q         Q_z = sum_l conj(e^{Sigma_l} C_l) dy_l
//             k_bwd_scan      dS_{z-1} = Q_z + conj(e^{Gamma_z}) dS_z, plus <dS_z, e^{Gamma}H_z>
//             k_bwd_mm        M = (C.B^T) o L, dM = dy x^H, dG = dM o conj(L), W = dM o conj(M)
//             k_bwd_dc/db/dx  the three gradient contractions per chunk
//             k_bwd_da        d(Sigma) -> reverse cumsum -> ddt and per-chunk dA partials
//             k_bwd_dA        dA[h] = sum over batch and chunks (fixed order, deterministic)
//
// Chunk states (S_z, the carried H_z and the state gradients) are stored per (b*H + h, chunk)
// as [p][n] complex64, i.e. [D][2N] floats with re/im interleaved; the tensor-core path uses the
// same layout so forward and backward paths can be paired freely.
//
// Chunk-local quantities match models/ssd_complex.py:82-119: Sigma_l is the inclusive cumsum of
// a within the chunk (:89), e^{Gamma - Sigma_s} is decay_states (:90), the causal decay
// e^{Sigma_l - Sigma_s} is L (:50-52, evaluated only for s <= l), and the carried state H_z is
// what the decay_chunk einsum (:98-111) builds, here by an O(n_chunks) scan.
#include <cuda_runtime.h>

#include "m3ssd_common.cuh"
#include "simt_path.h"

namespace m3ssd {
namespace simt {

constexpr int TS = 32;   // output tile rows / cols and K step
constexpr int NT = 256;  // threads per CTA for the tiled kernels

struct TileSmem {
  float2 a[TS][TS + 1];  // [k][m]
  float2 b[TS][TS + 1];  // [k][n]
};

// What a tile product needs of each term a * b: kFull the complex product; kBReal and kAReal a
// product whose b (a) is real; kRe only the real part; kReBReal only the real part with b real.
// Each drops the multiplications by a known zero or by a part nobody reads, in the same fused
// order as cfma, so a result that is computed equals cfma's bit for bit.
enum : int { kFull, kBReal, kAReal, kRe, kReBReal };
template <int KIND>
__device__ __forceinline__ void kfma(float2& acc, float2 a, float2 b) {
  if constexpr (KIND == kFull) {
    cfma(acc, a, b);
  } else if constexpr (KIND == kBReal) {
    acc.x = fmaf(a.x, b.x, acc.x);
    acc.y = fmaf(a.y, b.x, acc.y);
  } else if constexpr (KIND == kAReal) {
    acc.x = fmaf(a.x, b.x, acc.x);
    acc.y = fmaf(a.x, b.y, acc.y);
  } else if constexpr (KIND == kRe) {
    acc.x = fmaf(a.x, b.x, fmaf(-a.y, b.y, acc.x));
  } else {
    acc.x = fmaf(a.x, b.x, acc.x);
  }
}

// acc[i] accumulates output (row tm0 + 8 i, col tn) with tn = tid % 32, tm0 = tid / 32, for
// a TS x TS output tile: out[m][n] += sum_k fa(k, m) * fb(k, n) (the parts KIND asks for).
// fa/fb return 0 outside the problem. *_KFAST selects which index varies fastest across threads
// while staging (pick the one contiguous in global memory).
template <int KIND, bool A_KFAST, bool B_KFAST, class FA, class FB>
__device__ __forceinline__ void tile_mma(float2 (&acc)[4], int K, FA fa, FB fb, TileSmem& sm) {
  constexpr int kPer = TS * TS / NT;  // elements of each operand a thread stages per K step
  const int tid = threadIdx.x, tn = tid & 31, tm0 = tid >> 5;
  // the next K step's operands are read into registers while the current one is multiplied
  float2 ra[kPer], rb[kPer];
  auto fetch = [&](int k0) {
    const int kn = min(TS, K - k0);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * NT;
      const int ka = A_KFAST ? (i % TS) : (i / TS), m = A_KFAST ? (i / TS) : (i % TS);
      const int kb = B_KFAST ? (i % TS) : (i / TS), n = B_KFAST ? (i / TS) : (i % TS);
      ra[u] = ka < kn ? fa(k0 + ka, m) : cz();
      rb[u] = kb < kn ? fb(k0 + kb, n) : cz();
    }
  };
  fetch(0);
  for (int k0 = 0; k0 < K; k0 += TS) {
    const int kn = min(TS, K - k0);
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = tid + u * NT;
      sm.a[A_KFAST ? (i % TS) : (i / TS)][A_KFAST ? (i / TS) : (i % TS)] = ra[u];
      sm.b[B_KFAST ? (i % TS) : (i / TS)][B_KFAST ? (i / TS) : (i % TS)] = rb[u];
    }
    __syncthreads();
    if (k0 + TS < K) fetch(k0 + TS);
#pragma unroll 4
    for (int k = 0; k < kn; ++k) {
      const float2 bv = sm.b[k][tn];
#pragma unroll
      for (int i = 0; i < 4; ++i) kfma<KIND>(acc[i], sm.a[k][tm0 + 8 * i], bv);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ float2 warp_sum(float2 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  return v;
}

__host__ __device__ __forceinline__ int tiles(int n) { return (n + TS - 1) / TS; }

// chunks per batch of loads in the two scans: a batch's loads are all issued before its stores,
// so a thread waits on memory once per kScanBatch chunks instead of once per chunk
constexpr int kScanBatch = 8;

// ---------------------------------------------------------------------------------------------
// within-chunk inclusive cumsum of a = softplus(dt) * A (models/ssd_complex.py:82, :89)
// acs[(b*H + h) * Tp + t]; padded positions t >= T contribute a = 0.
// ---------------------------------------------------------------------------------------------
__global__ void k_chunk_cumsum(Problem p, float2* __restrict__ acs) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)p.Bsz * p.H * p.nc) return;
  const int z = (int)(idx % p.nc);
  const int bh = (int)(idx / p.nc);
  const int b = bh / p.H, h = bh % p.H;
  const float2 A = p.A[h];
  float2 s = cz();
  float2* out = acs + (long long)bh * p.Tp() + (long long)z * p.C;
  for (int l = 0; l < p.C; ++l) {
    const int t = z * p.C + l;
    if (t < p.T) {
      const float sp = softplus_f(ld_dt(p, b, t, h));
      s.x += sp * A.x;
      s.y += sp * A.y;
    }
    out[l] = s;
  }
}

// ---------------------------------------------------------------------------------------------
// forward stage 1: per-chunk state S_z[n,p] = sum_s e^{Gamma - Sigma_s} B[s,n] x[s,p]
// (models/ssd_complex.py:54 with decay_states from :90)
// ---------------------------------------------------------------------------------------------
template <bool XC>  // x complex
__global__ void __launch_bounds__(NT) k_fwd_state(Problem p, const float2* __restrict__ acs,
                                                  float2* __restrict__ states) {
  __shared__ TileSmem sm;
  __shared__ float2 dec[256];
  const int tP = tiles(p.D);
  const int n0 = (blockIdx.x / tP) * TS, p0 = (blockIdx.x % tP) * TS;
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const float2* ac = acs + (long long)bh * p.Tp() + (long long)z * p.C;
  const float2 gam = ac[p.C - 1];
  for (int s = threadIdx.x; s < p.C; s += NT) dec[s] = cexp(csub(gam, ac[s]));
  __syncthreads();
  const int t0 = z * p.C;
  float2 acc[4] = {cz(), cz(), cz(), cz()};
  auto fa = [&](int s, int m) -> float2 {
    const int n = n0 + m;
    return n < p.N ? cmul(dec[s], ld_B(p, b, t0 + s, h, n)) : cz();
  };
  auto fb = [&](int s, int j) -> float2 {
    const int d = p0 + j;
    return d < p.D ? ld_x(p, b, t0 + s, h, d) : cz();
  };
  tile_mma<XC ? kFull : kBReal, false, false>(acc, p.C, fa, fb, sm);
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
  float2* st = states + ((long long)bh * p.nc + z) * p.N * p.D;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = n0 + tm0 + 8 * i, d = p0 + tn;
    if (n < p.N && d < p.D) st[(long long)d * p.N + n] = acc[i];
  }
}

// ---------------------------------------------------------------------------------------------
// forward stage 2: sequential chunk scan, H_0 = 0, H_{z+1} = e^{Gamma_z} H_z + S_z.
// Overwrites S_z with H_z (the state entering chunk z), equal to the decay_chunk einsum at
// models/ssd_complex.py:98-111.
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_fwd_scan(Problem p, const float2* __restrict__ acs,
                                                  float2* __restrict__ states) {
  const int bh = blockIdx.y;
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= (long long)p.N * p.D) return;
  const long long nd = (long long)p.N * p.D;
  float2* st = states + (long long)bh * p.nc * nd + e;
  const float2* ac = acs + (long long)bh * p.Tp() + (p.C - 1);
  float2 hcur = cz();
  for (int z0 = 0; z0 < p.nc; z0 += kScanBatch) {
    float2 s[kScanBatch], g[kScanBatch];
#pragma unroll
    for (int u = 0; u < kScanBatch; ++u) {
      const int z = z0 + u;
      s[u] = z < p.nc ? st[z * nd] : cz();
      g[u] = z < p.nc ? ac[(long long)z * p.C] : cz();
    }
#pragma unroll
    for (int u = 0; u < kScanBatch; ++u) {
      const int z = z0 + u;
      if (z < p.nc) {
        st[z * nd] = hcur;
        hcur = cadd(cmul(cexp(g[u]), hcur), s[u]);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------------
// forward stage 3: y[l,p] = Re( sum_{s<=l} G[l,s] e^{Sigma_l-Sigma_s} x[s,p]
//                               + e^{Sigma_l} sum_n C[l,n] H_z[n,p] )
// (models/ssd_complex.py:53 and :115-119)
// ---------------------------------------------------------------------------------------------
// One CTA per (l tile, group of kOutTiles p tiles, chunk): each G tile is formed once for the
// whole group.
constexpr int kOutTiles = 2;
template <bool XC>  // x complex; only Re(y) is formed
__global__ void __launch_bounds__(NT) k_fwd_out(Problem p, const float2* __restrict__ acs,
                                                const float2* __restrict__ states,
                                                float* __restrict__ y) {
  __shared__ TileSmem sm;
  __shared__ float2 mt[TS][TS + 1];
  __shared__ float2 el[TS];
  const int tP = tiles(p.D), gP = (tP + kOutTiles - 1) / kOutTiles;
  const int l0 = (blockIdx.x / gP) * TS, pt0 = (blockIdx.x % gP) * kOutTiles;
  const int np = min(kOutTiles, tP - pt0);  // p tiles of this CTA (uniform over the block)
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const int t0 = z * p.C;
  const float2* ac = acs + (long long)bh * p.Tp() + t0;
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
  float2 accY[kOutTiles][4];
#pragma unroll
  for (int pt = 0; pt < kOutTiles; ++pt)
#pragma unroll
    for (int i = 0; i < 4; ++i) accY[pt][i] = cz();
  const int l_end = min(l0 + TS, p.C);
  for (int s0 = 0; s0 < l_end; s0 += TS) {
    float2 accG[4] = {cz(), cz(), cz(), cz()};
    auto fa = [&](int n, int m) -> float2 {
      const int l = l0 + m;
      return (l < p.C && n < p.N) ? ld_C(p, b, t0 + l, h, n) : cz();
    };
    auto fb = [&](int n, int j) -> float2 {
      const int s = s0 + j;
      return (s < p.C && n < p.N) ? ld_B(p, b, t0 + s, h, n) : cz();
    };
    tile_mma<kFull, true, true>(accG, p.N, fa, fb, sm);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int l = l0 + tm0 + 8 * i, s = s0 + tn;
      float2 m = cz();
      if (l < p.C && s <= l) m = cmul(accG[i], cexp(csub(ac[l], ac[s])));
      mt[tm0 + 8 * i][tn] = m;
    }
    __syncthreads();
    auto fa2 = [&](int k, int m) -> float2 { return mt[m][k]; };
#pragma unroll
    for (int pt = 0; pt < kOutTiles; ++pt) {
      if (pt >= np) break;
      const int p0 = (pt0 + pt) * TS;
      auto fb2 = [&](int k, int j) -> float2 {
        const int s = s0 + k, d = p0 + j;
        return (s < p.C && d < p.D) ? ld_x(p, b, t0 + s, h, d) : cz();
      };
      tile_mma<XC ? kRe : kReBReal, true, false>(accY[pt], min(TS, p.C - s0), fa2, fb2, sm);
    }
  }
  if (threadIdx.x < TS) {
    const int l = l0 + threadIdx.x;
    el[threadIdx.x] = l < p.C ? cexp(ac[l]) : cz();
  }
  __syncthreads();
  const float2* hz = states + ((long long)bh * p.nc + z) * p.N * p.D;
  auto fa3 = [&](int n, int m) -> float2 {
    const int l = l0 + m;
    return (l < p.C && n < p.N) ? cmul(el[m], ld_C(p, b, t0 + l, h, n)) : cz();
  };
#pragma unroll
  for (int pt = 0; pt < kOutTiles; ++pt) {
    if (pt >= np) break;
    const int p0 = (pt0 + pt) * TS;
    auto fb3 = [&](int n, int j) -> float2 {
      const int d = p0 + j;
      return (n < p.N && d < p.D) ? hz[(long long)d * p.N + n] : cz();
    };
    tile_mma<kRe, true, false>(accY[pt], p.N, fa3, fb3, sm);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int l = l0 + tm0 + 8 * i, d = p0 + tn, t = t0 + l;
      if (l < p.C && t < p.T && d < p.D)
        y[(((long long)b * p.T + t) * p.H + h) * p.D + d] = accY[pt][i].x;
    }
  }
}

// ---------------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------------
struct Grad {
  const float* dy; long long dys[4];
};
__device__ __forceinline__ float ld_dy(const Problem& p, const Grad& g, int b, int t, int h, int d) {
  if (t >= p.T) return 0.f;
  return g.dy[b * g.dys[0] + t * g.dys[1] + h * g.dys[2] + d * g.dys[3]];
}

// Q_z[n,p] = sum_l conj(e^{Sigma_l} C[l,n]) dy[l,p]: gradient reaching H_z through y of chunk z
__global__ void __launch_bounds__(NT) k_bwd_q(Problem p, Grad g, const float2* __restrict__ acs,
                                              float2* __restrict__ dsbuf) {
  __shared__ TileSmem sm;
  __shared__ float2 el[256];
  const int tP = tiles(p.D);
  const int n0 = (blockIdx.x / tP) * TS, p0 = (blockIdx.x % tP) * TS;
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const int t0 = z * p.C;
  const float2* ac = acs + (long long)bh * p.Tp() + t0;
  for (int l = threadIdx.x; l < p.C; l += NT) el[l] = cconj(cexp(ac[l]));
  __syncthreads();
  float2 acc[4] = {cz(), cz(), cz(), cz()};
  auto fa = [&](int l, int m) -> float2 {
    const int n = n0 + m;
    return n < p.N ? cmul(el[l], cconj(ld_C(p, b, t0 + l, h, n))) : cz();
  };
  auto fb = [&](int l, int j) -> float2 {
    const int d = p0 + j;
    return d < p.D ? make_float2(ld_dy(p, g, b, t0 + l, h, d), 0.f) : cz();
  };
  tile_mma<kBReal, false, false>(acc, p.C, fa, fb, sm);
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
  float2* q = dsbuf + ((long long)bh * p.nc + z) * p.N * p.D;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = n0 + tm0 + 8 * i, d = p0 + tn;
    if (n < p.N && d < p.D) q[(long long)d * p.N + n] = acc[i];
  }
}

// Reverse chunk scan of the state gradient: dS_{nc-1} = 0, dS_{z-1} = Q_z + conj(e^{Gamma_z}) dS_z.
// Overwrites Q_z with dS_z (gradient of the state leaving chunk z) and writes the per-block
// partial of <dS_z, e^{Gamma_z} H_z> (the gradient of Gamma_z through the carry).
__global__ void __launch_bounds__(256) k_bwd_scan(Problem p, const float2* __restrict__ acs,
                                                  const float2* __restrict__ states,
                                                  float2* __restrict__ dsbuf,
                                                  float2* __restrict__ gpart) {
  __shared__ float2 red[kScanBatch][8];  // per chunk of a batch, one partial per warp (8 warps)
  const int bh = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long nd = (long long)p.N * p.D;
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = e < nd;
  const float2* ac = acs + (long long)bh * p.Tp() + (p.C - 1);
  float2* ds = dsbuf + (long long)bh * p.nc * nd + (valid ? e : 0);
  const float2* hz = states + (long long)bh * p.nc * nd + (valid ? e : 0);
  float2 dS = cz();
  for (int z1 = p.nc - 1; z1 >= 0; z1 -= kScanBatch) {  // chunks z1, z1 - 1, ..., z1 - 7
    float2 q[kScanBatch], hv[kScanBatch], gz[kScanBatch];
#pragma unroll
    for (int u = 0; u < kScanBatch; ++u) {
      const int z = z1 - u;
      q[u] = (valid && z >= 0) ? ds[z * nd] : cz();
      hv[u] = (valid && z >= 0) ? hz[z * nd] : cz();
      gz[u] = z >= 0 ? ac[(long long)z * p.C] : cz();
    }
#pragma unroll
    for (int u = 0; u < kScanBatch; ++u) {
      const int z = z1 - u;
      float2 part = cz();
      if (z >= 0) {
        const float2 g = cexp(gz[u]);
        if (valid) ds[z * nd] = dS;
        part = cmul(dS, cconj(cmul(g, hv[u])));
        dS = cadd(q[u], cmul(cconj(g), dS));
      }
      part = warp_sum(part);
      if (lane == 0) red[u][warp] = part;
    }
    __syncthreads();
    if (threadIdx.x < kScanBatch && z1 - (int)threadIdx.x >= 0) {
      float2 v = cz();
#pragma unroll
      for (int w = 0; w < 8; ++w) v = cadd(v, red[threadIdx.x][w]);
      gpart[((long long)bh * p.nc + (z1 - (int)threadIdx.x)) * gridDim.x + blockIdx.x] = v;
    }
    __syncthreads();
  }
}

struct BwdBufs {
  float2* mbuf;      // (bh, z, l, s) M = G o L, zero for s > l
  float2* dgbuf;     // (bh, z, l, s) dG = dM o conj(L)
  float2* rowpart;   // (bh, z, l, s_tile)   sum_s W[l,s]
  float2* colpart;   // (bh, z, s, l_tile)   sum_l W[l,s]
  float2* rowcpart;  // (bh, z, l, n_tile)   sum_n dChat conj(Chat)
  float2* upart;     // (bh, z, s, n_tile)   sum_n dBhat conj(Bhat)
  float2* gpart;     // (bh, z, scan block)  <dS_z, e^Gamma H_z>
  float2* dapart;    // (bh, z)              sum_l da softplus(dt)
};

// Per (chunk, l-tile, s-tile): M, dM, dG, W and the row/column sums of W.
template <bool XC>  // x complex
__global__ void __launch_bounds__(NT) k_bwd_mm(Problem p, Grad g, const float2* __restrict__ acs,
                                               BwdBufs w) {
  __shared__ TileSmem sm;
  __shared__ float2 cred[8][TS];
  const int tC = tiles(p.C);
  const int lt = blockIdx.x / tC, st = blockIdx.x % tC;
  const int l0 = lt * TS, s0 = st * TS;
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const int t0 = z * p.C;
  const float2* ac = acs + (long long)bh * p.Tp() + t0;
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
  const long long cc = (long long)bh * p.nc + z;
  float2 accG[4] = {cz(), cz(), cz(), cz()};
  float2 accM[4] = {cz(), cz(), cz(), cz()};
  if (st <= lt) {
    auto fa = [&](int n, int m) -> float2 {
      const int l = l0 + m;
      return (l < p.C && n < p.N) ? ld_C(p, b, t0 + l, h, n) : cz();
    };
    auto fb = [&](int n, int j) -> float2 {
      const int s = s0 + j;
      return (s < p.C && n < p.N) ? ld_B(p, b, t0 + s, h, n) : cz();
    };
    tile_mma<kFull, true, true>(accG, p.N, fa, fb, sm);
    auto fa2 = [&](int d, int m) -> float2 {
      const int l = l0 + m;
      return (l < p.C && d < p.D) ? make_float2(ld_dy(p, g, b, t0 + l, h, d), 0.f) : cz();
    };
    auto fb2 = [&](int d, int j) -> float2 {
      const int s = s0 + j;
      return (s < p.C && d < p.D) ? cconj(ld_x(p, b, t0 + s, h, d)) : cz();
    };
    tile_mma<XC ? kAReal : kReBReal, true, true>(accM, p.D, fa2, fb2, sm);  // dy real
  }
  float2 colsum = cz();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + tm0 + 8 * i, s = s0 + tn;
    const bool valid = (st <= lt) && l < p.C && s < p.C && s <= l;
    float2 mv = cz(), dgv = cz(), wv = cz();
    if (valid) {
      const float2 L = cexp(csub(ac[l], ac[s]));
      mv = cmul(accG[i], L);
      dgv = cmul(accM[i], cconj(L));
      wv = cmul(accM[i], cconj(mv));
    }
    if (l < p.C && s < p.C) {
      w.mbuf[(cc * p.C + l) * p.C + s] = mv;
      w.dgbuf[(cc * p.C + l) * p.C + s] = dgv;
    }
    const float2 rs = warp_sum(wv);
    if (tn == 0 && l < p.C) w.rowpart[(cc * p.C + l) * tC + st] = rs;
    colsum = cadd(colsum, wv);
  }
  cred[tm0][tn] = colsum;
  __syncthreads();
  if (threadIdx.x < TS) {
    float2 v = cz();
#pragma unroll
    for (int r = 0; r < 8; ++r) v = cadd(v, cred[r][threadIdx.x]);
    const int s = s0 + threadIdx.x;
    if (s < p.C) w.colpart[(cc * p.C + s) * tC + lt] = v;
  }
}

// dC[l,n] = sum_s dG[l,s] conj(B[s,n]) + conj(e^{Sigma_l}) sum_p dy[l,p] conj(H_z[n,p])
__global__ void __launch_bounds__(NT) k_bwd_dc(Problem p, Grad g, const float2* __restrict__ acs,
                                               const float2* __restrict__ states, BwdBufs w,
                                               float2* __restrict__ dC) {
  __shared__ TileSmem sm;
  const int tN = tiles(p.N);
  const int l0 = (blockIdx.x / tN) * TS, n0 = (blockIdx.x % tN) * TS;
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const int t0 = z * p.C;
  const float2* ac = acs + (long long)bh * p.Tp() + t0;
  const long long cc = (long long)bh * p.nc + z;
  const float2* hz = states + cc * p.N * p.D;
  float2 acc1[4] = {cz(), cz(), cz(), cz()};
  float2 acc2[4] = {cz(), cz(), cz(), cz()};
  auto fa = [&](int s, int m) -> float2 {
    const int l = l0 + m;
    return l < p.C ? w.dgbuf[(cc * p.C + l) * p.C + s] : cz();
  };
  auto fb = [&](int s, int j) -> float2 {
    const int n = n0 + j;
    return n < p.N ? cconj(ld_B(p, b, t0 + s, h, n)) : cz();
  };
  // dG[l][s] is zero for s > l: s stops at this tile's last row
  tile_mma<kFull, true, false>(acc1, min(p.C, l0 + TS), fa, fb, sm);
  auto fa2 = [&](int d, int m) -> float2 {
    const int l = l0 + m;
    return l < p.C ? make_float2(ld_dy(p, g, b, t0 + l, h, d), 0.f) : cz();
  };
  auto fb2 = [&](int d, int j) -> float2 {
    const int n = n0 + j;
    return n < p.N ? cconj(hz[(long long)d * p.N + n]) : cz();
  };
  tile_mma<kAReal, true, true>(acc2, p.D, fa2, fb2, sm);  // dy real
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int l = l0 + tm0 + 8 * i, n = n0 + tn, t = t0 + l;
    float2 rv = cz();
    if (l < p.C && n < p.N) {
      const float2 e = cexp(ac[l]);
      const float2 c = ld_C(p, b, t, h, n);
      if (t < p.T)
        dC[(((long long)b * p.T + t) * p.H + h) * p.N + n] = cadd(acc1[i], cmul(cconj(e), acc2[i]));
      rv = cmul(acc2[i], cconj(cmul(e, c)));
    }
    rv = warp_sum(rv);
    if (tn == 0 && l < p.C) w.rowcpart[(cc * p.C + l) * tN + blockIdx.x % tN] = rv;
  }
}

// dB[s,n] = sum_l dG[l,s] conj(C[l,n]) + conj(e^{Gamma-Sigma_s}) sum_p dS[n,p] conj(x[s,p])
template <bool XC>  // x complex
__global__ void __launch_bounds__(NT) k_bwd_db(Problem p, const float2* __restrict__ acs,
                                               const float2* __restrict__ dsbuf, BwdBufs w,
                                               float2* __restrict__ dB) {
  __shared__ TileSmem sm;
  const int tN = tiles(p.N);
  const int s0 = (blockIdx.x / tN) * TS, n0 = (blockIdx.x % tN) * TS;
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const int t0 = z * p.C;
  const float2* ac = acs + (long long)bh * p.Tp() + t0;
  const float2 gam = ac[p.C - 1];
  const long long cc = (long long)bh * p.nc + z;
  const float2* dsz = dsbuf + cc * p.N * p.D;
  float2 acc1[4] = {cz(), cz(), cz(), cz()};
  float2 acc2[4] = {cz(), cz(), cz(), cz()};
  // dG[l][s] is zero for l < s: l starts at this tile's first row (l = s0 + k)
  auto fa = [&](int k, int m) -> float2 {
    const int s = s0 + m;
    return s < p.C ? w.dgbuf[(cc * p.C + s0 + k) * p.C + s] : cz();
  };
  auto fb = [&](int k, int j) -> float2 {
    const int n = n0 + j;
    return n < p.N ? cconj(ld_C(p, b, t0 + s0 + k, h, n)) : cz();
  };
  tile_mma<kFull, false, false>(acc1, p.C - s0, fa, fb, sm);
  auto fa2 = [&](int d, int m) -> float2 {
    const int s = s0 + m;
    return s < p.C ? cconj(ld_x(p, b, t0 + s, h, d)) : cz();
  };
  auto fb2 = [&](int d, int j) -> float2 {
    const int n = n0 + j;
    return n < p.N ? dsz[(long long)d * p.N + n] : cz();
  };
  tile_mma<XC ? kFull : kAReal, true, true>(acc2, p.D, fa2, fb2, sm);
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = s0 + tm0 + 8 * i, n = n0 + tn, t = t0 + s;
    float2 uv = cz();
    if (s < p.C && n < p.N) {
      const float2 e = cexp(csub(gam, ac[s]));
      if (t < p.T)
        dB[(((long long)b * p.T + t) * p.H + h) * p.N + n] = cadd(acc1[i], cmul(cconj(e), acc2[i]));
      uv = cmul(acc2[i], cconj(cmul(e, ld_B(p, b, t, h, n))));
    }
    uv = warp_sum(uv);
    if (tn == 0 && s < p.C) w.upart[(cc * p.C + s) * tN + blockIdx.x % tN] = uv;
  }
}

// dx[s,p] = sum_l conj(M[l,s]) dy[l,p] + sum_n conj(e^{Gamma-Sigma_s} B[s,n]) dS[n,p]
template <bool XC>  // x complex (for a real x only Re(dx) is formed)
__global__ void __launch_bounds__(NT) k_bwd_dx(Problem p, Grad g, const float2* __restrict__ acs,
                                               const float2* __restrict__ dsbuf, BwdBufs w,
                                               void* __restrict__ dx) {
  __shared__ TileSmem sm;
  __shared__ float2 es[TS];
  const int tP = tiles(p.D);
  const int s0 = (blockIdx.x / tP) * TS, p0 = (blockIdx.x % tP) * TS;
  const int z = blockIdx.y, bh = blockIdx.z, b = bh / p.H, h = bh % p.H;
  const int t0 = z * p.C;
  const float2* ac = acs + (long long)bh * p.Tp() + t0;
  const long long cc = (long long)bh * p.nc + z;
  const float2* dsz = dsbuf + cc * p.N * p.D;
  if (threadIdx.x < TS) {
    const int s = s0 + threadIdx.x;
    es[threadIdx.x] = s < p.C ? cexp(csub(ac[p.C - 1], ac[s])) : cz();
  }
  __syncthreads();
  float2 acc[4] = {cz(), cz(), cz(), cz()};
  // M[l][s] is zero for l < s: l starts at this tile's first row (l = s0 + k)
  auto fa = [&](int k, int m) -> float2 {
    const int s = s0 + m;
    return s < p.C ? cconj(w.mbuf[(cc * p.C + s0 + k) * p.C + s]) : cz();
  };
  auto fb = [&](int k, int j) -> float2 {
    const int d = p0 + j;
    return d < p.D ? make_float2(ld_dy(p, g, b, t0 + s0 + k, h, d), 0.f) : cz();
  };
  tile_mma<XC ? kBReal : kReBReal, false, false>(acc, p.C - s0, fa, fb, sm);  // dy real
  auto fa2 = [&](int n, int m) -> float2 {
    const int s = s0 + m;
    return (s < p.C && n < p.N) ? cconj(cmul(es[m], ld_B(p, b, t0 + s, h, n))) : cz();
  };
  auto fb2 = [&](int n, int j) -> float2 {
    const int d = p0 + j;
    return (n < p.N && d < p.D) ? dsz[(long long)d * p.N + n] : cz();
  };
  tile_mma<XC ? kFull : kRe, true, false>(acc, p.N, fa2, fb2, sm);
  const int tn = threadIdx.x & 31, tm0 = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int s = s0 + tm0 + 8 * i, d = p0 + tn, t = t0 + s;
    if (s < p.C && d < p.D && t < p.T) {
      const long long o = (((long long)b * p.T + t) * p.H + h) * p.D + d;
      if (XC) reinterpret_cast<float2*>(dx)[o] = acc[i];
      else reinterpret_cast<float*>(dx)[o] = acc[i].x;
    }
  }
}

// d(Sigma_l) from all partials, reverse cumsum to d(a_t), then ddt and the per-chunk dA partial.
__global__ void k_bwd_da(Problem p, const float2* __restrict__ acs, BwdBufs w, int scan_blocks,
                         float* __restrict__ ddt) {
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)p.Bsz * p.H * p.nc) return;
  const int z = (int)(idx % p.nc);
  const int bh = (int)(idx / p.nc);
  const int b = bh / p.H, h = bh % p.H;
  const int tC = tiles(p.C), tN = tiles(p.N);
  const long long cc = (long long)bh * p.nc + z;
  const float2 A = p.A[h];
  // gradient of Gamma_z: sum_s u_s + <dS_z, e^Gamma H_z>
  float2 dgam = cz();
  for (int s = 0; s < p.C; ++s)
    for (int j = 0; j < tN; ++j) dgam = cadd(dgam, w.upart[(cc * p.C + s) * tN + j]);
  for (int j = 0; j < scan_blocks; ++j) dgam = cadd(dgam, w.gpart[cc * scan_blocks + j]);
  float2 run = cz(), dap = cz();
  for (int l = p.C - 1; l >= 0; --l) {
    float2 dsig = (l == p.C - 1) ? dgam : cz();
    for (int j = 0; j < tC; ++j) dsig = cadd(dsig, w.rowpart[(cc * p.C + l) * tC + j]);
    for (int j = 0; j < tN; ++j) dsig = cadd(dsig, w.rowcpart[(cc * p.C + l) * tN + j]);
    for (int j = 0; j < tC; ++j) dsig = csub(dsig, w.colpart[(cc * p.C + l) * tC + j]);
    for (int j = 0; j < tN; ++j) dsig = csub(dsig, w.upart[(cc * p.C + l) * tN + j]);
    run = cadd(run, dsig);  // d a_l = sum_{l' >= l} d Sigma_{l'}
    const int t = z * p.C + l;
    if (t < p.T) {
      const float v = ld_dt(p, b, t, h);
      const float sp = softplus_f(v);
      ddt[((long long)b * p.T + t) * p.H + h] = (run.x * A.x + run.y * A.y) * softplus_grad_f(v);
      dap = cadd(dap, cscale(run, sp));
    }
  }
  w.dapart[cc] = dap;
}

__global__ void k_bwd_dA(Problem p, const float2* __restrict__ dapart, float2* __restrict__ dA) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= p.H) return;
  float2 acc = cz();
  for (int b = 0; b < p.Bsz; ++b)
    for (int z = 0; z < p.nc; ++z) acc = cadd(acc, dapart[((long long)b * p.H + h) * p.nc + z]);
  dA[h] = acc;
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
static size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct FwdLayout {
  size_t acs, total;
};
struct BwdLayout {
  size_t acs, dsbuf, mbuf, dgbuf, rowpart, colpart, rowcpart, upart, gpart, dapart, total;
};

// The first 256 bytes of every workspace are the status area (device error word at offset 0).
constexpr size_t kStatusBytes = 256;

static FwdLayout fwd_layout(const Problem& p) {
  FwdLayout L;
  size_t off = kStatusBytes;
  L.acs = off; off += align256(sizeof(float2) * (size_t)p.Bsz * p.H * p.Tp());
  L.total = off;
  return L;
}

static int scan_blocks_for(const Problem& p) { return (int)((p.N * (long long)p.D + 255) / 256); }

static BwdLayout bwd_layout(const Problem& p) {
  BwdLayout L;
  const size_t bhz = (size_t)p.Bsz * p.H * p.nc;
  const size_t tC = (size_t)tiles(p.C), tN = (size_t)tiles(p.N);
  size_t off = kStatusBytes;
  L.acs = off;      off += align256(sizeof(float2) * (size_t)p.Bsz * p.H * p.Tp());
  L.dsbuf = off;    off += align256(sizeof(float2) * bhz * p.N * p.D);
  L.mbuf = off;     off += align256(sizeof(float2) * bhz * p.C * p.C);
  L.dgbuf = off;    off += align256(sizeof(float2) * bhz * p.C * p.C);
  L.rowpart = off;  off += align256(sizeof(float2) * bhz * p.C * tC);
  L.colpart = off;  off += align256(sizeof(float2) * bhz * p.C * tC);
  L.rowcpart = off; off += align256(sizeof(float2) * bhz * p.C * tN);
  L.upart = off;    off += align256(sizeof(float2) * bhz * p.C * tN);
  L.gpart = off;    off += align256(sizeof(float2) * bhz * scan_blocks_for(p));
  L.dapart = off;   off += align256(sizeof(float2) * bhz);
  L.total = off;
  return L;
}

size_t states_bytes(const Problem& p) {
  return sizeof(float2) * (size_t)p.Bsz * p.H * p.nc * p.N * p.D;
}
size_t fwd_workspace_bytes(const Problem& p) { return fwd_layout(p).total; }
size_t bwd_workspace_bytes(const Problem& p) { return bwd_layout(p).total; }

static int launch_ok() { return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH; }

int run_fwd(const Problem& p, float* y, void* states, void* ws, cudaStream_t st) {
  const FwdLayout L = fwd_layout(p);
  float2* acs = reinterpret_cast<float2*>(static_cast<char*>(ws) + L.acs);
  float2* S = static_cast<float2*>(states);
  const long long nbhz = (long long)p.Bsz * p.H * p.nc;
  if (cudaMemsetAsync(ws, 0, kStatusBytes, st) != cudaSuccess) return M3SSD_ERR_LAUNCH;
  k_chunk_cumsum<<<(unsigned)((nbhz + 127) / 128), 128, 0, st>>>(p, acs);
  const dim3 g_np((unsigned)(tiles(p.N) * tiles(p.D)), (unsigned)p.nc, (unsigned)(p.Bsz * p.H));
  (p.x_complex ? k_fwd_state<true> : k_fwd_state<false>)<<<g_np, NT, 0, st>>>(p, acs, S);
  const dim3 g_scan((unsigned)scan_blocks_for(p), (unsigned)(p.Bsz * p.H));
  k_fwd_scan<<<g_scan, 256, 0, st>>>(p, acs, S);
  const dim3 g_lp((unsigned)(tiles(p.C) * ((tiles(p.D) + kOutTiles - 1) / kOutTiles)),
                  (unsigned)p.nc, (unsigned)(p.Bsz * p.H));
  (p.x_complex ? k_fwd_out<true> : k_fwd_out<false>)<<<g_lp, NT, 0, st>>>(p, acs, S, y);
  return launch_ok();
}

int run_bwd(const Problem& p, const float* dy, const long long dys[4], const void* states,
            void* dx, float2* dA, float2* dB, float2* dC, float* ddt, void* ws, cudaStream_t st) {
  const BwdLayout L = bwd_layout(p);
  char* base = static_cast<char*>(ws);
  float2* acs = reinterpret_cast<float2*>(base + L.acs);
  BwdBufs w;
  float2* dsbuf = reinterpret_cast<float2*>(base + L.dsbuf);
  w.mbuf = reinterpret_cast<float2*>(base + L.mbuf);
  w.dgbuf = reinterpret_cast<float2*>(base + L.dgbuf);
  w.rowpart = reinterpret_cast<float2*>(base + L.rowpart);
  w.colpart = reinterpret_cast<float2*>(base + L.colpart);
  w.rowcpart = reinterpret_cast<float2*>(base + L.rowcpart);
  w.upart = reinterpret_cast<float2*>(base + L.upart);
  w.gpart = reinterpret_cast<float2*>(base + L.gpart);
  w.dapart = reinterpret_cast<float2*>(base + L.dapart);
  Grad g;
  g.dy = dy;
  for (int i = 0; i < 4; ++i) g.dys[i] = dys[i];
  const float2* S = static_cast<const float2*>(states);
  const long long nbhz = (long long)p.Bsz * p.H * p.nc;
  const unsigned bh = (unsigned)(p.Bsz * p.H), nc = (unsigned)p.nc;
  if (cudaMemsetAsync(ws, 0, kStatusBytes, st) != cudaSuccess) return M3SSD_ERR_LAUNCH;
  k_chunk_cumsum<<<(unsigned)((nbhz + 127) / 128), 128, 0, st>>>(p, acs);
  k_bwd_q<<<dim3((unsigned)(tiles(p.N) * tiles(p.D)), nc, bh), NT, 0, st>>>(p, g, acs, dsbuf);
  const int sb = scan_blocks_for(p);
  k_bwd_scan<<<dim3((unsigned)sb, bh), 256, 0, st>>>(p, acs, S, dsbuf, w.gpart);
  (p.x_complex ? k_bwd_mm<true> : k_bwd_mm<false>)<<<dim3((unsigned)(tiles(p.C) * tiles(p.C)), nc, bh), NT, 0, st>>>(p, g, acs, w);
  k_bwd_dc<<<dim3((unsigned)(tiles(p.C) * tiles(p.N)), nc, bh), NT, 0, st>>>(p, g, acs, S, w, dC);
  (p.x_complex ? k_bwd_db<true> : k_bwd_db<false>)<<<dim3((unsigned)(tiles(p.C) * tiles(p.N)), nc, bh), NT, 0, st>>>(p, acs, dsbuf, w, dB);
  (p.x_complex ? k_bwd_dx<true> : k_bwd_dx<false>)<<<dim3((unsigned)(tiles(p.C) * tiles(p.D)), nc, bh), NT, 0, st>>>(p, g, acs, dsbuf, w, dx);
  k_bwd_da<<<(unsigned)((nbhz + 127) / 128), 128, 0, st>>>(p, acs, w, sb, ddt);
  k_bwd_dA<<<(unsigned)((p.H + 127) / 128), 128, 0, st>>>(p, w.dapart, dA);
  return launch_ok();
}

}  // namespace simt
}  // namespace m3ssd

// Long sequences, few of them: the tensor-core path run as G chains per sequence.
//
// The one-pass kernels hand the state from chunk to chunk of a sequence (forward: H_z -> H_{z+1};
// backward: dS_z -> dS_{z-1}); each hand-off costs a few microseconds of latency, so a sequence of
// nc chunks takes at least nc hand-offs whatever the work. At B4 L16384 with two heads per GPU
// (8 sequences of 256 chunks) that chain, not HBM, sets the time. Here each sequence's chunks run
// as G chains of nc / G chunks, in two passes:
//
//   forward   pass 1: the tensor-core forward, every chain from a zero entry state; its end state
//                     L_s goes to scratch (its y is overwritten by pass 2)
//             chain:  S_0 = h0 (or 0), S_{s+1} = D_s S_s + L_s over the segments (D_s = the
//                     segment's total decay, the product of its chunks' e^Gamma), S_G = final state
//             pass 2: the tensor-core forward, every chain from its true entry state S_s: y and
//                     the chunk-entry states
//   backward  pass 1: every chain's entry-state gradient P_s from a zero end-state gradient
//                     (k_chain_bwd_pass1_tiled / k_chain_bwd_pass1, CUDA cores, one CTA per
//                     chain: only the carry)
//             chain:  dS_G = dhT (or 0), dS_s = P_{s+1} + conj(D_{s+1}) dS_{s+1} going back, and
//                     each segment's last-chunk d Sigma term <dS_s, conj(S_{s+1})>
//             pass 2: the tensor-core backward, every chain from its true end-state gradient
//
// Every chain's algebra is the reference's recurrence split at segment boundaries
// (s_t = e^{a_t} s_{t-1} + B_t x_t^T is linear in s), so the result equals the one-pass path's
// up to rounding.
#include <cuda_runtime.h>

#include "tc_path.h"

namespace m3ssd {
namespace tc {

namespace {

constexpr int kMaxChains = 64;     // chains per sequence
constexpr int kStateElems = 64 * 64;  // complex elements of one state

size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }

// scratch after the one-pass workspace: two per-chain state arrays (B*H*G states each)
size_t chain_states_bytes(const Problem& p, int G) {
  return (size_t)p.Bsz * p.H * G * kStateElems * sizeof(float2);
}

// D_s for s = 0..G-1 of sequence bh into shared memory (threads s < G)
__device__ __forceinline__ void segment_decays(const ChunkRec* recs, int bh, int nc, int G,
                                               float2* D) {
  const int seg = nc / G;
  for (int s = threadIdx.x; s < G; s += blockDim.x) {
    float2 d = make_float2(1.f, 0.f);
    const ChunkRec* r = recs + (long long)bh * nc + (long long)s * seg;
    for (int j = 0; j < seg; ++j) {
      const float2 g = r[j].g;
      d = make_float2(d.x * g.x - d.y * g.y, d.x * g.y + d.y * g.x);
    }
    D[s] = d;
  }
  __syncthreads();
}

// forward chain over the segments of one sequence, one complex element per thread
__global__ void __launch_bounds__(256) k_chain_fwd(const ChunkRec* __restrict__ recs, int nc, int G,
                                                   const float2* __restrict__ h0,
                                                   const float2* __restrict__ L,
                                                   float2* __restrict__ S, float2* __restrict__ hT) {
  __shared__ float2 D[kMaxChains];
  const int bh = blockIdx.x;
  segment_decays(recs, bh, nc, G, D);
  const int e = blockIdx.y * 256 + threadIdx.x;
  float2 s = h0 != nullptr ? h0[(long long)bh * kStateElems + e] : make_float2(0.f, 0.f);
  for (int k = 0; k < G; ++k) {
    const long long i = ((long long)bh * G + k) * kStateElems + e;
    S[i] = s;
    const float2 l = L[i], d = D[k];
    s = make_float2(d.x * s.x - d.y * s.y + l.x, d.x * s.y + d.y * s.x + l.y);
  }
  if (hT != nullptr) hT[(long long)bh * kStateElems + e] = s;
}

// backward chain: end-state gradients of every segment from the entry-state gradients of pass 1
__global__ void __launch_bounds__(256) k_chain_bwd(const ChunkRec* __restrict__ recs, int nc, int G,
                                                   const float2* __restrict__ dhT,
                                                   const float2* __restrict__ P,
                                                   float2* __restrict__ dE, float2* __restrict__ dh0) {
  __shared__ float2 D[kMaxChains];
  const int bh = blockIdx.x;
  segment_decays(recs, bh, nc, G, D);
  const int e = blockIdx.y * 256 + threadIdx.x;
  float2 g = dhT != nullptr ? dhT[(long long)bh * kStateElems + e] : make_float2(0.f, 0.f);
  for (int k = G - 1; k >= 0; --k) {
    const long long i = ((long long)bh * G + k) * kStateElems + e;
    dE[i] = g;
    const float2 q = P[i], d = D[k];  // dS at the entry of segment k = P_k + conj(D_k) dS_end
    g = make_float2(q.x + d.x * g.x + d.y * g.y, q.y + d.x * g.y - d.y * g.x);
  }
  if (dh0 != nullptr) dh0[(long long)bh * kStateElems + e] = g;
}

// <dE_s, conj(S_{s+1})> per chain: the d Sigma term of a segment's last position from its end
// state. S_{s+1} is the chunk-entry state tile of chunk (s + 1) * seg in `states` (the forward's
// thread-major layout: float4 f holds, of row p = 16 (w mod 4) + (l mod 16), the complex columns
// n0, n0 + 1 with n0 = 32 (w / 4) + 16 (l / 16) + 8 (f / 1024) + 2 ((f / 256) mod 4), where
// t = f mod 256, w = t / 32, l = t mod 32); the last segment's end state is the final state hT
// ((n, p) layout), or absent when no end-state gradient comes in (then its dE is zero).
__global__ void __launch_bounds__(256) k_chain_dgam(const float* __restrict__ states, int nc, int G,
                                                    const float2* __restrict__ dE,
                                                    const float2* __restrict__ hT,
                                                    float2* __restrict__ dgam) {
  __shared__ float2 red[8];
  const int sg = blockIdx.x, bh = sg / G, s = sg - bh * G, seg = nc / G;
  const float2* de = dE + (long long)sg * kStateElems;
  float2 acc = make_float2(0.f, 0.f);
  if (s + 1 < G) {
    const float4* tile =
        reinterpret_cast<const float4*>(states + ((long long)bh * nc + (long long)(s + 1) * seg) * 64 * 128);
    for (int f = threadIdx.x; f < 2048; f += 256) {
      const int t = f & 255, w = t >> 5, l = t & 31;
      const int prow = 16 * (w & 3) + (l & 15);
      const int n0 = 32 * (w >> 2) + 16 * (l >> 4) + 8 * (f >> 10) + 2 * ((f >> 8) & 3);
      const float4 h = tile[f];
      const float2 a = de[n0 * 64 + prow], b = de[(n0 + 1) * 64 + prow];
      acc.x += a.x * h.x + a.y * h.y + b.x * h.z + b.y * h.w;
      acc.y += a.y * h.x - a.x * h.y + b.y * h.z - b.x * h.w;
    }
  } else if (hT != nullptr) {
    const float2* hh = hT + (long long)bh * kStateElems;
    for (int e = threadIdx.x; e < kStateElems; e += 256) {
      const float2 a = de[e], h = hh[e];
      acc.x += a.x * h.x + a.y * h.y;
      acc.y += a.y * h.x - a.x * h.y;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
    acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float2 t = red[0];
    for (int w = 1; w < 8; ++w) {
      t.x += red[w].x;
      t.y += red[w].y;
    }
    dgam[sg] = t;
  }
}

// First backward pass of the chained form on CUDA cores, one CTA per chain, its chunks in reverse,
// the chain's carry in registers: G <- conj(e^Gamma) G + sum_l w_l[n] dy_l[p] with
// w_l = conj(C_l e^{Sigma_l}), from zero; the chain's entry-state gradient goes to
// out[bh * G + segment] in the (n, p) layout of the state arguments. Only the carry of a chunk is
// needed, not its gradients, so this replaces a full tensor-core backward pass (~80 ns per chunk
// of throughput) by one 64 x 64 x 64 complex-by-real product per chunk (~35 ns). Each thread owns
// a 4 n x 4 p block of the carry. (The same form for the forward's end states measured slower
// than the tensor-core forward pass, whose chunks cost ~43 ns: along a chain each chunk here
// takes ~8 us.)
struct CarryPassArgs {
  const float2* bc;  // C, interleaved complex or planar (see Problem)
  long long bcs[4];
  int planar;
  const void* dy;
  long long dys[4];
  int dy_bf16;
  const ChunkRec* recs;
  int T, H, nc, G;
};

__global__ void __launch_bounds__(256) k_chain_bwd_pass1(const CarryPassArgs a,
                                                         float2* __restrict__ out) {
  __shared__ __align__(16) float2 sW[64][64];
  __shared__ __align__(16) float sR[64][64];
  const int tid = threadIdx.x;
  const int sg = blockIdx.x, bh = sg / a.G, sgm = sg - bh * a.G, seg = a.nc / a.G;
  const int b = bh / a.H, h = bh - b * a.H;
  const int n0 = 4 * (tid >> 4), p0 = 4 * (tid & 15);
  float2 st[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) st[i][k] = cz();
  for (int it = 0; it < seg; ++it) {
    const int z = sgm * seg + seg - 1 - it;
    const ChunkRec* rec = a.recs + (long long)bh * a.nc + z;
    __syncthreads();  // the previous chunk's tiles are no longer read
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int e = tid + 256 * i, l = e >> 6, c = e & 63, t = z * 64 + l;
      float2 v = cz();
      float r = 0.f;
      if (t < a.T) {
        if (a.planar) {
          const float* f = reinterpret_cast<const float*>(a.bc) + b * a.bcs[0] + t * a.bcs[1] +
                           h * a.bcs[2] + c * a.bcs[3];
          v = make_float2(f[0], f[(long long)a.H * 64]);
        } else {
          v = a.bc[b * a.bcs[0] + t * a.bcs[1] + h * a.bcs[2] + c * a.bcs[3]];
        }
        const long long o = b * a.dys[0] + t * a.dys[1] + h * a.dys[2] + c * a.dys[3];
        r = a.dy_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.dy)[o])
                      : static_cast<const float*>(a.dy)[o];
      }
      // conj(C e^{Sigma_l}) = conj(C) el conj(cis)
      const float2 cs = rec->cis[l];
      sW[l][c] = cmul(cconj(v), make_float2(rec->el[l] * cs.x, -rec->el[l] * cs.y));
      sR[l][c] = r;
    }
    __syncthreads();
    float2 acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[i][k] = cz();
#pragma unroll 4
    for (int l = 0; l < 64; ++l) {
      const float4 w01 = *reinterpret_cast<const float4*>(&sW[l][n0]);
      const float4 w23 = *reinterpret_cast<const float4*>(&sW[l][n0 + 2]);
      const float4 r4 = *reinterpret_cast<const float4*>(&sR[l][p0]);
      const float2 w[4] = {make_float2(w01.x, w01.y), make_float2(w01.z, w01.w),
                           make_float2(w23.x, w23.y), make_float2(w23.z, w23.w)};
      const float r[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[i][k].x = fmaf(w[i].x, r[k], acc[i][k].x);
          acc[i][k].y = fmaf(w[i].y, r[k], acc[i][k].y);
        }
    }
    const float2 f = cconj(rec->g);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) st[i][k] = cadd(cmul(f, st[i][k]), acc[i][k]);
  }
  float2* dst = out + (long long)sg * kStateElems;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4* row = reinterpret_cast<float4*>(dst + (n0 + i) * 64 + p0);
    row[0] = make_float4(st[i][0].x, st[i][0].y, st[i][1].x, st[i][1].y);
    row[1] = make_float4(st[i][2].x, st[i][2].y, st[i][3].x, st[i][3].y);
  }
}

// The same carry pass with the next chunk's C and dy tiles copied into shared memory (cp.async,
// 16 bytes per copy) while the current chunk is multiplied, and the decay applied to the landed C
// tile in place. For interleaved C with a contiguous state dimension and fp32 dy with a contiguous
// head dimension, rows 16-byte aligned (carry_tiled_ok); other layouts take k_chain_bwd_pass1.
constexpr int kCarryTiledSmem = 2 * 64 * 64 * ((int)sizeof(float2) + (int)sizeof(float));

__device__ __forceinline__ void cp_async16(float* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

__global__ void __launch_bounds__(256) k_chain_bwd_pass1_tiled(const CarryPassArgs a,
                                                               float2* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  float2* sC = reinterpret_cast<float2*>(smem);                      // [2][64 l][64 n]
  float* sD = reinterpret_cast<float*>(smem + 2 * 64 * 64 * sizeof(float2));  // [2][64 l][64 p]
  const int tid = threadIdx.x;
  const int sg = blockIdx.x, bh = sg / a.G, sgm = sg - bh * a.G, seg = a.nc / a.G;
  const int b = bh / a.H, h = bh - b * a.H;
  const int n0 = 4 * (tid >> 4), p0 = 4 * (tid & 15);
  const float* dyf = static_cast<const float*>(a.dy);
  // copies of chunk `it` (chunks in reverse) into buffer `buf`; rows past T are zero-filled
  auto issue = [&](int it, int buf) {
    const int z = sgm * seg + seg - 1 - it;
    float* cdst = reinterpret_cast<float*>(sC + buf * 4096);
    float* ddst = sD + buf * 4096;
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // C: 64 rows x 32 copies of 2 complex
      const int e = tid + 256 * i, l = e >> 5, q = e & 31, t = z * 64 + l;
      float* d = cdst + l * 128 + 4 * q;
      if (t < a.T)
        cp_async16(d, a.bc + b * a.bcs[0] + t * a.bcs[1] + h * a.bcs[2] + 2 * q);
      else
        *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // dy: 64 rows x 16 copies of 4 floats
      const int e = tid + 256 * i, l = e >> 4, q = e & 15, t = z * 64 + l;
      float* d = ddst + l * 64 + 4 * q;
      if (t < a.T)
        cp_async16(d, dyf + b * a.dys[0] + t * a.dys[1] + h * a.dys[2] + 4 * q);
      else
        *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  float2 st[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) st[i][k] = cz();
  issue(0, 0);
  for (int it = 0; it < seg; ++it) {
    const int buf = it & 1;
    if (it + 1 < seg) {
      issue(it + 1, buf ^ 1);  // that buffer was last read before the previous iteration's barrier
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // every thread's copies of this chunk have landed
    const int z = sgm * seg + seg - 1 - it;
    const ChunkRec* rec = a.recs + (long long)bh * a.nc + z;
    float2* cb = sC + buf * 4096;
    const float* db = sD + buf * 4096;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {  // conj(C e^{Sigma_l}) = conj(C) el conj(cis), in place
      const int e = tid + 256 * i, l = e >> 6;
      const float2 cs = rec->cis[l];
      const float el = rec->el[l];
      cb[e] = cmul(cconj(cb[e]), make_float2(el * cs.x, -el * cs.y));
    }
    __syncthreads();
    float2 acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[i][k] = cz();
#pragma unroll 4
    for (int l = 0; l < 64; ++l) {
      const float4 w01 = *reinterpret_cast<const float4*>(cb + l * 64 + n0);
      const float4 w23 = *reinterpret_cast<const float4*>(cb + l * 64 + n0 + 2);
      const float4 r4 = *reinterpret_cast<const float4*>(db + l * 64 + p0);
      const float2 w[4] = {make_float2(w01.x, w01.y), make_float2(w01.z, w01.w),
                           make_float2(w23.x, w23.y), make_float2(w23.z, w23.w)};
      const float r[4] = {r4.x, r4.y, r4.z, r4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          acc[i][k].x = fmaf(w[i].x, r[k], acc[i][k].x);
          acc[i][k].y = fmaf(w[i].y, r[k], acc[i][k].y);
        }
    }
    const float2 f = cconj(rec->g);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int k = 0; k < 4; ++k) st[i][k] = cadd(cmul(f, st[i][k]), acc[i][k]);
    __syncthreads();  // this buffer is refilled by the next iteration's copies
  }
  float2* dst = out + (long long)sg * kStateElems;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float4* row = reinterpret_cast<float4*>(dst + (n0 + i) * 64 + p0);
    row[0] = make_float4(st[i][0].x, st[i][0].y, st[i][1].x, st[i][1].y);
    row[1] = make_float4(st[i][2].x, st[i][2].y, st[i][3].x, st[i][3].y);
  }
}

// 16-byte copies of whole rows: interleaved C with a contiguous state dimension, fp32 dy with a
// contiguous head dimension, every row start 16-byte aligned
bool carry_tiled_ok(const Problem& p, const void* dy, const long long dys[4]) {
  if (p.bc_planar || p.y_bf16) return false;
  if (p.cs[3] != 1 || p.cs[0] % 2 || p.cs[1] % 2 || p.cs[2] % 2) return false;
  if (reinterpret_cast<uintptr_t>(p.Cm) % 16 || reinterpret_cast<uintptr_t>(dy) % 16) return false;
  return dys[3] == 1 && dys[0] % 4 == 0 && dys[1] % 4 == 0 && dys[2] % 4 == 0;
}

CarryPassArgs carry_pass_args(const Problem& p, const void* dy, const long long dys[4],
                              const ChunkRec* recs, int G) {
  CarryPassArgs a{};
  a.bc = p.Cm;
  for (int i = 0; i < 4; ++i) {
    a.bcs[i] = p.cs[i];
    a.dys[i] = dys[i];
  }
  a.planar = p.bc_planar;
  a.dy = dy;
  a.dy_bf16 = p.y_bf16;
  a.recs = recs;
  a.T = p.T;
  a.H = p.H;
  a.nc = (p.T + 63) / 64;
  a.G = G;
  return a;
}

}  // namespace

// Time model of one pass (microseconds, fitted to one-pass runs on B200): a ticket (one chunk of
// one sequence) costs `ticket` of throughput with the GPU full, a hand-off `hop` of latency on its
// chain, and a pass takes about the larger of the two plus a fifth of the smaller (B16 L2048 H16:
// work-bound; B4 L16384 with 2 or 16 heads: chain-bound). The chained form runs two passes over
// chains of nc / G chunks plus the segment chain. G = 1 unless chains are clearly faster.
int chains_for(const Problem& p, bool backward) {
  if (p.x_complex) return 1;  // complex x runs as two one-pass real passes (tc_complex.cu)
  const int nc = (p.T + 63) / 64;
  const double bh = (double)p.Bsz * p.H;
  const double ticket = backward ? 0.070 : 0.039, hop = backward ? 5.2 : 4.3;
  const double work = bh * nc * ticket;
  auto pass = [&](double chain) {
    return work > chain ? work + 0.2 * chain : chain + 0.2 * work;
  };
  const double one_pass = pass(nc * hop);
  double best = one_pass;
  int best_g = 1;
  for (int G = 2; G <= kMaxChains && nc / G >= 2; G *= 2) {
    if (nc % G != 0) break;  // a larger power of two does not divide nc either
    // first pass (tc_chain_state.cu: each chunk's two tiles, 48 KB, read at ~45% of HBM
    // bandwidth, ~17 ns of throughput per chunk, ~4.5 us per chunk along a chain), the
    // tensor-core pass, the chains
    const double first = fmax(bh * nc * 0.017, (double)(nc / G) * 4.5) + 5.0;
    const double est = first + pass((double)(nc / G) * hop) + 10.0 + 0.5 * G;
    if (est < best) {
      best = est;
      best_g = G;
    }
  }
  return best < 0.8 * one_pass ? best_g : 1;
}

size_t fwd_chains_workspace_bytes(const Problem& p, int G) {
  return al256(fwd_workspace_bytes(p)) + 2 * chain_states_bytes(p, G);
}

size_t bwd_chains_workspace_bytes(const Problem& p, int G) {
  return al256(bwd_workspace_bytes(p, G)) + 2 * chain_states_bytes(p, G) +
         al256((size_t)p.Bsz * p.H * G * sizeof(float2));
}

int run_fwd_chains(const Problem& p, void* y, void* states, void* ws, cudaStream_t st,
                   const void* h0, void* hT, int G) {
  const int nc = (p.T + 63) / 64;
  if (G < 2 || G > kMaxChains || nc % G != 0) return M3SSD_ERR_SHAPE;
  char* base = static_cast<char*>(ws);
  float2* L = reinterpret_cast<float2*>(base + al256(fwd_workspace_bytes(p)));
  float2* S = L + (size_t)p.Bsz * p.H * G * kStateElems;
  ChunkRec* recs = reinterpret_cast<ChunkRec*>(static_cast<char*>(states) + states_h_bytes(p));
  const long long* xs = p.xs;
  if (chain_state_tc_ok(p, true, p.x, xs, 0)) {
    // first pass as one GEMM per chain (tc_chain_state.cu), after the decay records
    if (cudaMemsetAsync(ws, 0, 4, st) != cudaSuccess) return M3SSD_ERR_LAUNCH;
    int rc = run_chunk_prep(p, recs, st);
    if (rc != M3SSD_OK) return rc;
    rc = run_chain_state(p, true, p.x, xs, 0, recs, G, L, static_cast<uint32_t*>(ws), st);
    if (rc != M3SSD_OK) return rc;
  } else {
    // first pass as a tensor-core forward from zero entry states (its y is rewritten below)
    const int rc = run_fwd(p, y, states, ws, st, nullptr, L, G, true, true);
    if (rc != M3SSD_OK) return rc;
  }
  k_chain_fwd<<<dim3(p.Bsz * p.H, kStateElems / 256), 256, 0, st>>>(
      recs, nc, G, static_cast<const float2*>(h0), L, S, static_cast<float2*>(hT));
  if (cudaGetLastError() != cudaSuccess) return M3SSD_ERR_LAUNCH;
  return run_fwd(p, y, states, ws, st, S, nullptr, G, false, false);
}

int run_bwd_chains(const Problem& p, const void* dy, const long long dys[4], const void* states,
                   const BwdOut& out, void* ws, cudaStream_t st, const void* hT, const void* dhT,
                   void* dh0, int G) {
  const int nc = (p.T + 63) / 64;
  if (G < 2 || G > kMaxChains || nc % G != 0) return M3SSD_ERR_SHAPE;
  if ((dhT != nullptr) != (hT != nullptr)) return M3SSD_ERR_NULL;
  char* base = static_cast<char*>(ws);
  float2* P = reinterpret_cast<float2*>(base + al256(bwd_workspace_bytes(p, G)));
  float2* dE = P + (size_t)p.Bsz * p.H * G * kStateElems;
  float2* dgam = dE + (size_t)p.Bsz * p.H * G * kStateElems;
  const ChunkRec* recs =
      reinterpret_cast<const ChunkRec*>(static_cast<const char*>(states) + states_h_bytes(p));
  const CarryPassArgs ca = carry_pass_args(p, dy, dys, recs, G);
  // the first pass reports into the status word, which the tensor-core pass below then keeps
  if (cudaMemsetAsync(ws, 0, 4, st) != cudaSuccess) return M3SSD_ERR_LAUNCH;
  if (chain_state_tc_ok(p, false, dy, dys, p.y_bf16)) {
    const int rc =
        run_chain_state(p, false, dy, dys, p.y_bf16, recs, G, P, static_cast<uint32_t*>(ws), st);
    if (rc != M3SSD_OK) return rc;
  } else if (carry_tiled_ok(p, dy, dys)) {
    if (!ensure_smem_attr(reinterpret_cast<const void*>(k_chain_bwd_pass1_tiled),
                          (int)kCarryTiledSmem))
      return M3SSD_ERR_LAUNCH;
    k_chain_bwd_pass1_tiled<<<p.Bsz * p.H * G, 256, kCarryTiledSmem, st>>>(ca, P);
  } else {
    k_chain_bwd_pass1<<<p.Bsz * p.H * G, 256, 0, st>>>(ca, P);
  }
  k_chain_bwd<<<dim3(p.Bsz * p.H, kStateElems / 256), 256, 0, st>>>(
      recs, nc, G, static_cast<const float2*>(dhT), P, dE, static_cast<float2*>(dh0));
  k_chain_dgam<<<p.Bsz * p.H * G, 256, 0, st>>>(static_cast<const float*>(states), nc, G, dE,
                                                static_cast<const float2*>(hT), dgam);
  if (cudaGetLastError() != cudaSuccess) return M3SSD_ERR_LAUNCH;
  return run_bwd(p, dy, dys, states, out, ws, st, nullptr, dE, nullptr, G, dgam, false);
}

}  // namespace tc
}  // namespace m3ssd

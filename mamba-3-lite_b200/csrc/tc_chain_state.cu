// First passes of the chained form (tc_long.cu) on the tensor cores: a chain's end state from a
// zero entry state (forward) and its entry-state gradient from a zero end-state gradient
// (backward), one CTA per chain.
//
// Both are a sum over the chain's positions t of a complex column times a real row:
//   forward   L[n][p] = sum_t (d_z cis(theta_Gamma,z) exp(rho_Gamma,z - rho_l) conj(cis theta_l)
//                                B_t[n]) x_t[p]
//             with d_z = prod over the chain's later chunks of e^Gamma (the carry H_{z+1} =
//             e^Gamma H_z + cis(theta_Gamma) S~_z unrolled from H = 0);
//   backward  P[n][p] = sum_t (c_z conj(C_t[n] exp(Sigma_l))) dy_t[p]
//             with c_z = prod over the chain's earlier chunks of conj(e^Gamma) (the carry
//             dS_{z-1} = Q_z + conj(e^Gamma) dS_z unrolled from dS = 0),
// l the position within chunk z. So each chain's state is one GEMM with K = the chain's
// positions: D[p][n re/im] = sum_t R_t[p] W_t[n], R = x or dy (real), W the complex operand with
// its per-position factor folded in. Operands are split-bf16 as in the chunk kernels (R's hi and
// lo rows stacked in groups of 16 over M = 128, W's hi and lo as two passes), both MN-major in
// 128-byte swizzled tiles, fp32 accumulation in 128 TMEM columns. The next chunk's rows are
// loaded into registers while a chunk's 8 MMAs run; operand tiles are double buffered. The CUDA-core carry pass and the forward's first tensor-core pass did the same work
// with a chunk-by-chunk carry (tc_long.cu).
#include <cuda.h>
#include <cuda_runtime.h>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"
#include "tc_path.h"
#include "tc_trace.cuh"

namespace m3ssd {
namespace tc {

M3_TRACE_DEFINE(m3ssd_trace_set_chain_state)

namespace {

constexpr int kThreads = 256;
constexpr uint32_t kTile = 16384;                  // one operand tile: 2 x 64 values x 64 rows bf16
constexpr uint32_t kBufBytes = 3 * kTile;          // R stacked | W hi | W lo
constexpr uint32_t kSmemBytes = 2 * kBufBytes + 1024 + 1024;
constexpr uint32_t kTmemCols = 128;

struct ChainStateArgs {
  const float2* W;  // B (forward) or C (backward): interleaved complex (B, T, H, 64), or planar
  long long ws[4];  // its strides in complex elements (planar: in floats)
  int w_planar;     // planar: real parts at W, imaginary parts H * 64 floats further
  const void* R;    // x (forward, fp32) or dy (backward, fp32 or bf16): (B, T, H, 64)
  long long rs[4];  // its strides in elements
  int r_bf16;
  const ChunkRec* recs;
  int T, H, nc, G;
  uint32_t* err;
};

// byte offset of 16-byte chunk `c` (0..15 over the two 64-value blocks) in row t of a tile
__device__ __forceinline__ uint32_t tile_off(uint32_t t, uint32_t c) {
  return (c >> 3) * 8192u + t * 128u + (((c & 7u) ^ (t & 7u)) << 4);
}

}  // namespace

template <bool kFwd>
__global__ void __launch_bounds__(kThreads, 2)
    k_chain_state_tc(const ChainStateArgs a, float2* __restrict__ out) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * kBufBytes);  // one per buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + 2 * kBufBytes + 64);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sg = blockIdx.x, bh = sg / a.G, sgm = sg - bh * a.G, seg = a.nc / a.G;
  const int b = bh / a.H, h = bh - b * a.H;
  // this thread's row of a chunk and its 16 values: complex n (W) or p (R) = 16 g .. 16 g + 15
  const int tl = tid >> 2, g = tid & 3;

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) M3_TRACE(63, 0);

  // chunk of iteration `it`: forward from the chain's last chunk back, backward from its first
  auto chunk_of = [&](int it) { return sgm * seg + (kFwd ? seg - 1 - it : it); };
  struct Rows {
    float4 w[8];      // 16 complex of W
    float r[16];      // 16 values of R
    float2 cs, gz;    // the chunk record's cis(theta_l) of this row and e^Gamma
    float2 ct;        // cis(theta_Gamma) (forward)
    float dl;         // exp(rho_Gamma - rho_l) (forward) or exp(rho_l) (backward)
  };
  auto load = [&](int z, Rows& d) {
    const ChunkRec* rec = a.recs + (long long)bh * a.nc + z;
    d.cs = __ldg(&rec->cis[tl]);
    d.gz = __ldg(&rec->g);
    d.ct = kFwd ? __ldg(&rec->ct) : make_float2(0.f, 0.f);
    d.dl = kFwd ? __ldg(&rec->dec[tl]) : __ldg(&rec->el[tl]);
    const int t = z * 64 + tl;
    if (t >= a.T) {
#pragma unroll
      for (int i = 0; i < 8; ++i) d.w[i] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 16; ++i) d.r[i] = 0.f;
      return;
    }
    if (a.w_planar) {  // the same (Re, Im) pairs as the interleaved layout, so the same results
      const float* w = reinterpret_cast<const float*>(a.W) + b * a.ws[0] + (long long)t * a.ws[1] +
                       h * a.ws[2] + 16 * g;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 re = __ldg(reinterpret_cast<const float4*>(w) + i);
        const float4 im = __ldg(reinterpret_cast<const float4*>(w + (long long)a.H * 64) + i);
        d.w[2 * i] = make_float4(re.x, im.x, re.y, im.y);
        d.w[2 * i + 1] = make_float4(re.z, im.z, re.w, im.w);
      }
    } else {
      const float2* w = a.W + b * a.ws[0] + (long long)t * a.ws[1] + h * a.ws[2] + 16 * g;
#pragma unroll
      for (int i = 0; i < 8; ++i) d.w[i] = __ldg(reinterpret_cast<const float4*>(w) + i);
    }
    const long long ro = b * a.rs[0] + (long long)t * a.rs[1] + h * a.rs[2] + 16 * g;
    if (a.r_bf16) {
      const uint4* r = reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.R) + ro);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint4 q = __ldg(r + i);
        const uint32_t u[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          d.r[8 * i + 2 * k] = __uint_as_float(u[k] << 16);
          d.r[8 * i + 2 * k + 1] = __uint_as_float(u[k] & 0xFFFF0000u);
        }
      }
    } else {
      const float4* r = reinterpret_cast<const float4*>(static_cast<const float*>(a.R) + ro);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 q = __ldg(r + i);
        d.r[4 * i] = q.x;
        d.r[4 * i + 1] = q.y;
        d.r[4 * i + 2] = q.z;
        d.r[4 * i + 3] = q.w;
      }
    }
  };

  float2 run = make_float2(1.f, 0.f);  // the running decay product (d_z or c_z)
  // chunk `it` from the rows in `cur`, which then takes the rows of chunk it + 1
  auto step = [&](int it, Rows& cur) {
    const uint32_t buf = (uint32_t)it & 1u;
    const uint32_t base = sb + buf * kBufBytes;
    // the MMAs of two chunks ago have read this buffer
    if (warp == 0) M3_TRACE(it, 0);
    if (it >= 2) mbar_wait(&bar[buf], (uint32_t)((it >> 1) - 1) & 1u, a.err, kErrMmaWait);
    if (warp == 0) M3_TRACE(it, 1);
    {
      // this position's complex factor; the running product is the same in every thread
      const float2 cs = cur.cs;
      float2 f;
      if constexpr (kFwd) {  // W = B f,  f = d_z cis(theta_Gamma) exp(rho_Gamma - rho_l) conj(cis_l)
        const float2 ct = cur.ct, dz = run;
        const float2 u = make_float2(dz.x * ct.x - dz.y * ct.y, dz.x * ct.y + dz.y * ct.x);
        const float d = cur.dl;
        f = make_float2(d * (u.x * cs.x + u.y * cs.y), d * (u.y * cs.x - u.x * cs.y));
      } else {  // W = conj(C) f,  f = c_z exp(rho_l) conj(cis_l)
        const float e = cur.dl;
        const float2 c = run;
        f = make_float2(e * (c.x * cs.x + c.y * cs.y), e * (c.y * cs.x - c.x * cs.y));
      }
      // W: values j = 2n (Re), 2n + 1 (Im) for n = 16 g .. 16 g + 15: chunks 4 g .. 4 g + 3
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float4 q = cur.w[2 * k + i];
          const float2 c0 = kFwd ? make_float2(q.x, q.y) : make_float2(q.x, -q.y);
          const float2 c1 = kFwd ? make_float2(q.z, q.w) : make_float2(q.z, -q.w);
          v[4 * i] = c0.x * f.x - c0.y * f.y;
          v[4 * i + 1] = c0.x * f.y + c0.y * f.x;
          v[4 * i + 2] = c1.x * f.x - c1.y * f.y;
          v[4 * i + 3] = c1.x * f.y + c1.y * f.x;
        }
        uint4 hi, lo;
        split8(v, hi, lo);
        const uint32_t o = tile_off((uint32_t)tl, 4u * (uint32_t)g + (uint32_t)k);
        st_shared_v4(base + kTile + o, hi);
        st_shared_v4(base + 2 * kTile + o, lo);
      }
      // R: p = 16 g .. 16 g + 15, hi at stacked rows m = 32 g + (p mod 16), lo 16 further
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = cur.r[8 * k + i];
        uint4 hi, lo;
        split8(v, hi, lo);
        st_shared_v4(base + tile_off((uint32_t)tl, 4u * (uint32_t)g + (uint32_t)k), hi);
        st_shared_v4(base + tile_off((uint32_t)tl, 4u * (uint32_t)g + 2u + (uint32_t)k), lo);
      }
      const float2 gz = cur.gz;
      run = kFwd ? make_float2(run.x * gz.x - run.y * gz.y, run.x * gz.y + run.y * gz.x)
                 : make_float2(run.x * gz.x + run.y * gz.y, run.y * gz.x - run.x * gz.y);
    }
    if (warp == 0) M3_TRACE(it, 2);
    if (it + 1 < seg) load(chunk_of(it + 1), cur);  // lands while this chunk's MMAs run
    fence_proxy_async_smem();
    tc_fence_before_sync();
    __syncthreads();
    if (warp == 0) M3_TRACE(it, 3);
    if (tid == 0) {
      tc_fence_after_sync();
      const uint32_t idesc = idesc_bf16(128, 128, 1, 1);
#pragma unroll
      for (int hp = 0; hp < 2; ++hp)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_bf16_ss(tmem, sdesc(base + k * 2048u, 8192, 1024),
                      sdesc(base + (1u + (uint32_t)hp) * kTile + k * 2048u, 8192, 1024), idesc,
                      (it | hp | k) != 0 ? 1u : 0u);
      mma_commit(&bar[buf]);
      M3_TRACE(it, 4);
    }
  };
  Rows rows;
  load(chunk_of(0), rows);
  for (int it = 0; it < seg; ++it) step(it, rows);
  // every MMA is done once the last chunk's commit has arrived
  const int last = seg - 1;
  if (warp == 0) M3_TRACE(seg, 0);
  mbar_wait(&bar[last & 1], (uint32_t)(last >> 1) & 1u, a.err, kErrMmaWait);
  if (warp == 0) M3_TRACE(seg, 1);
  tc_fence_after_sync();
  {
    // TMEM lane m = 32 q + (lane): p = 16 q + lane mod 16, hi (lanes 0-15) or lo (16-31); columns
    // 64 ch .. 64 ch + 63 of this warp. Each lane keeps half of them after adding hi and lo.
    const int q = warp & 3, ch = warp >> 2, part = lane >> 4;
    float v0[32], v1[32];
    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 64u * ch, v0);
    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 64u * ch + 32u, v1);
    tmem_ld_wait();
    float2* dst = out + (long long)sg * 64 * 64 + 16 * q + (lane & 15);
    const int n0 = 32 * ch + 16 * part;
#pragma unroll
    for (int c = 0; c < 32; c += 2) {
      const float s0 = part ? v0[c] : v1[c], s1 = part ? v0[c + 1] : v1[c + 1];
      const float r0 = __shfl_xor_sync(0xffffffffu, s0, 16);
      const float r1 = __shfl_xor_sync(0xffffffffu, s1, 16);
      const float re = (part ? v1[c] : v0[c]) + r0, im = (part ? v1[c + 1] : v0[c + 1]) + r1;
      dst[(long long)(n0 + c / 2) * 64] = make_float2(re, im);
    }
  }
  if (warp == 0) M3_TRACE(seg, 2);
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

namespace {

bool vec_rows(const void* ptr, const long long st[4], long long unit) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 || st[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (st[i] % unit) return false;
  return true;
}

}  // namespace

bool chain_state_tc_ok(const Problem& p, bool forward, const void* r, const long long rs[4],
                       int r_bf16) {
  const float2* w = forward ? p.Bm : p.Cm;
  const long long* ws = forward ? p.bs : p.cs;
  // 16-byte rows: complex strides even (planar: float strides multiples of 4, the imaginary rows
  // H * 64 floats on), real strides multiples of 4 (fp32) or 8 (bf16)
  const bool w_ok = p.bc_planar ? vec_rows(w, ws, 4) && ws[2] == 64 : vec_rows(w, ws, 2);
  return w_ok && vec_rows(r, rs, r_bf16 ? 8 : 4);
}

int run_chain_state(const Problem& p, bool forward, const void* r, const long long rs[4],
                    int r_bf16, const ChunkRec* recs, int G, float2* out, uint32_t* err,
                    cudaStream_t st) {
  ChainStateArgs a{};
  a.W = forward ? p.Bm : p.Cm;
  a.w_planar = p.bc_planar;
  for (int i = 0; i < 4; ++i) {
    a.ws[i] = forward ? p.bs[i] : p.cs[i];
    a.rs[i] = rs[i];
  }
  a.R = r;
  a.r_bf16 = r_bf16;
  a.recs = recs;
  a.T = p.T;
  a.H = p.H;
  a.nc = (p.T + 63) / 64;
  a.G = G;
  a.err = err;
  auto kern = forward ? k_chain_state_tc<true> : k_chain_state_tc<false>;
  if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kSmemBytes))
    return M3SSD_ERR_LAUNCH;
  kern<<<p.Bsz * p.H * G, kThreads, kSmemBytes, st>>>(a, out);
  return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace m3ssd

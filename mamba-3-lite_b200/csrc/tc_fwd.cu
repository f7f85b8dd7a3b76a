// Tensor-core forward of the complex chunkwise SSD for head_dim = state_dim = 64, real x.
//
// Persistent CTAs (two per SM) take chunk tickets (chunk-major order over all b*H sequences) from a
// global counter. Per ticket (64 positions of one (b, h)), with Sigma_l = rho_l + i theta_l the
// within-chunk cumsum of a = softplus(dt) A (models/ssd_complex.py:82, :89), Gamma = Sigma_63:
//
//   C'[l,n] = C[l,n] cis(theta_l)          B'[s,n] = B[s,n] conj(cis(theta_s))
//   G  = Re(C' B'^T)                       (= Re(C B^T o cis(theta_l - theta_s)), K = 2N)
//   Mr = exp(rho_l - rho_s) G  for s <= l (the causal decay L of :50-52, exp only where s <= l)
//   Y1 = Mr x                              (intra-chunk output, :53)
//   S~ = sum_s exp(rho_Gamma - rho_s) B'[s] x[s]^T    (chunk state, :54, before the cis(theta_Gamma))
//   H_{z+1} = e^Gamma H_z + cis(theta_Gamma) S~       (the carry of :98-111 as a scan)
//   y  = Y1 + exp(rho_l) Re(C' H_z)        (:115-119)
//
// All four contractions run on tcgen05 (kind::f16) with split-bf16 operands and fp32 TMEM
// accumulators (tc_common.cuh). B and C tiles arrive by TMA; x and dt by 128-bit loads
// prefetched one ticket ahead. H_z is handed from the CTA that processed chunk z-1 of the same
// sequence through global memory (it is also the `states` output the backward reads) with a
// release flag; waits are bounded and report kErrFlagWait instead of hanging. A state tile is
// stored thread-major (float4 i of thread t at [i][t]) so each warp access is 512 contiguous bytes;
// y leaves through a swizzled staging tile and TMA stores.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <string.h>

#include <mutex>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"
#include "tc_path.h"
#include "tc_trace.cuh"

namespace m3ssd {
namespace tc {

M3_TRACE_DEFINE(m3ssd_trace_set_fwd)

namespace {

constexpr int kThreads = 256;

// Shared memory map (offsets from a 1024-aligned base), ~100 KB so two CTAs share an SM:
// one CTA's memory waits and barriers overlap the other's MMAs and epilogues.
constexpr uint32_t OFF_CX = 0;       // TMA tile of C (fp32 64 x 128, or Re | Im 64 x 64 each),
                                     // then C'x stacked (A operand)
constexpr uint32_t OFF_BX = 32768;   // TMA tile of B, then B'x hi | lo (64 x 128 each 16 KB),
                                     // then conj(H_z) hi | lo as [k-atom][p][64] (K-major B)
constexpr uint32_t OFF_XH = 65536;   // x hi [s][p]
constexpr uint32_t OFF_XL = 73728;   // x lo
constexpr uint32_t OFF_XT = 81920;   // x~ stacked [p-group][s][64], then Mr stacked [128][s],
                                     // then the y staging tile (two 32-float segments)
constexpr uint32_t OFF_MISC = 98304;
constexpr uint32_t kSmemBytes = OFF_MISC + 2048 + 1024;
constexpr uint32_t kTmaBytes = 2u * 64u * 128u * 4u;

// TMEM columns (256 per CTA): G then Y1 share [0, 64)
constexpr uint32_t COL_G = 0, COL_Y1 = 0, COL_S = 64, COL_Y2 = 192, kTmemCols = 256;

struct Misc {
  ChunkRec rec;  // this chunk's decay quantities (bulk-copied with the B/C tiles)
  uint64_t bar_tma, bar_mma1, bar_mma2, bar_mma3;
  int first, nxt;
  int h_ready;
  uint32_t tmem_base;
};
static_assert(sizeof(Misc) <= 2048, "misc area");

struct FwdParams {
  int Bsz, T, H, nc, total;
  const float* x;
  long long xs[4];
  // 1: 16 consecutive values of a row by four 128-bit loads. 2 or 3: x is the real (2) or the
  // imaginary (3) part of complex values (strides of 2 floats): eight 128-bit loads of the complex
  // pairs, keeping that part
  int x_vec;
  const ChunkRec* recs;
  float* states;
  uint32_t* flags;
  uint32_t* counter;
  uint32_t* err;
  int y_bf16;  // y leaves as bfloat16 (one 64-column staging segment) instead of float32 (two)
  // state carry (optional): initial state h0 and final state hT, (B, H, N, D) complex64
  // contiguous = s[n][p] of the reference's recurrence, the transpose of a state tile H[p][n]
  const float2* h0;
  float2* hT;
  // segments: each sequence's chunks run as G chains of seg = nc / G chunks (G = 1: one chain).
  // A chain starts from h0 (per (sequence, segment), or zero) and its end state goes to hT.
  int G, seg;
  // complex x runs as two real passes (x = xr + i xi: y = F(xr; C) + F(xi; i C)): the factor C is
  // multiplied by as it is read (1, or i in the second pass), and whether y is added to what the
  // first pass stored (TMA reduce-add) instead of stored
  float2 crot;
  int y_accum;
};

// (chunk, sequence, segment) of a ticket: chunk-within-segment major, so every chain's first
// chunk comes before any second chunk and a ticket only waits on smaller ones
struct FwdPos {
  int z, bh, j, sg;  // chunk, sequence, chunk within its segment, bh * G + segment
};
template <bool kChains>
__device__ __forceinline__ FwdPos fwd_pos(int tk, int BH, int G, int seg) {
  FwdPos q;
  if constexpr (!kChains) {  // one chain per sequence
    q.z = q.j = tk / BH;
    q.bh = q.sg = tk - q.z * BH;
    return q;
  }
  q.j = tk / (BH * G);
  const int rest = tk - q.j * BH * G;
  const int sgm = rest / BH;
  q.bh = rest - sgm * BH;
  q.z = sgm * seg + q.j;
  q.sg = q.bh * G + sgm;
  return q;
}

__device__ __forceinline__ void load_x16(const FwdParams& p, int b, int t, int h, int p0,
                                         float (&xv)[16]) {
  if (t >= p.T) {
#pragma unroll
    for (int i = 0; i < 16; ++i) xv[i] = 0.f;
    return;
  }
  const float* base = p.x + b * p.xs[0] + (long long)t * p.xs[1] + h * p.xs[2];
  if (p.x_vec == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = ldg_nc_v4(base + p0 + 4 * i);
      xv[4 * i] = v.x;
      xv[4 * i + 1] = v.y;
      xv[4 * i + 2] = v.z;
      xv[4 * i + 3] = v.w;
    }
  } else if (p.x_vec >= 2) {
    const int part = p.x_vec - 2;
    const float* pairs = base - part + 2 * p0;  // the complex values p0 .. p0 + 15
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 v = ldg_nc_v4(pairs + 4 * i);
      xv[2 * i] = part ? v.y : v.x;
      xv[2 * i + 1] = part ? v.w : v.z;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) xv[i] = __ldg(base + (long long)(p0 + i) * p.xs[3]);
  }
}

__device__ __forceinline__ float2 cmulf(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// fp32 staging tile for a TMA store: 32-float column segment of a 64-row tile, 128-byte rows,
// 16-byte chunks swizzled by row (the CU_TENSOR_MAP_SWIZZLE_128B layout)
__device__ __forceinline__ uint32_t stage_addr(uint32_t seg_base, uint32_t row, uint32_t chunk) {
  return seg_base + row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void split_store16(uint32_t hi_addr, uint32_t lo_addr, const float* v) {
  float w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = v[i];
  uint4 hi, lo;
  split8(w, hi, lo);
  st_shared_v4(hi_addr, hi);
  st_shared_v4(lo_addr, lo);
}

}  // namespace

// kPlanar: B and C tiles arrive as separate real and imaginary 64 x 64 fp32 tiles (the in_proj
// column layout) instead of one interleaved 64 x 128 tile; everything after the transform is shared
// kStateFirst: H_{z+1} is formed and released as soon as S~ and H_z are in, before epilogue 1,
// behind a block barrier of its own (the control warp's release fence then delays its epilogue):
// for problems with few independent chains, whose time is the chain of chunk-to-chunk hand-offs
template <bool kPlanar, bool kChains, bool kStateFirst>
__global__ void __launch_bounds__(kThreads, 2)
    k_fwd_tc(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
             const __grid_constant__ CUtensorMap tmY, const FwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  Misc& m = *reinterpret_cast<Misc*>(smem + OFF_MISC);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int sub = warp & 3, wg = warp >> 2, part = lane >> 4;
  const int r = 16 * sub + (lane & 15);  // logical row of this TMEM lane (position l, or p)
  const int BH = p.Bsz * p.H;
  // ticket counter, TMA issue and hand-off flags are handled by one lane of warp 7 so warps 0-1
  // (cumsum) and thread 0 (MMA issue) never stall on them
  const bool ctrl = tid == kThreads - 32;

  if (tid == 0) {
    mbar_init(&m.bar_tma, 1);
    mbar_init(&m.bar_mma1, 1);
    mbar_init(&m.bar_mma2, 1);
    mbar_init(&m.bar_mma3, 1);
    fence_barrier_init();
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmC);
    prefetch_tmap(&tmY);
    m.first = (int)atomicAdd(p.counter, 1u);
  }
  if (warp == 0) {
    tmem_alloc(&m.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = m.tmem_base;
  const uint32_t lane_off = (uint32_t)(32 * sub) << 16;

  int ticket = m.first;
  float xv[16];
  auto prefetch_regs = [&](int tk) {
    const FwdPos q = fwd_pos<kChains>(tk, BH, p.G, p.seg);
    const int z = q.z, bh = q.bh;
    const int b = bh / p.H, h = bh - b * p.H, t0 = z * 64;
    load_x16(p, b, t0 + (tid >> 2), h, 16 * (tid & 3), xv);
  };
  if (ticket < p.total) prefetch_regs(ticket);
  // B, C tiles and the decay record of a ticket (issued once the previous ticket's MMAs are done)
  auto issue_tma = [&](int tk) {
    const FwdPos q = fwd_pos<kChains>(tk, BH, p.G, p.seg);
    const int z = q.z, bh = q.bh;
    const int b = bh / p.H, h = bh - b * p.H;
    mbar_arrive_expect_tx(&m.bar_tma, kTmaBytes + (uint32_t)sizeof(ChunkRec));
    tma_load_4d(smem + OFF_BX, &tmB, &m.bar_tma, 0, h, z * 64, b);
    tma_load_4d(smem + OFF_CX, &tmC, &m.bar_tma, 0, h, z * 64, b);
    if constexpr (kPlanar) {  // imaginary parts: H*N floats after the real parts (row h + H)
      tma_load_4d(smem + OFF_BX + 16384, &tmB, &m.bar_tma, 0, p.H + h, z * 64, b);
      tma_load_4d(smem + OFF_CX + 16384, &tmC, &m.bar_tma, 0, p.H + h, z * 64, b);
    }
    bulk_load(&m.rec, p.recs + (long long)bh * p.nc + z, (uint32_t)sizeof(ChunkRec), &m.bar_tma);
  };
  if (ctrl && ticket < p.total) issue_tma(ticket);
  int yb = 0, yh = 0, yt0 = 0;  // (ctrl) output tile staged by the previous ticket
  uint32_t h_probe = 0;         // (ctrl) H_z flag as seen halfway through the operand transform

  uint32_t iter = 0;
  while (ticket < p.total) {
    const uint32_t ph = iter & 1u;
    const FwdPos q = fwd_pos<kChains>(ticket, BH, p.G, p.seg);
    const int z = q.z, bh = q.bh, j = q.j;
    const int b = bh / p.H, h = bh - b * p.H, t0 = z * 64;
    __syncthreads();  // previous ticket done: its MMAs completed, its y tile staged
    if (warp == 0) M3_TRACE(iter, 0);
    int next = 0;     // grabbed late in this ticket so the window of open tickets stays small
    if (ctrl) {
      if (iter > 0) {  // the previous ticket's y: two 32-column fp32 segments (one bf16) from sXT
        tma_put_4d(&tmY, smem + OFF_XT, 0, yh, yt0, yb, p.y_accum != 0);
        if (!p.y_bf16) tma_put_4d(&tmY, smem + OFF_XT + 8192, 32, yh, yt0, yb, p.y_accum != 0);
        bulk_commit_group();
      }
      yb = b;
      yh = h;
      yt0 = t0;
    }

    // ---- TMA tiles of B and C land in the operand buffers; rotate and split them in place:
    // B first, then x and x~, so S~ = x~^T B'x runs on the tensor core while C is converted
    mbar_wait(&m.bar_tma, ph, p.err, kErrTmaWait);
    if (warp == 0) M3_TRACE(iter, 1);
    // all raw values of one tile in registers (each thread: rows j/16, complex 4 (j%16) .. +3 for
    // j = tid + 256 it); written back in place after a barrier
    auto read_tile = [&](uint32_t base, float4 (&r4)[4][2]) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int j = tid + kThreads * it;
        if constexpr (kPlanar) {  // Re and Im of complex 4q .. 4q+3 of row l, interleaved here
          const float* src = reinterpret_cast<const float*>(smem + base) + (j >> 4) * 64 + 4 * (j & 15);
          const float4 re = *reinterpret_cast<const float4*>(src);
          const float4 im = *reinterpret_cast<const float4*>(src + 4096);
          r4[it][0] = make_float4(re.x, im.x, re.y, im.y);
          r4[it][1] = make_float4(re.z, im.z, re.w, im.w);
        } else {
          // 32 bytes per thread: lanes 4-7 of each group of 8 read their second float4 first,
          // so each 8-lane phase of a 128-bit load covers all 32 banks once
          const float* src = reinterpret_cast<const float*>(smem + base) + (j >> 4) * 128 + 8 * (j & 15);
          const int sw = (j >> 2) & 1;
          const float4 a = *reinterpret_cast<const float4*>(src + 4 * sw);
          const float4 b = *reinterpret_cast<const float4*>(src + 4 - 4 * sw);
          r4[it][0] = sw ? b : a;
          r4[it][1] = sw ? a : b;
        }
      }
    };
    // tile 0: C -> C'x (stacked); tile 1: B -> B'x hi | lo
    auto write_tile = [&](int tile, const float4 (&r4)[4][2]) {
#pragma unroll
      for (int it = 0; it < 4; ++it) {
        const int j = tid + kThreads * it;
        const int l = j >> 4, q = j & 15;
        const float2 cs = tile == 0 ? cmulf(m.rec.cis[l], p.crot) : m.rec.cis[l];
        const uint32_t ka = (uint32_t)q >> 3, ch = (uint32_t)q & 7u;
        const float rv[8] = {r4[it][0].x, r4[it][0].y, r4[it][0].z, r4[it][0].w,
                             r4[it][1].x, r4[it][1].y, r4[it][1].z, r4[it][1].w};
        float v[8];
        if (tile == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {  // C * cis(theta_l)
            v[2 * u] = rv[2 * u] * cs.x - rv[2 * u + 1] * cs.y;
            v[2 * u + 1] = rv[2 * u] * cs.y + rv[2 * u + 1] * cs.x;
          }
          split_store16(sb + OFF_CX + ka * 16384u + swz(stack_row(l, 0), ch),
                        sb + OFF_CX + ka * 16384u + swz(stack_row(l, 1), ch), v);
        } else {
#pragma unroll
          for (int u = 0; u < 4; ++u) {  // conj(B * conj(cis(theta_s)))
            v[2 * u] = rv[2 * u] * cs.x + rv[2 * u + 1] * cs.y;
            v[2 * u + 1] = rv[2 * u] * cs.y - rv[2 * u + 1] * cs.x;
          }
          split_store16(sb + OFF_BX + ka * 8192u + swz(l, ch),
                        sb + OFF_BX + 16384u + ka * 8192u + swz(l, ch), v);
        }
      }
    };
    float4 rc[4][2];  // the raw C tile, read once B'x and x~ are written
    {
      float4 rb[4][2];
      read_tile(OFF_BX, rb);
      if (ctrl) bulk_wait_read_all();  // sXT (y staging) is rewritten below
      __syncthreads();
      if (warp == 0) M3_TRACE(iter, 2);
      write_tile(1, rb);
      // x (hi, lo) and x~ = exp(rho_Gamma - rho_s) x, stacked over p
      const int s = tid >> 2, pg = tid & 3;
      split_store16(sb + OFF_XH + swz(s, 2 * pg), sb + OFF_XL + swz(s, 2 * pg), xv);
      split_store16(sb + OFF_XH + swz(s, 2 * pg + 1), sb + OFF_XL + swz(s, 2 * pg + 1), xv + 8);
      const float dd = m.rec.dec[s];
      float xt[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) xt[u] = dd * xv[u];
      const uint32_t xtb = sb + OFF_XT + (uint32_t)(pg >> 1) * 8192u;
      const uint32_t c4 = 4u * (uint32_t)(pg & 1);
      split_store16(xtb + swz(s, c4 + 0), xtb + swz(s, c4 + 2), xt);
      split_store16(xtb + swz(s, c4 + 1), xtb + swz(s, c4 + 3), xt + 8);
      read_tile(OFF_CX, rc);
      if (warp == 0) M3_TRACE(iter, 3);
      // is H_z already published? (then its loads overlap the first MMAs.) Probed as late as
      // the probe's round trip still hides behind the rest of the transform: its value is
      // stored to shared memory at the end of the transform
      if (ctrl) h_probe = (j == 0) ? 1u : ld_relaxed_gpu(p.flags + (long long)bh * p.nc + z);
    }
    fence_proxy_async_smem();
    __syncthreads();
    if (warp == 0) M3_TRACE(iter, 4);
    if (tid == 0) {  // MMA batch 1a: S~^T = x~^T B'x (M128 N128)
      tc_fence_after_sync();
      const uint32_t idS = idesc_bf16(128, 128, 1, 1);
#pragma unroll
      for (int hl = 0; hl < 2; ++hl)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_bf16_ss(tmem + COL_S, sdesc(sb + OFF_XT + j * 2048u, 8192, 1024),
                      sdesc(sb + OFF_BX + hl * 16384u + j * 2048u, 8192, 1024), idS,
                      (hl | j) != 0);
    }
    write_tile(0, rc);
    if (ctrl) {  // a published H_z is read by every thread after the barrier below
      if (j > 0 && h_probe != 0u) fence_acquire_gpu();
      m.h_ready = (int)h_probe;
    }
    fence_proxy_async_smem();
    __syncthreads();
    const bool h_early = m.h_ready != 0;
    if (warp == 0) M3_TRACE(iter, 5);
    // not yet published at the probe: every thread looks again now (no barrier needed later: each
    // thread orders its own H loads after its own observation of the flag)
    uint32_t h_late = 1u;
    if (j > 0 && !h_early) h_late = ld_relaxed_gpu(p.flags + (long long)bh * p.nc + z);

    // ---- MMA batch 1b: G = C'x B'x^T (M128 N64); the commit covers S~ too
    if (tid == 0) {
      tc_fence_after_sync();
      M3_TRACE(iter, 17);
      const uint32_t idG = idesc_bf16(128, 64, 0, 0);
#pragma unroll
      for (int hl = 0; hl < 2; ++hl)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_bf16_ss(tmem + COL_G, sdesc(sb + OFF_CX + (j >> 2) * 16384u + (j & 3) * 32u, 16, 1024),
                      sdesc(sb + OFF_BX + hl * 16384u + (j >> 2) * 8192u + (j & 3) * 32u, 16, 1024),
                      idG, (hl | j) != 0);
      mma_commit(&m.bar_mma1);
    }
    if (warp == 0) M3_TRACE(iter, 6);
    float hz[32];
    if (j == 0) {  // a chain's entry state: zero, or h0 (row p = r, complex n = 32 wg + 16 part + c/2)
      if (p.h0 != nullptr) {
        const float2* src = p.h0 + ((long long)q.sg * 64 + 32 * wg + 16 * part) * 64 + r;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float2 v = __ldcg(src + c * 64);
          hz[2 * c] = v.x;
          hz[2 * c + 1] = v.y;
        }
      } else {
#pragma unroll
        for (int c = 0; c < 32; ++c) hz[c] = 0.f;
      }
    } else if (h_early) {  // H_z already published: load it while the MMAs run
      const float4* src =
          reinterpret_cast<const float4*>(p.states + ((long long)bh * p.nc + z) * 64 * 128) + tid;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 v = __ldcg(src + i * kThreads);
        hz[4 * i] = v.x;
        hz[4 * i + 1] = v.y;
        hz[4 * i + 2] = v.z;
        hz[4 * i + 3] = v.w;
      }
    }

    auto load_hz = [&]() {
      // ---- H_z from the predecessor chunk (bounded wait on its release flag if not yet seen)
      if (j > 0 && !h_early) {
        if (h_late == 0u) flag_wait_relaxed(p.flags + (long long)bh * p.nc + z, p.err);
        fence_acquire_gpu();
        const float4* src =
            reinterpret_cast<const float4*>(p.states + ((long long)bh * p.nc + z) * 64 * 128) + tid;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 v = __ldcg(src + i * kThreads);
          hz[4 * i] = v.x;
          hz[4 * i + 1] = v.y;
          hz[4 * i + 2] = v.z;
          hz[4 * i + 3] = v.w;
        }
      }
    };
    auto state_update = [&]() {
      // ---- state update H_{z+1} = e^Gamma H_z + cis(theta_Gamma) S~ (S~ is done since the first
      // MMA wait). In the default order it runs before the barrier that starts Y1 and Y2: its
      // gpu-scope release then runs while the tensor core computes them instead of holding up
      // the control warp's output epilogue
      {
        const float2 g = m.rec.g, ct = m.rec.ct;
        float4* tile0 = reinterpret_cast<float4*>(p.states + (long long)bh * p.nc * 64 * 128) + tid;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float s0[16], s1[16];
          tmem_ld16(tmem + lane_off + COL_S + 64u * wg + 16u * hh, s0);
          tmem_ld16(tmem + lane_off + COL_S + 64u * wg + 32u + 16u * hh, s1);
          tmem_ld_wait();
          float hn[16];
#pragma unroll
          for (int c = 0; c < 16; c += 2) {
            const float sa = part ? s0[c] : s1[c];
            const float sbv = part ? s0[c + 1] : s1[c + 1];
            const float ra = __shfl_xor_sync(0xffffffffu, sa, 16);
            const float rbv = __shfl_xor_sync(0xffffffffu, sbv, 16);
            const float sr = (part ? s1[c] : s0[c]) + ra;
            const float si = -((part ? s1[c + 1] : s0[c + 1]) + rbv);  // B'x is conjugated
            const int k = 16 * hh + c;
            const float2 hv = cmulf(g, make_float2(hz[k], hz[k + 1]));
            const float2 sv = cmulf(ct, make_float2(sr, si));
            hn[c] = hv.x + sv.x;
            hn[c + 1] = hv.y + sv.y;
          }
          if (j == 0) {  // a chain's first chunk stores its own entry state tile (the backward reads it)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              __stcg(tile0 + (long long)z * 64 * 32 + (4 * hh + i) * kThreads,
                     make_float4(hz[16 * hh + 4 * i], hz[16 * hh + 4 * i + 1],
                                 hz[16 * hh + 4 * i + 2], hz[16 * hh + 4 * i + 3]));
          }
          if (j + 1 < (kChains ? p.seg : p.nc)) {
            float4* dst = tile0 + (long long)(z + 1) * 64 * 32;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              __stcg(dst + (4 * hh + i) * kThreads,
                     make_float4(hn[4 * i], hn[4 * i + 1], hn[4 * i + 2], hn[4 * i + 3]));
          } else if (p.hT != nullptr) {  // the chain's end state, transposed to (n, p)
            float2* dst = p.hT + ((long long)q.sg * 64 + 32 * wg + 16 * part + 8 * hh) * 64 + r;
#pragma unroll
            for (int c = 0; c < 8; ++c) __stcg(dst + c * 64, make_float2(hn[2 * c], hn[2 * c + 1]));
          }
        }
      }
    };
    // ---- epilogue 1: Mr = exp(rho_l - rho_s) G (s <= l), split-bf16, stacked rows (over x~)
    float el_r;  // exp(rho_r), kept for the output (the record slot is refilled before it)
    mbar_wait(&m.bar_mma1, ph, p.err, kErrMmaWait);
    if (warp == 0) M3_TRACE(iter, 7);
    tc_fence_after_sync();
    if constexpr (kStateFirst) {  // H_{z+1} out to the next chunk's ticket first
      load_hz();
      state_update();
      tc_fence_before_sync();
      __syncthreads();
      if (ctrl && j + 1 < (kChains ? p.seg : p.nc))
        st_release_gpu(p.flags + (long long)bh * p.nc + z + 1, 1u);
    }
    {
      float v[32];
      tmem_ld32(tmem + lane_off + COL_G + 32u * wg, v);
      tmem_ld_wait();
      if (warp == 0) M3_TRACE(iter, 19);
      float mr[16];
      const float rl = m.rec.rho2[r];
      el_r = m.rec.el[r];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float send = part ? v[c] : v[16 + c];
        const float recv = __shfl_xor_sync(0xffffffffu, send, 16);
        const float gsum = (part ? v[16 + c] : v[c]) + recv;
        const int s = 32 * wg + 16 * part + c;
        mr[c] = (s <= r) ? exp2f(rl - m.rec.rho2[s]) * gsum : 0.f;
      }
      const uint32_t ch = 4u * wg + 2u * part;
      split_store16(sb + OFF_XT + swz(stack_row(r, 0), ch), sb + OFF_XT + swz(stack_row(r, 1), ch), mr);
      split_store16(sb + OFF_XT + swz(stack_row(r, 0), ch + 1),
                    sb + OFF_XT + swz(stack_row(r, 1), ch + 1), mr + 8);
    }

    if (warp == 0) M3_TRACE(iter, 8);
    int nn = 0;
    if (ctrl) nn = (int)atomicAdd(p.counter, 1u);  // next ticket; stored at the state update

    if constexpr (!kStateFirst) load_hz();
    if (warp == 0) M3_TRACE(iter, 9);
    // conj(H_z) interleaved as a K-major B operand [k-atom][p][64 k] (hi | lo), over B'x
    {
      float w[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) w[c] = (c & 1) ? -hz[c] : hz[c];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        split_store16(sb + OFF_BX + (uint32_t)wg * 8192u + swz(r, 4 * part + jj),
                      sb + OFF_BX + 16384u + (uint32_t)wg * 8192u + swz(r, 4 * part + jj),
                      w + 8 * jj);
    }
    if (ctrl) m.nxt = nn;
    if constexpr (!kStateFirst) state_update();
    fence_proxy_async_smem();
    tc_fence_before_sync();
    __syncthreads();
    next = m.nxt;
    if (warp == 0) M3_TRACE(iter, 10);
    if (tid == 0) {  // Y1 = Mr x, Y2 = Re(C' H_z) as C'x conj(H)x
      tc_fence_after_sync();
      M3_TRACE(iter, 18);
      const uint32_t idY1 = idesc_bf16(128, 64, 0, 1);
#pragma unroll
      for (int hl = 0; hl < 2; ++hl)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_bf16_ss(tmem + COL_Y1, sdesc(sb + OFF_XT + j * 32u, 16, 1024),
                      sdesc(sb + (hl ? OFF_XL : OFF_XH) + j * 2048u, 8192, 1024), idY1,
                      (hl | j) != 0);
      mma_commit(&m.bar_mma2);
      M3_TRACE(iter, 20);
      const uint32_t idY2 = idesc_bf16(128, 64, 0, 0);
#pragma unroll
      for (int hl = 0; hl < 2; ++hl)
#pragma unroll
        for (int j = 0; j < 8; ++j)
          mma_bf16_ss(tmem + COL_Y2, sdesc(sb + OFF_CX + (j >> 2) * 16384u + (j & 3) * 32u, 16, 1024),
                      sdesc(sb + OFF_BX + hl * 16384u + (j >> 2) * 8192u + (j & 3) * 32u, 16, 1024),
                      idY2, (hl | j) != 0);
      mma_commit(&m.bar_mma3);
    }
    if (warp == 0) M3_TRACE(iter, 11);
    if (warp == 0) M3_TRACE(iter, 12);
    // the barrier orders every thread's H stores before this gpu-scope release (its fence holds
    // the control thread's warp ~1 us; the Y MMAs run meanwhile)
    if (!kStateFirst && ctrl && j + 1 < (kChains ? p.seg : p.nc))
      st_release_gpu(p.flags + (long long)bh * p.nc + z + 1, 1u);
    if (ctrl) M3_TRACE(iter, 16);

    // ---- output y = Y1 + exp(rho_l) Y2 into the staging tile in sXT; the next ticket's B, C
    // tiles and record load as soon as the last MMA has read sCX / sBX
    mbar_wait(&m.bar_mma2, ph, p.err, kErrMmaWait);
    mbar_wait(&m.bar_mma3, ph, p.err, kErrMmaWait);
    if (warp == 0) M3_TRACE(iter, 13);
    tc_fence_after_sync();
    if (ctrl && next < p.total) issue_tma(next);
    // x of the next ticket, issued after the waits (a wait that falls through to its out-of-line
    // polling loop would first wait for loads in flight into registers it saves)
    if (next < p.total) prefetch_regs(next);
    {
      float y1[32], y2[32];
      tmem_ld32(tmem + lane_off + COL_Y1 + 32u * wg, y1);
      tmem_ld32(tmem + lane_off + COL_Y2 + 32u * wg, y2);
      tmem_ld_wait();
      float out[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float s1v = part ? y1[c] : y1[16 + c];
        const float s2v = part ? y2[c] : y2[16 + c];
        const float r1 = __shfl_xor_sync(0xffffffffu, s1v, 16);
        const float r2 = __shfl_xor_sync(0xffffffffu, s2v, 16);
        const float a1 = (part ? y1[16 + c] : y1[c]) + r1;
        const float a2 = (part ? y2[16 + c] : y2[c]) + r2;
        out[c] = a1 + el_r * a2;
      }
      if (p.y_bf16) {  // columns 32 wg + 16 part .. +15 = 16-byte chunks 4 wg + 2 part, +1
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const __nv_bfloat162 v2 = __floats2bfloat162_rn(out[2 * i], out[2 * i + 1]);
          w[i] = *reinterpret_cast<const uint32_t*>(&v2);
        }
        const uint32_t c0 = 4u * (uint32_t)wg + 2u * (uint32_t)part;
        st_shared_v4(stage_addr(sb + OFF_XT, (uint32_t)r, c0), make_uint4(w[0], w[1], w[2], w[3]));
        st_shared_v4(stage_addr(sb + OFF_XT, (uint32_t)r, c0 + 1u),
                     make_uint4(w[4], w[5], w[6], w[7]));
      } else {
        const uint32_t seg = sb + OFF_XT + (uint32_t)wg * 8192u;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          st_shared_v4(stage_addr(seg, (uint32_t)r, (uint32_t)(4 * part + i)),
                       make_uint4(__float_as_uint(out[4 * i]), __float_as_uint(out[4 * i + 1]),
                                  __float_as_uint(out[4 * i + 2]), __float_as_uint(out[4 * i + 3])));
      }
      fence_proxy_async_smem();
    }
    if (warp == 0) M3_TRACE(iter, 14);
    tc_fence_before_sync();
    ticket = next;
    ++iter;
  }
  __syncthreads();
  if (ctrl) {
    if (iter > 0) {  // the last ticket's y
      tma_put_4d(&tmY, smem + OFF_XT, 0, yh, yt0, yb, p.y_accum != 0);
      if (!p.y_bf16) tma_put_4d(&tmY, smem + OFF_XT + 8192, 32, yh, yt0, yb, p.y_accum != 0);
      bulk_commit_group();
    }
    bulk_wait_all();
  }
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
namespace {

// TMA needs a 16-byte aligned base and 16-byte multiples for every stride but the innermost
bool bc_tma_ok(const Problem& p, const void* ptr, const long long st[4]) {
  if (st[3] != 1) return false;
  if (p.bc_planar) {  // float strides; the imaginary rows sit H*N floats after the real ones
    if (st[2] != p.N) return false;
    for (int i = 0; i < 2; ++i)
      if (st[i] <= 0 || (st[i] % 4) != 0) return false;
  } else {            // complex strides
    for (int i = 0; i < 3; ++i)
      if (st[i] <= 0 || (st[i] % 2) != 0) return false;
  }
  return (reinterpret_cast<uintptr_t>(ptr) % 16) == 0;
}

}  // namespace

// cuTensorMapEncodeTiled is a driver API; it is resolved through the runtime so the library does
// not link libcuda (it loads on machines without a driver, where only host queries work).
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// Host-side caches of what every call would otherwise redo: encoded tensor maps (a map depends only
// on its address, shape, strides, box and modes, not on the memory's contents or lifetime), the SM
// count and the dynamic shared memory attribute of each kernel, per device. One mutex guards all;
// each lookup is a short linear scan.
namespace {
struct MapKey {
  CUtensorMapDataType dtype;
  CUtensorMapSwizzle swizzle;
  CUtensorMapL2promotion l2;
  const void* ptr;
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  cuuint32_t box[4];
};
struct MapEntry {
  bool used;
  MapKey key;
  CUtensorMap map;
};
constexpr int kMapCache = 64;
constexpr int kMaxDev = 64;
std::mutex g_cache_mu;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
int g_sms[kMaxDev] = {};
struct AttrEntry {
  const void* func;
  int dev;
  int bytes;
};
AttrEntry g_attrs[64];
int g_nattrs = 0;

// cuTensorMapEncodeTiled of a 4-D map (element strides 1, no interleave, no out-of-bounds NaN
// fill), served from the cache when the same map was encoded before
bool encode4(CUtensorMap* map, CUtensorMapDataType dtype, const void* ptr,
             const cuuint64_t dims[4], const cuuint64_t strides[3], const cuuint32_t box[4],
             CUtensorMapSwizzle swizzle, CUtensorMapL2promotion l2) {
  MapKey k;
  memset(&k, 0, sizeof(k));  // padding takes part in the comparison
  k.dtype = dtype;
  k.swizzle = swizzle;
  k.l2 = l2;
  k.ptr = ptr;
  memcpy(k.dims, dims, sizeof(k.dims));
  memcpy(k.strides, strides, sizeof(k.strides));
  memcpy(k.box, box, sizeof(k.box));
  std::lock_guard<std::mutex> lock(g_cache_mu);
  for (int i = 0; i < kMapCache; ++i)
    if (g_maps[i].used && memcmp(&g_maps[i].key, &k, sizeof(k)) == 0) {
      *map = g_maps[i].map;
      return true;
    }
  const PFN_cuTensorMapEncodeTiled_v12000 encode = encode_fn();
  if (!encode) return false;
  cuuint32_t es[4] = {1u, 1u, 1u, 1u};
  const CUresult rc = encode(map, dtype, 4, const_cast<void*>(ptr), dims, strides, box, es,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, l2,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (rc != CUDA_SUCCESS) return false;
  MapEntry& e = g_maps[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  e.used = true;
  e.key = k;
  e.map = *map;
  return true;
}
}  // namespace

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return 0;
  std::lock_guard<std::mutex> lock(g_cache_mu);
  if (g_sms[dev] == 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return 0;
    g_sms[dev] = sms;
  }
  return g_sms[dev];
}

bool ensure_smem_attr(const void* func, int bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(g_cache_mu);
  for (int i = 0; i < g_nattrs; ++i)
    if (g_attrs[i].func == func && g_attrs[i].dev == dev && g_attrs[i].bytes >= bytes) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) !=
      cudaSuccess)
    return false;
  if (g_nattrs < 64) g_attrs[g_nattrs++] = AttrEntry{func, dev, bytes};
  return true;
}

static bool encode_bc_map_impl(CUtensorMap* map, const void* ptr, const Problem& p, const long long st[4]) {
  // interleaved: (B, T, H, 2N floats), box 64 steps x 2N floats of one head.
  // planar: (B, T, 2H, N floats) where row h is Re of head h and row H + h its Im (Im follows
  // Re by H*N floats in the in_proj layout), box 64 steps x N floats.
  const bool pl = p.bc_planar != 0;
  cuuint64_t dims[4] = {(cuuint64_t)(pl ? p.N : 2 * p.N), (cuuint64_t)(pl ? 2 * p.H : p.H),
                        (cuuint64_t)p.T, (cuuint64_t)p.Bsz};
  const cuuint64_t esz = pl ? 4u : 8u;
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * esz, (cuuint64_t)st[1] * esz,
                           (cuuint64_t)st[0] * esz};
  cuuint32_t box[4] = {pl ? 64u : 128u, 1u, 64u, 1u};
  return encode4(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ptr, dims, strides, box,
                 CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

bool encode_bc_tensor_map(CUtensorMap* map, const void* ptr, const Problem& p,
                          const long long st[4]) {
  return encode_bc_map_impl(map, ptr, p, st);
}

bool encode_out_tensor_map(CUtensorMap* map, void* ptr, const Problem& p, int row_floats) {
  const long long rf = row_floats;
  return encode_out_map_strided(map, ptr, p, row_floats, p.H, rf, rf * p.H, rf * p.H * p.T);
}

bool encode_out_map_bf16(CUtensorMap* map, void* ptr, const Problem& p) {
  if ((reinterpret_cast<uintptr_t>(ptr) % 16) != 0) return false;
  cuuint64_t dims[4] = {64u, (cuuint64_t)p.H, (cuuint64_t)p.T, (cuuint64_t)p.Bsz};
  cuuint64_t strides[3] = {128u, 128u * (cuuint64_t)p.H, 128u * (cuuint64_t)p.H * (cuuint64_t)p.T};
  cuuint32_t box[4] = {64u, 1u, 64u, 1u};
  return encode4(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, ptr, dims, strides, box,
                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

bool encode_out_map_strided(CUtensorMap* map, void* ptr, const Problem& p, int row_floats,
                            int rows, long long s_row, long long s_t, long long s_b) {
  if ((reinterpret_cast<uintptr_t>(ptr) % 16) != 0) return false;
  if (s_row <= 0 || s_t <= 0 || s_b <= 0 || s_row % 4 || s_t % 4 || s_b % 4) return false;
  cuuint64_t dims[4] = {(cuuint64_t)row_floats, (cuuint64_t)rows, (cuuint64_t)p.T,
                        (cuuint64_t)p.Bsz};
  cuuint64_t strides[3] = {(cuuint64_t)s_row * 4u, (cuuint64_t)s_t * 4u, (cuuint64_t)s_b * 4u};
  cuuint32_t box[4] = {32u, 1u, 64u, 1u};
  return encode4(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, ptr, dims, strides, box,
                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE);
}

bool fwd_supported(const Problem& p) {
  if (p.D != 64 || p.N != 64 || p.x_complex) return false;
  if (!bc_tma_ok(p, p.Bm, p.bs) || !bc_tma_ok(p, p.Cm, p.cs)) return false;
  const long long total = (long long)p.Bsz * p.H * ((p.T + 63) / 64);
  return total < (1ll << 30);
}

size_t states_bytes(const Problem& p) { return states_h_bytes(p) + chunk_prep_bytes(p); }

size_t fwd_workspace_bytes(const Problem& p) {
  const size_t nc = (size_t)((p.T + 63) / 64);
  return 256 + 4 * (size_t)p.Bsz * p.H * nc;
}

int run_fwd(const Problem& p, void* y, void* states, void* ws, cudaStream_t st, const void* h0,
            void* hT, int G, bool prep, bool clear_status, const void* recs_in, float2 crot,
            bool y_accum) {
  FwdParams fp{};
  fp.Bsz = p.Bsz;
  fp.T = p.T;
  fp.H = p.H;
  fp.nc = (p.T + 63) / 64;
  fp.total = p.Bsz * p.H * fp.nc;
  fp.x = static_cast<const float*>(p.x);
  for (int i = 0; i < 4; ++i) fp.xs[i] = p.xs[i];
  const uintptr_t xa = reinterpret_cast<uintptr_t>(p.x);
  const bool rows16 = p.xs[0] % 4 == 0 && p.xs[1] % 4 == 0 && p.xs[2] % 4 == 0;
  fp.x_vec = (p.xs[3] == 1 && rows16 && xa % 16 == 0) ? 1
             : (p.x_pair && p.xs[3] == 2 && rows16 && (xa & ~uintptr_t(4)) % 16 == 0)
                 ? 2 + (int)((xa >> 2) & 1)
                 : 0;
  fp.states = static_cast<float*>(states);
  ChunkRec* recs = recs_in != nullptr
                      ? static_cast<ChunkRec*>(const_cast<void*>(recs_in))
                      : reinterpret_cast<ChunkRec*>(static_cast<char*>(states) + states_h_bytes(p));
  fp.recs = recs;
  fp.crot = crot;
  fp.y_accum = y_accum ? 1 : 0;
  if (y_accum && p.y_bf16) return M3SSD_ERR_SHAPE;  // y accumulates in fp32 only
  uint32_t* w = static_cast<uint32_t*>(ws);
  fp.err = w;
  fp.counter = w + 1;
  fp.flags = w + 64;
  fp.y_bf16 = p.y_bf16;
  fp.h0 = static_cast<const float2*>(h0);
  fp.hT = static_cast<float2*>(hT);
  if (G < 1 || fp.nc % G != 0) return M3SSD_ERR_SHAPE;
  fp.G = G;
  fp.seg = fp.nc / G;
  CUtensorMap tmB, tmC, tmY;
  if (!encode_bc_tensor_map(&tmB, p.Bm, p, p.bs) || !encode_bc_tensor_map(&tmC, p.Cm, p, p.cs) ||
      !(p.y_bf16 ? encode_out_map_bf16(&tmY, y, p) : encode_out_tensor_map(&tmY, y, p, 64)))
    return M3SSD_ERR_LAUNCH;
  // status word (unless an earlier pass of the same call already reported into it), ticket
  // counter and hand-off flags start at zero
  const size_t keep = clear_status ? 0 : 4;
  if (cudaMemsetAsync(static_cast<char*>(ws) + keep, 0, fwd_workspace_bytes(p) - keep, st) !=
      cudaSuccess)
    return M3SSD_ERR_LAUNCH;
  if (prep) {
    const int rc = run_chunk_prep(p, recs, st);
    if (rc != M3SSD_OK) return rc;
  }
  const int sms = sm_count();
  if (sms <= 0) return M3SSD_ERR_DEVICE;
  // few independent chains (sequences x chains per sequence): the chunk-to-chunk hand-offs, ~4.3 us
  // each, take longer than the tickets' throughput (~39 ns each), so the state goes first
  const bool state_first = (double)p.Bsz * p.H * G * 0.039 < 4.3;
  auto kern = state_first
                  ? (p.bc_planar ? (G > 1 ? k_fwd_tc<true, true, true> : k_fwd_tc<true, false, true>)
                                 : (G > 1 ? k_fwd_tc<false, true, true> : k_fwd_tc<false, false, true>))
                  : (p.bc_planar ? (G > 1 ? k_fwd_tc<true, true, false> : k_fwd_tc<true, false, false>)
                                 : (G > 1 ? k_fwd_tc<false, true, false> : k_fwd_tc<false, false, false>));
  if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kSmemBytes))
    return M3SSD_ERR_LAUNCH;
  const int grid = fp.total < 2 * sms ? fp.total : 2 * sms;
  kern<<<grid, kThreads, kSmemBytes, st>>>(tmB, tmC, tmY, fp);
  return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace m3ssd

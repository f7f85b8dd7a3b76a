// Tensor-core backward of the complex chunkwise SSD for head_dim = state_dim = 64, real x.
//
// Persistent CTAs take chunk tickets in reverse chunk order. With the forward's rotated
// operands (C' = C cis(theta_l), B' = B conj(cis(theta_s)), Mr = exp(rho_l - rho_s) Re(C'B'^T)
// for s <= l, dec_s = exp(rho_Gamma - rho_s), e_l = exp(rho_l)) and dS_z the gradient of the
// state leaving chunk z (the reverse scan of the decay_chunk carry, models/ssd_complex.py:98-111):
//
//   dM  = dy x^T,  dG' = exp(rho_l - rho_s) dM  (s <= l)                 (through :50-53)
//   dx  = Mr^T dy + dec_s Re(conj(B') dS'),       dS' = conj(cis(theta_Gamma)) dS_z
//   dC' = dG' conj(B') + e_l dy conj(H_z)^T,      dC = dC' conj(cis(theta_l))   (:53, :115)
//   dB' = dG'^T conj(C') + dec_s x dS'^T,         dB = dB' cis(theta_s)          (:53, :54)
//   dS_{z-1} = e_l-weighted conj(C')^T dy + conj(e^Gamma) dS_z                    (carry)
//   d Sigma_l = sum_n dC conj(C) - sum_n dB conj(B) + [l = 63] <dS_z, H_{z+1}>
//   d a_t = reverse within-chunk cumsum of d Sigma;  ddt = Re(da conj(A)) softplus'(dt),
//   dA = sum da softplus(dt)                                                       (:82, :89)
//
// The d Sigma identity holds because every use of C[l] carries e^{Sigma_l}, every use of B[s]
// carries e^{-Sigma_s}, and Gamma enters only through H_{z+1}. Nine contractions per chunk run on
// tcgen05 (kind::f16) with split-bf16 operands stacked in groups of 8 rows (stack8) so each
// shared buffer serves as a stacked A operand and as a plain B operand. dS_z is handed from the
// CTA that processed chunk z+1 through one slot per chain in global memory (L2) with release flags.
// Warps: 16 workers (operand transforms, epilogues, carry), one control warp (tickets, every TMA
// and bulk copy, every MMA), one hand-off warp (the dS release and d Sigma -> ddt, dA partials).
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"
#include "tc_path.h"
#include "tc_trace.cuh"

namespace m3ssd {
namespace tc {

M3_TRACE_DEFINE(m3ssd_trace_set_bwd)

namespace {

constexpr int kWorkers = 512;              // warps 0-15: operand transforms and epilogues
constexpr int kCtlWarp = kWorkers / 32;    // warp 16: tickets, TMA/bulk loads and stores, MMA issue
constexpr int kRelWarp = kCtlWarp + 1;     // warp 17: publishes each ticket's dS hand-off
constexpr int kThreads = kWorkers + 64;
// shared memory map
constexpr uint32_t OFF_C = 0;        // C'x stacked [2 k-atoms][128][64]; raw C tile lands first
constexpr uint32_t OFF_B = 32768;    // B'x (conjugate-interleaved) stacked; raw B tile lands first
constexpr uint32_t OFF_X = 65536;    // x stacked over s [128][64 p]
constexpr uint32_t OFF_DY = 81920;   // dy stacked over l [128][64 p]
constexpr uint32_t OFF_DYT = 98304;  // e_l dy stacked over p, MN [2][64 l][64]; then Mr (same form)
constexpr uint32_t OFF_DGK = 114688; // dG' stacked over l [128][64 s]
constexpr uint32_t OFF_DGM = 131072; // dG' stacked over s, MN [2][64 l][64]
constexpr uint32_t OFF_DS = 147456;  // dS_z (fp32, lands by bulk copy), then dS'x hi | lo
constexpr uint32_t OFF_H = 180224;   // H_z (fp32, lands by bulk copy), then conj(H_z) hi | lo
constexpr uint32_t OFF_MISC = 212992;
constexpr uint32_t kMiscBytes = 13312;
constexpr uint32_t kSmemBytes = OFF_MISC + kMiscBytes + 1024;
constexpr uint32_t kLoadBytes = 64u * 128u * 4u + (uint32_t)sizeof(ChunkRec);  // C tile + record
constexpr uint32_t kTmemCols = 512;
// dS hand-off slots per chain. One is enough: the chunk z ticket's bulk load of dS_z has landed
// (bar_ds) before its workers store dS_{z-1} over it, and only that ticket reads dS_z. A single
// 32 KB slot per chain keeps the ring small enough to stay in L2 between its write and its read
// (with four, the slots' lines were evicted and written back to DRAM: ~0.2 GB per block-shape call).
constexpr int kRingSlots = 1;
// TMEM columns: batch 1, batch 2, batch 3 (reusing batch-1 columns), dBb (reusing dCa)
constexpr uint32_t COL_G = 0, COL_DM = 64, COL_Q = 128, COL_DCA = 256, COL_DCB = 384;
constexpr uint32_t COL_DXA = 0, COL_DXB = 64, COL_DBA = 128, COL_DBB = 256;

struct Misc {
  ChunkRec rec[2];  // decay records of the current and the next ticket
  // control -> workers: C tile + record landed, B tile landed, H_z landed, dS landed, ticket
  // published, MMA commits 1..4, and the staging buffers of the previous ticket's dx / dB stores
  // read (stfree)
  uint64_t bar_tma, bar_tmb, bar_h, bar_ds, bar_ctl, bar1, bar2, bar3, bar4, bar_stfree;
  // workers -> control (one arrival per worker warp): opa x, dy, e dy written; opc C'; ops1 B';
  // oph conj(H); ops2 dS' written and epilogue 1 done; ops3 carry done; colfree dCa's columns
  // read; dc / dx / db staging tiles written. Every wait is on the phase of the current ticket:
  // no barrier can complete twice before its waiter looks, so a parity never repeats under one.
  uint64_t bar_opa, bar_opc, bar_oph, bar_ops1, bar_ops2, bar_ops3, bar_colfree, bar_dc, bar_dx,
      bar_db;
  // by ticket parity, read by the hand-off warp after the workers are done with the ticket:
  float4 dgam[2];       // <dS_z, H_{z+1}> from the chunk z+1 ticket (lands with dS_z)
  float2 rc[2][4][64];  // sum_n dC'_{ln} conj(C'_{ln}) over the four 16-state column groups
  float2 rb[2][4][64];  // sum_n dB'_{sn} conj(B'_{sn})
  float2 dgp[2][kWorkers / 32];  // per-warp partials of <dS_{z-1}, H_z>
  // hand-off warp -> control and workers: a ticket's dS hand-off is published and its d Sigma
  // is done (the control publishes ticket i + 1 and the workers finish the carry of ticket i + 1
  // only after ticket i - 1 is, so no wait of the hand-off warp ever sees a phase parity repeat)
  uint64_t bar_rel;
  int tick[2];
  uint32_t tmem_base;
};
static_assert(sizeof(Misc) <= kMiscBytes, "misc area");

struct BwdParams {
  int Bsz, T, H, nc, total;
  const float* x;
  long long xs[4];
  int x_vec;
  const void* dy;  // float32, or bfloat16 with dy_bf16
  long long dys[4];
  int dy_vec;
  int dy_bf16;
  const float2* A;
  const float2* Bm;
  long long bs[4];
  const float2* Cm;
  long long cs[4];
  const ChunkRec* recs;
  const float* states;
  float* ddt;
  long long ddt_sb, ddt_st;  // ddt[b, t, h] at b * ddt_sb + t * ddt_st + h
  int hp;                    // planar B / C and dB / dC: H (the Im rows' offset), else 0
  float2* dapart;
  float* ring;
  float4* dgring;
  uint32_t* flags;
  uint32_t* counter;
  uint32_t* err;
  // state carry (optional): gradient of the final state in, of the initial state out, both
  // (B, H, N, D) complex64 = the transpose of a state tile; <dhT, hT> per sequence (the
  // [l = 63] d Sigma term of the last chunk)
  const float2* dhT;
  float2* dh0;
  const float2* dgam_last;
  int G, seg;  // chains per sequence and chunks per chain (see TicketPos)
  // the complex-x second pass (see run_bwd_complex): C is multiplied by crot as it is read (dC then
  // takes conj(crot) of its gradient), and dB, dC, ddt and the dA partials are added to what the
  // first pass left (accum)
  float2 crot;
  int accum;
};

// (sequence, chunk) of a ticket: tickets run over sequences (then segments) fastest, chunks
// within a segment in reverse order. Each sequence's chunks form G chains of seg = nc / G chunks
// (G = 1: one chain); a chain's last chunk takes dS from dhT (or zero) and its first chunk's
// carry is the chain's entry-state gradient. sg = bh * G + segment indexes per-chain data.
struct TicketPos {
  int bh, z, b, h, sg;
  bool first, last;
};
template <bool kChains>
__device__ __forceinline__ TicketPos ticket_pos(int tk, int BH, int H, int G, int seg) {
  TicketPos q;
  if constexpr (!kChains) {  // one chain per sequence (seg = nc)
    const int zr = tk / BH;
    q.bh = q.sg = tk - zr * BH;
    q.z = seg - 1 - zr;
    q.first = q.z == 0;
    q.last = zr == 0;
    q.b = q.bh / H;
    q.h = q.bh - q.b * H;
    return q;
  }
  const int zr = tk / (BH * G);
  const int rest = tk - zr * BH * G;
  const int sgm = rest / BH;
  q.bh = rest - sgm * BH;
  const int j = seg - 1 - zr;
  q.z = sgm * seg + j;
  q.sg = q.bh * G + sgm;
  q.first = j == 0;
  q.last = j == seg - 1;
  q.b = q.bh / H;
  q.h = q.bh - q.b * H;
  return q;
}

// Four K-steps of one accumulation, operand descriptors advancing by AS / BS bytes per step (the
// descriptor's address field holds address >> 4). Fully unrolled: issued from a loop, each
// tcgen05.mma waits on the previous iteration's bookkeeping, and the batches ran ~1.7x slower.
// Starts the accumulator over when `fresh`.
template <uint32_t AS, uint32_t BS>
__device__ __forceinline__ void mma_run4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc,
                                         bool fresh) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    mma_bf16_ss(d, a + (uint64_t)(j * (AS >> 4)), b + (uint64_t)(j * (BS >> 4)), idesc,
                (fresh && j == 0) ? 0u : 1u);
}

// ---------------------------------------------------------------- control-warp helpers
// (out of line: each runs once per ticket, and the kernel must stay small for the I-cache)
// C tile and decay record (bar_tma), once the epilogue of dC has read sC; B tile (bar_tmb) once the
// epilogue of dB has read sB
// (hp > 0: planar tiles, the real part into the first 16 KB and the imaginary part, row hp + h of
// the map, into the second)
static __device__ __noinline__ void ctl_load_c(const CUtensorMap* tmC, uint8_t* smem, Misc* m,
                                               const ChunkRec* recs, int nc, TicketPos q, int slot,
                                               int hp) {
  mbar_arrive_expect_tx(&m->bar_tma, kLoadBytes);
  tma_load_4d(smem + OFF_C, tmC, &m->bar_tma, 0, q.h, q.z * 64, q.b);
  if (hp > 0) tma_load_4d(smem + OFF_C + 16384, tmC, &m->bar_tma, 0, hp + q.h, q.z * 64, q.b);
  bulk_load(&m->rec[slot], recs + (long long)q.bh * nc + q.z, (uint32_t)sizeof(ChunkRec),
            &m->bar_tma);
}
static __device__ __noinline__ void ctl_load_b(const CUtensorMap* tmB, uint8_t* smem, Misc* m,
                                               TicketPos q, int hp) {
  mbar_arrive_expect_tx(&m->bar_tmb, 64u * 128u * 4u);
  tma_load_4d(smem + OFF_B, tmB, &m->bar_tmb, 0, q.h, q.z * 64, q.b);
  if (hp > 0) tma_load_4d(smem + OFF_B + 16384, tmB, &m->bar_tmb, 0, hp + q.h, q.z * 64, q.b);
}
static __device__ __noinline__ void ctl_load_h(uint8_t* smem, Misc* m, const float* states, int nc,
                                               TicketPos q) {
  mbar_arrive_expect_tx(&m->bar_h, 32768u);
  bulk_load(smem + OFF_H, states + ((long long)q.bh * nc + q.z) * 64 * 128, 32768u, &m->bar_h);
}
// dS_z (and <dS_z, H_{z+1}>) from the chunk z+1 ticket once its flag is published
static __device__ __noinline__ void ctl_load_ds(uint8_t* smem, Misc* m, const float* ring,
                                                const float4* dgring, const uint32_t* flags,
                                                uint32_t* err, int nc, TicketPos q, int slot) {
  if (q.last) {
    mbar_arrive(&m->bar_ds);
    return;
  }
  flag_wait(flags + (long long)q.bh * nc + q.z, err);
  fence_proxy_async_global();  // the ring was written with plain stores by another CTA
  mbar_arrive_expect_tx(&m->bar_ds, 32768u + 16u);
  bulk_load(smem + OFF_DS, ring + ((long long)q.sg * kRingSlots + (q.z % kRingSlots)) * 64 * 128,
            32768u,
            &m->bar_ds);
  bulk_load(&m->dgam[slot], dgring + (long long)q.sg * kRingSlots + (q.z % kRingSlots), 16u,
            &m->bar_ds);
}
// TMA stores of a 64-row output tile from its 32-float staging segments (segments 0, 1 at off01,
// 2, 3 at off23), one bulk group. hp > 0: planar complex tile, segments 0, 1 hold the real parts
// (row h of the map) and 2, 3 the imaginary parts (row hp + h).
static __device__ __noinline__ void ctl_store_tile(const CUtensorMap* map, uint8_t* smem,
                                                   uint32_t off01, uint32_t off23, int nseg,
                                                   TicketPos q, int hp, bool accum) {
  for (int seg = 0; seg < nseg; ++seg)
    tma_put_4d(map, smem + (seg < 2 ? off01 : off23) + (seg & 1) * 8192,
               hp > 0 ? 32 * (seg & 1) : 32 * seg, hp > 0 ? q.h + hp * (seg >> 1) : q.h,
               q.z * 64, q.b, accum);
  bulk_commit_group();
}

// 8 consecutive bfloat16 values widened to float (zeros past the end of the sequence)
__device__ __forceinline__ void load8_bf16(const __nv_bfloat16* base, long long pstride, int vec,
                                           bool valid, int p0, float* v) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return;
  }
  if (vec) {
    uint4 q;
    asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(q.x), "=r"(q.y), "=r"(q.z), "=r"(q.w)
                 : "l"(base + p0));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __bfloat162float(base[(long long)(p0 + i) * pstride]);
  }
}

// 8 consecutive floats x[b, t, h, p0 .. p0+7] (zeros past the end of the sequence)
__device__ __forceinline__ void load8(const float* base, long long pstride, int vec, bool valid,
                                      int p0, float* v) {
  if (!valid) {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    return;
  }
  if (vec) {
    const float4 q0 = ldg_nc_v4(base + p0), q1 = ldg_nc_v4(base + p0 + 4);
    v[0] = q0.x; v[1] = q0.y; v[2] = q0.z; v[3] = q0.w;
    v[4] = q1.x; v[5] = q1.y; v[6] = q1.z; v[7] = q1.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __ldg(base + (long long)(p0 + i) * pstride);
  }
}

__device__ __forceinline__ float2 cmul2(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

__device__ __forceinline__ void split8_store(uint32_t hi_addr, uint32_t lo_addr, const float* v) {
  float w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = v[i];
  uint4 h, l;
  split8(w, h, l);
  st_shared_v4(hi_addr, h);
  st_shared_v4(lo_addr, l);
}

// the issuing warp's lane arrives once every lane's shared-memory writes are visible to the
// async proxy (tensor core, TMA) and its TMEM reads are complete
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  fence_proxy_async_smem();
  tc_fence_before_sync();
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

__device__ __forceinline__ void workers_sync() { named_sync(1, kWorkers); }

// fp32 staging tile for a TMA store: 32-float column segment of a 64-row tile, 128-byte rows,
// 16-byte chunks swizzled by row (the CU_TENSOR_MAP_SWIZZLE_128B layout)
__device__ __forceinline__ uint32_t stage_addr(uint32_t seg_base, uint32_t row, uint32_t chunk) {
  return seg_base + row * 128u + ((chunk ^ (row & 7u)) << 4);
}
// segment s of a staged tile whose segments 0, 1 sit at seg01 and 2, 3 at seg23
__device__ __forceinline__ uint32_t stage_seg(uint32_t seg01, uint32_t seg23, uint32_t s) {
  return (s < 2u ? seg01 : seg23) + (s & 1u) * 8192u;
}

// ---------------------------------------------------------------- worker helpers (out of line)
// The same epilogue over a warp's 32 accumulator columns (16 complex) in the 16x256b TMEM layout:
// the hi-row and lo-row partials of a logical row sit 8 lanes apart (stack8), which that load shape
// hands to the same thread, so they add in registers (no shuffle, no select). Thread t of the
// warp in lane quadrant `sub` and column group `grp` takes logical rows 16 sub + t/4 (lanes +0..15)
// and 16 sub + 8 + t/4 (lanes +16..31), complex 16 grp + 4 k + t%4 for k = 0..3. Staging: fp32
// interleaved in segment grp, or (kPlanar) Re in segment grp/2 and Im in 2 + grp/2. Row sums
// sum v conj(X) with X the split operand at xop (k-atom grp/2), reduced over the quad; returns
// them for both rows (every lane of a quad holds the quad's sums).
template <bool kPlanar>
__device__ __forceinline__ void combine_rows2(uint32_t ta, uint32_t tb, const float* wrow,
                                              const float2* rotrow, bool conj_out,
                                              uint32_t seg01, uint32_t seg23, int sub, int grp,
                                              uint32_t xop, uint64_t* colfree, int lane,
                                              float2& acc_a, float2& acc_b, uint32_t it,
                                              int tslot, float2 extra) {
  const int q4 = lane & 3, rr = lane >> 2;
  const float cj = conj_out ? -1.f : 1.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    float a[16], bb[16];
    tmem_ld16x256_x4(ta + ((uint32_t)(16 * half) << 16), a);
    tmem_ld16x256_x4(tb + ((uint32_t)(16 * half) << 16), bb);
    tmem_ld_wait();
    if ((threadIdx.x >> 5) == 0) M3_TRACE(it, tslot + 2 * half);
    if (half == 1 && colfree != nullptr) warp_arrive(colfree, lane);
    const uint32_t row = (uint32_t)(16 * sub + 8 * half + rr);
    const float w = wrow[row];
    const float2 rot = cmul2(rotrow[row], extra);
    const float2 nr = make_float2(rot.x, -rot.y);
    const uint32_t xrow = stack8(row, 0u);  // its lo part is 8 stacked rows (1024 bytes) on
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 v = make_float2((a[4 * k] + a[4 * k + 2]) + w * (bb[4 * k] + bb[4 * k + 2]),
                                   (a[4 * k + 1] + a[4 * k + 3]) + w * (bb[4 * k + 1] + bb[4 * k + 3]));
      // X: bf16 hi | lo pair of complex 16 grp + 4k + q4, 16-byte chunk 4 (grp mod 2) + k
      const uint32_t xa =
          xop + swz(xrow, 4u * ((uint32_t)grp & 1u) + (uint32_t)k) + 4u * (uint32_t)q4;
      const float2 xv = unsplit2(ld_shared_u32(xa), ld_shared_u32(xa + 1024u));
      acc.x += v.x * xv.x + v.y * xv.y;
      acc.y += v.y * xv.x - v.x * xv.y;
      const float2 r2 = cmul2(v, nr);
      if constexpr (kPlanar) {
        const uint32_t ch = 4u * ((uint32_t)grp & 1u) + (uint32_t)k;
        st_shared_f32(stage_addr(stage_seg(seg01, seg23, (uint32_t)grp >> 1), row, ch) + 4u * q4,
                      r2.x);
        st_shared_f32(stage_addr(stage_seg(seg01, seg23, 2u + ((uint32_t)grp >> 1)), row, ch) +
                          4u * q4,
                      cj * r2.y);
      } else {
        st_shared_f2(stage_addr(stage_seg(seg01, seg23, (uint32_t)grp), row,
                                2u * (uint32_t)k + ((uint32_t)q4 >> 1)) +
                         8u * ((uint32_t)q4 & 1u),
                     r2.x, cj * r2.y);
      }
    }
#pragma unroll
    for (int o = 1; o <= 2; o <<= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, o);
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, o);
    }
    if (half == 0) acc_a = acc; else acc_b = acc;
    if ((threadIdx.x >> 5) == 0) M3_TRACE(it, tslot + 2 * half + 1);
  }
}

}  // namespace

// kPlanar: B and C arrive, and dB and dC leave, as separate real and imaginary tiles (the in_proj
// column layout); everything else is shared
// kCarryFirst: the workers form the carry (and so release dS_{z-1} to the next chunk's ticket)
// before epilogue 1 instead of after it: for problems with few independent chains, whose time is
// the chain of chunk-to-chunk hand-offs rather than the tickets' throughput
template <bool kPlanar, bool kChains, bool kCarryFirst>
__global__ void __launch_bounds__(kThreads, 1)
    k_bwd_tc(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
             const __grid_constant__ CUtensorMap tmDX, const __grid_constant__ CUtensorMap tmDB,
             const __grid_constant__ CUtensorMap tmDC, const BwdParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sb = smem_u32(smem);
  Misc& m = *reinterpret_cast<Misc*>(smem + OFF_MISC);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int BH = p.Bsz * p.H;

  if (tid == 0) {
    uint64_t* one[11] = {&m.bar_tma, &m.bar_tmb, &m.bar_h, &m.bar_ds,     &m.bar_ctl, &m.bar1,
                         &m.bar2,    &m.bar3,    &m.bar4,  &m.bar_stfree, &m.bar_rel};
    uint64_t* eight[10] = {&m.bar_opa,  &m.bar_opc, &m.bar_oph,     &m.bar_ops1, &m.bar_ops2,
                           &m.bar_ops3, &m.bar_dc,  &m.bar_colfree, &m.bar_dx,   &m.bar_db};
#pragma unroll
    for (int i = 0; i < 11; ++i) mbar_init(one[i], 1);
#pragma unroll
    for (int i = 0; i < 10; ++i) mbar_init(eight[i], kWorkers / 32);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(&m.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = m.tmem_base;

  if (warp == kRelWarp) {
    // ================================ hand-off warp ================================
    // Per ticket, off the workers' and the control's paths:
    //  * once the workers' carries are done (bar_ops3), lane 0 publishes dS_{z-1} and
    //    <dS_{z-1}, H_z> for the chunk z-1 ticket. The release's fence holds its thread ~1 us
    //    (longer with the same thread's stores or bulk copies in flight).
    //  * once the workers' dB epilogue is done (bar_db; the dC one came before), d Sigma ->
    //    reverse cumsum -> ddt and the chunk's dA partial: lane L takes positions L and L + 32,
    //    each half is scanned within the warp, then the upper half's total is added to the lower.
    // Every wait is on the current ticket's phase (bar_rel back-pressure, see Misc).
    mbar_wait(&m.bar_ctl, 0u, p.err, kErrMmaWait);
    int cur = m.tick[0];
    uint32_t it = 0;
    while (cur < p.total) {
      const uint32_t ph = it & 1u;
      const TicketPos q = ticket_pos<kChains>(cur, BH, p.H, p.G, p.seg);
      const float2 Ah = p.A[q.h];
      mbar_wait(&m.bar_ops3, ph, p.err, kErrMmaWait);
      mbar_wait(&m.bar_ctl, ph ^ 1u, p.err, kErrMmaWait);
      const int nxt = m.tick[(it + 1) & 1];
      if (lane == 0 && !q.first) {
        float2 dg = make_float2(0.f, 0.f);
#pragma unroll
        for (int w = 0; w < kWorkers / 32; ++w) {
          dg.x += m.dgp[ph][w].x;
          dg.y += m.dgp[ph][w].y;
        }
        __stcg(p.dgring + (long long)q.sg * kRingSlots + ((q.z - 1) % kRingSlots),
               make_float4(dg.x, dg.y, 0.f, 0.f));
        // the workers' ring stores happened before their bar_ops3 arrivals
        fence_proxy_async_global();
        st_release_gpu(p.flags + (long long)q.bh * p.nc + q.z - 1, 1u);
      }
      __syncwarp();
      // the row sums of this ticket are in once every worker warp has arrived at bar_db; its
      // record slot and <dS_z, H_{z+1}> are not reloaded before this warp's bar_rel arrival
      mbar_wait(&m.bar_db, ph, p.err, kErrMmaWait);
      M3_TRACE(it, 31);
      {
        const ChunkRec& rec = m.rec[ph];
        const float2 dgam = !q.last ? make_float2(m.dgam[ph].x, m.dgam[ph].y)
                            : p.dgam_last != nullptr ? p.dgam_last[q.sg]
                                                     : make_float2(0.f, 0.f);
        const int t0 = q.z * 64;
        float2 dv[2];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int l = lane + 32 * u;
          dv[u] = make_float2(
              (m.rc[ph][0][l].x + m.rc[ph][1][l].x) + (m.rc[ph][2][l].x + m.rc[ph][3][l].x) -
                  ((m.rb[ph][0][l].x + m.rb[ph][1][l].x) + (m.rb[ph][2][l].x + m.rb[ph][3][l].x)),
              (m.rc[ph][0][l].y + m.rc[ph][1][l].y) + (m.rc[ph][2][l].y + m.rc[ph][3][l].y) -
                  ((m.rb[ph][0][l].y + m.rb[ph][1][l].y) + (m.rb[ph][2][l].y + m.rb[ph][3][l].y)));
        }
        if (lane == 31) {
          dv[1].x += dgam.x;
          dv[1].y += dgam.y;
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {  // suffix sums within each half
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const float ux = __shfl_down_sync(0xffffffffu, dv[u].x, o);
            const float uy = __shfl_down_sync(0xffffffffu, dv[u].y, o);
            if (lane + o < 32) {
              dv[u].x += ux;
              dv[u].y += uy;
            }
          }
        }
        const float2 hi_total = make_float2(__shfl_sync(0xffffffffu, dv[1].x, 0),
                                            __shfl_sync(0xffffffffu, dv[1].y, 0));
        const float2 s0 = make_float2(dv[0].x + hi_total.x, dv[0].y + hi_total.y);
        const float2 s1 = dv[1];
        float2 dap[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int l = lane + 32 * u, t = t0 + l;
          const float2 da = u ? s1 : s0;
          if (t < p.T) {
            float* dst = p.ddt + q.b * p.ddt_sb + (long long)t * p.ddt_st + q.h;
            const float v = (da.x * Ah.x + da.y * Ah.y) * rec.dsp[l];
            *dst = p.accum ? *dst + v : v;
            dap[u] = make_float2(da.x * rec.sp[l], da.y * rec.sp[l]);
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            dap[u].x += __shfl_xor_sync(0xffffffffu, dap[u].x, o);
            dap[u].y += __shfl_xor_sync(0xffffffffu, dap[u].y, o);
          }
        }
        if (lane == 0)
          p.dapart[(long long)q.bh * p.nc + q.z] =
              make_float2(dap[0].x + dap[1].x, dap[0].y + dap[1].y);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&m.bar_rel);
      cur = nxt;
      ++it;
    }
  } else if (warp == kCtlWarp) {
    // =============================== control warp (lane 0) ===============================
    if (lane == 0) {
      prefetch_tmap(&tmB);
      prefetch_tmap(&tmC);
      prefetch_tmap(&tmDX);
      prefetch_tmap(&tmDB);
      prefetch_tmap(&tmDC);
      int cur = (int)atomicAdd(p.counter, 1u);
      m.tick[0] = cur;
      mbar_arrive(&m.bar_ctl);
      TicketPos qc = ticket_pos<kChains>(cur, BH, p.H, p.G, p.seg);
      if (cur < p.total) {
        ctl_load_c(&tmC, smem, &m, p.recs, p.nc, qc, 0, p.hp);
        ctl_load_b(&tmB, smem, &m, qc, p.hp);
        ctl_load_h(smem, &m, p.states, p.nc, qc);
        ctl_load_ds(smem, &m, p.ring, p.dgring, p.flags, p.err, p.nc, qc, 0);
      }
      uint32_t it = 0;
      while (cur < p.total) {
        const uint32_t ph = it & 1u;
        // claim the next ticket now; its value is only needed when it is published after batch 1
        const int nxt = (int)atomicAdd(p.counter, 1u);
        // batch 1, each contraction once its operands are converted: dM = dy x^T, then
        // Q^T = (e dy)^T C'x, G = C'x B'x^T (the commit after G covers these three), then
        // dCb = dy conj(H)^T (columns nobody else uses; the next commit covers it)
        const uint32_t id64 = idesc_bf16(128, 64, 0, 0), idq = idesc_bf16(128, 128, 1, 1);
        const uint32_t id128 = idesc_bf16(128, 128, 0, 1);
        mbar_wait(&m.bar_opa, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 21);
        tc_fence_after_sync();
#pragma unroll
        for (int hp = 0; hp < 2; ++hp)
          mma_run4<32, 32>(tmem + COL_DM, sdesc(sb + OFF_DY, 16, 1024),
                           sdesc(sb + OFF_X + hp * 1024u, 16, 2048), id64, hp == 0);
        mbar_wait(&m.bar_opc, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 22);
        tc_fence_after_sync();
#pragma unroll
        for (int hp = 0; hp < 2; ++hp)
          mma_run4<2048, 4096>(tmem + COL_Q, sdesc(sb + OFF_DYT, 8192, 1024),
                               sdesc(sb + OFF_C + hp * 1024u, 16384, 2048), idq, hp == 0);
        mbar_wait(&m.bar_ops1, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 23);
        tc_fence_after_sync();
#pragma unroll
        for (int hp = 0; hp < 2; ++hp)
#pragma unroll
          for (int ka = 0; ka < 2; ++ka)
            mma_run4<32, 32>(tmem + COL_G, sdesc(sb + OFF_C + ka * 16384u, 16, 1024),
                             sdesc(sb + OFF_B + ka * 16384u + hp * 1024u, 16, 2048), id64, hp == 0 && ka == 0);
        mma_commit(&m.bar1);
        mbar_wait(&m.bar_oph, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 24);
        tc_fence_after_sync();
#pragma unroll
        for (int hp = 0; hp < 2; ++hp)
          mma_run4<32, 2048>(tmem + COL_DCB, sdesc(sb + OFF_DY, 16, 1024),
                             sdesc(sb + OFF_H + hp * 16384u, 8192, 1024), id128, hp == 0);
        // publish the next ticket (workers prefetch its x and dy), once the hand-off warp is done
        // with the ticket before this one (so no waiter ever sees a phase parity repeat)
        if (it > 0) mbar_wait(&m.bar_rel, (it - 1) & 1u, p.err, kErrMmaWait);
        m.tick[(it + 1) & 1] = nxt;
        mbar_arrive(&m.bar_ctl);
        const TicketPos qn = ticket_pos<kChains>(nxt, BH, p.H, p.G, p.seg);
        // Each remaining contraction as soon as its operands are written and its TMEM columns
        // read.
        // After epilogue 1 (dG', Mr written; G, dM read): dCa = dG' conj(B'), dXa = Mr^T dy,
        // dXb = conj(B') dS' into the columns of G and dM
        mbar_wait(&m.bar_ops2, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 25);
        tc_fence_after_sync();
        {
#pragma unroll
          for (int hp = 0; hp < 2; ++hp)
            mma_run4<32, 4096>(tmem + COL_DCA, sdesc(sb + OFF_DGK, 16, 1024),
                               sdesc(sb + OFF_B + hp * 1024u, 16384, 2048), id128, hp == 0);
          mma_commit(&m.bar2);
          const uint32_t idxa = idesc_bf16(128, 64, 1, 1), idxb = idesc_bf16(128, 64, 0, 0);
#pragma unroll
          for (int hp = 0; hp < 2; ++hp) {
            mma_run4<2048, 4096>(tmem + COL_DXA, sdesc(sb + OFF_DYT, 8192, 1024),
                                 sdesc(sb + OFF_DY + hp * 1024u, 8192, 2048), idxa, hp == 0);
#pragma unroll
            for (int ka = 0; ka < 2; ++ka)
              mma_run4<32, 32>(tmem + COL_DXB, sdesc(sb + OFF_B + ka * 16384u, 16, 1024),
                               sdesc(sb + OFF_DS + hp * 16384u + ka * 8192u, 16, 1024), idxb, hp == 0 && ka == 0);
          }
          mma_commit(&m.bar3);
        }
        // after the carry (Q read): dBa = dG'^T conj(C') into the columns of Q
        mbar_wait(&m.bar_ops3, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 26);
        tc_fence_after_sync();
        {
          const uint32_t idba = idesc_bf16(128, 128, 1, 1);
#pragma unroll
          for (int hp = 0; hp < 2; ++hp)
            mma_run4<2048, 4096>(tmem + COL_DBA, sdesc(sb + OFF_DGM, 8192, 1024),
                                 sdesc(sb + OFF_C + hp * 1024u, 16384, 2048), idba, hp == 0);
        }
        // dBb = x dS'x^T (MN) into the columns dCa used, once the workers have read them; its
        // commit also covers dBa
        mbar_wait(&m.bar_colfree, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 27);
        tc_fence_after_sync();
        {
          const uint32_t idbb = idesc_bf16(128, 128, 0, 1);
#pragma unroll
          for (int hp = 0; hp < 2; ++hp)
            mma_run4<32, 2048>(tmem + COL_DBB, sdesc(sb + OFF_X, 16, 1024),
                               sdesc(sb + OFF_DS + hp * 16384u, 8192, 1024), idbb, hp == 0);
          mma_commit(&m.bar4);
        }
        // dC from its staging tile in sH; the epilogue of dC has read sC, and once dBa has too,
        // the next C tile and record (its slot was the previous ticket's, which every worker warp
        // finished before arriving at bar_ops1 of this one); the next H_z into sH once the store
        // has read it
        mbar_wait(&m.bar_dc, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 28);
        ctl_store_tile(&tmDC, smem, OFF_H, OFF_H + 16384u, 4, qc, p.hp, p.accum != 0);
        if (nxt < p.total) {
          mbar_wait(&m.bar4, ph, p.err, kErrMmaWait);
          ctl_load_c(&tmC, smem, &m, p.recs, p.nc, qn, (int)((it + 1) & 1), p.hp);
        }
        bulk_wait_read_all();
        if (nxt < p.total) ctl_load_h(smem, &m, p.states, p.nc, qn);
        // dx from sDGK, dB from sDYT / sDGM; the next B tile (the epilogue of dB has read sB) and
        // the next dS (dBb has read sDS)
        mbar_wait(&m.bar_dx, ph, p.err, kErrMmaWait);
        ctl_store_tile(&tmDX, smem, OFF_DGK, OFF_DGK, 2, qc, 0, false);
        mbar_wait(&m.bar_db, ph, p.err, kErrMmaWait);
        M3_TRACE(it, 29);
        ctl_store_tile(&tmDB, smem, OFF_DYT, OFF_DGM, 4, qc, p.hp, p.accum != 0);
        if (nxt < p.total) ctl_load_b(&tmB, smem, &m, qn, p.hp);
        bulk_wait_read_all();
        mbar_arrive(&m.bar_stfree);
        if (nxt < p.total)
          ctl_load_ds(smem, &m, p.ring, p.dgring, p.flags, p.err, p.nc, qn, (int)((it + 1) & 1));
        M3_TRACE(it, 30);
        cur = nxt;
        qc = qn;
        ++it;
      }
      bulk_wait_all();
    }
    __syncwarp();
  } else {
    // =============================== worker warps 0-15 ===============================
    // TMEM lane quadrant sub = warp mod 4; column group grp = warp / 4 takes 32 of the 128
    // columns of a complex accumulator (16 of a 64-column one). Accumulators are read in the
    // 16x256b shape: each thread gets two logical rows (16 sub + 8 h + lane/4) and column pairs
    // 8 k + 2 (lane%4), +1 of the warp's columns, with the hi and lo partial rows (8 lanes apart
    // in the stacking) both in its registers.
    const int sub = warp & 3, grp = warp >> 2;
    const uint32_t lane_off = (uint32_t)(32 * sub) << 16;
    // x / dy staging: row xs0, columns 8 (tid & 7) .. + 7 (8 lanes per row)
    const int xs0 = tid >> 3, xp0 = 8 * (tid & 7);
    mbar_wait(&m.bar_ctl, 0u, p.err, kErrMmaWait);
    int next = m.tick[0];
    // The loop turns between tickets: the epilogues of the ticket in flight run (x and dy of
    // ticket `next` are loaded into registers during them), then ticket `next` starts.
    bool active = false;  // a ticket's epilogues are pending
    uint32_t it = 0;      // index of that ticket
    TicketPos q{};
    int t0 = 0;
    for (;;) {
      // x and dy rows of ticket `next`: pulled into L2 during the epilogues (a register prefetch
      // would keep 16 registers live through them and spill at this kernel's register budget);
      // the register loads follow at the start of that ticket
      auto prefetch_l2 = [&]() {
        if (next < p.total) {
          const TicketPos qx = ticket_pos<kChains>(next, BH, p.H, p.G, p.seg);
          const int tx = qx.z * 64 + xs0;
          if (tx < p.T) {
            prefetch_l2_line(p.x + qx.b * p.xs[0] + (long long)tx * p.xs[1] + qx.h * p.xs[2] +
                             (long long)xp0 * p.xs[3]);
            const long long go = qx.b * p.dys[0] + (long long)tx * p.dys[1] +
                                 qx.h * p.dys[2] + (long long)xp0 * p.dys[3];
            prefetch_l2_line(static_cast<const char*>(p.dy) + go * (p.dy_bf16 ? 2 : 4));
          }
        }
      };
      if (active) {
        const uint32_t ph = it & 1u;
        const ChunkRec& rec = m.rec[ph];
        // ---- epilogue 2: dC = (dCa + e_l dCb) conj(cis(theta_l)) -> staging tile in sH, once
        // every warp's carry has read conj(H_z) there (bar2 can complete before that)
        mbar_wait(&m.bar_ops3, ph, p.err, kErrMmaWait);
        mbar_wait(&m.bar2, ph, p.err, kErrMmaWait);
        if (warp == 0) M3_TRACE(it, 15);
        prefetch_l2();
        tc_fence_after_sync();
        {
          float2 acc_a, acc_b;
          combine_rows2<kPlanar>(tmem + lane_off + COL_DCA + 32u * grp,
                                 tmem + lane_off + COL_DCB + 32u * grp, rec.el, rec.cis, false,
                                 sb + OFF_H, sb + OFF_H + 16384u, sub, grp,
                                 sb + OFF_C + ((uint32_t)grp >> 1) * 16384u, &m.bar_colfree, lane,
                                 acc_a, acc_b, it, 32, p.crot);
          if ((lane & 3) == 0) {
            m.rc[ph][grp][16 * sub + (lane >> 2)] = acc_a;
            m.rc[ph][grp][16 * sub + 8 + (lane >> 2)] = acc_b;
          }
        }
        warp_arrive(&m.bar_dc, lane);
        if (warp == 0) M3_TRACE(it, 16);

        // ---- epilogue 3: dx = dXa + dec_s dXb -> staging tile in sDGK
        mbar_wait(&m.bar3, ph, p.err, kErrMmaWait);
        if (warp == 0) M3_TRACE(it, 17);
        tc_fence_after_sync();
        {  // 16x256b reads as in epilogue 1; each column pair leaves as one 8-byte store
          const int q4 = lane & 3, rr = lane >> 2;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float xa[8], xb[8];
            const uint32_t tl = tmem + lane_off + ((uint32_t)(16 * h) << 16) + 16u * grp;
            tmem_ld16x256_x2(tl + COL_DXA, xa);
            tmem_ld16x256_x2(tl + COL_DXB, xb);
            tmem_ld_wait();
            const uint32_t row = (uint32_t)(16 * sub + 8 * h + rr);
            const float d = rec.dec[row];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const uint32_t c0 = 16u * (uint32_t)grp + 8u * (uint32_t)k + 2u * (uint32_t)q4;
              st_shared_f2(stage_addr(sb + OFF_DGK + (c0 >> 5) * 8192u, row, (c0 & 31u) >> 2) +
                               4u * (c0 & 3u),
                           (xa[4 * k] + xa[4 * k + 2]) + d * (xb[4 * k] + xb[4 * k + 2]),
                           (xa[4 * k + 1] + xa[4 * k + 3]) + d * (xb[4 * k + 1] + xb[4 * k + 3]));
            }
          }
        }
        warp_arrive(&m.bar_dx, lane);
        if (warp == 0) M3_TRACE(it, 18);
        // ---- epilogue 4: dB = conj(dBa + dec_s dBb) cis(theta_s) -> staging tiles in sDYT, sDGM
        mbar_wait(&m.bar4, ph, p.err, kErrMmaWait);
        if (warp == 0) M3_TRACE(it, 19);
        tc_fence_after_sync();
        {
          float2 acc_a, acc_b;
          combine_rows2<kPlanar>(tmem + lane_off + COL_DBA + 32u * grp,
                                 tmem + lane_off + COL_DBB + 32u * grp, rec.dec, rec.cis, true,
                                 sb + OFF_DYT, sb + OFF_DGM, sub, grp,
                                 sb + OFF_B + ((uint32_t)grp >> 1) * 16384u, nullptr, lane, acc_a,
                                 acc_b, it, 36, make_float2(1.f, 0.f));
          if ((lane & 3) == 0) {  // conj: dB' conj(B')
            m.rb[ph][grp][16 * sub + (lane >> 2)] = make_float2(acc_a.x, -acc_a.y);
            m.rb[ph][grp][16 * sub + 8 + (lane >> 2)] = make_float2(acc_b.x, -acc_b.y);
          }
        }
        warp_arrive(&m.bar_db, lane);
        if (warp == 0) M3_TRACE(it, 20);
        ++it;
      }
      if (next >= p.total) break;

      // =================== ticket `next` starts ===================
      active = true;
      q = ticket_pos<kChains>(next, BH, p.H, p.G, p.seg);
      t0 = q.z * 64;
      const uint32_t ph = it & 1u;
      const ChunkRec& rec = m.rec[ph];
      if (warp == 0) M3_TRACE(it, 0);
      float xv[8], gv[8];  // this thread's 8 values of x and of dy (row xs0)
      {
        const int tx = t0 + xs0;
        const float* xr = p.x + q.b * p.xs[0] + (long long)tx * p.xs[1] + q.h * p.xs[2];
        const long long go = q.b * p.dys[0] + (long long)tx * p.dys[1] + q.h * p.dys[2];
        load8(xr, p.xs[3], p.x_vec, tx < p.T, xp0, xv);
        if (p.dy_bf16)
          load8_bf16(static_cast<const __nv_bfloat16*>(p.dy) + go, p.dys[3], p.dy_vec, tx < p.T,
                     xp0, gv);
        else
          load8(static_cast<const float*>(p.dy) + go, p.dys[3], p.dy_vec, tx < p.T, xp0, gv);
      }
      mbar_wait(&m.bar_tma, ph, p.err, kErrTmaWait);  // C tile, decay record
      if (warp == 0) M3_TRACE(it, 1);

      // ---- x, dy stacked over rows (K = p); e_l dy stacked over p (MN) once the previous
      // ticket's dx / dB stores have read sDGK / sDYT / sDGM
      {
        const uint32_t s = (uint32_t)xs0;
        split8_store(sb + OFF_X + swz(stack8(s, 0), tid & 7), sb + OFF_X + swz(stack8(s, 1), tid & 7),
                     xv);
        split8_store(sb + OFF_DY + swz(stack8(s, 0), tid & 7),
                     sb + OFF_DY + swz(stack8(s, 1), tid & 7), gv);
        if (warp == 0) M3_TRACE(it, 44);
        if (it > 0) mbar_wait(&m.bar_stfree, ph ^ 1u, p.err, kErrMmaWait);
        if (warp == 0) M3_TRACE(it, 45);
        const float e = rec.el[s];
        float w[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) w[u] = e * gv[u];
        const uint32_t mh = stack8((uint32_t)xp0, 0u), ml = stack8((uint32_t)xp0, 1u);
        split8_store(sb + OFF_DYT + (mh >> 6) * 8192u + swz(s, (mh & 63u) >> 3),
                     sb + OFF_DYT + (ml >> 6) * 8192u + swz(s, (ml & 63u) >> 3), w);
      }
      warp_arrive(&m.bar_opa, lane);  // dM may start
      if (warp == 0) M3_TRACE(it, 2);
      // ---- raw tiles -> split operands, in place: C' = C cis(theta_l) and
      // conj(B') = conj(B conj(cis(theta_s))) stacked (16 lanes per row), conj(H_z) hi | lo from
      // the forward's thread-major state tile (float4 i of forward thread f at [i][f]; f holds row
      // 16 (f/32 mod 4) + f mod 16, columns 64 (f/128) + 32 (f/16 mod 2) .. +31)
#pragma unroll 1
      for (int tile = 0; tile < 3; ++tile) {  // C (then Q may start), B (then G), H_z (then dCb)
        if (tile == 1) mbar_wait(&m.bar_tmb, ph, p.err, kErrTmaWait);
        if (tile == 2) mbar_wait(&m.bar_h, ph, p.err, kErrTmaWait);
        if (warp == 0) M3_TRACE(it, 3 + 2 * tile);
        const uint32_t base = tile == 0 ? OFF_C : (tile == 1 ? OFF_B : OFF_H);
        const bool stacked = tile != 2;
        const float sg = tile == 0 ? 1.f : -1.f;
        const int f = tid & 255;  // forward thread whose state values this thread converts
        float4 r4[2][2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int j = tid + kWorkers * i;
          const int k = 2 * (tid >> 8) + i;  // its float4 pair (2k, 2k+1) of the state tile
          if (kPlanar && stacked) {  // Re and Im of complex 4q .. 4q+3 of row l, 16 KB apart
            const float4* src = reinterpret_cast<const float4*>(smem + base) + (j >> 4) * 16 + (j & 15);
            const float4 re = src[0], im = src[1024];
            r4[i][0] = make_float4(re.x, im.x, re.y, im.y);
            r4[i][1] = make_float4(re.z, im.z, re.w, im.w);
          } else if (stacked) {
            // 32 bytes per thread: lanes 4-7 of each group of 8 read their second float4 first,
            // so each 8-lane phase of a 128-bit load covers all 32 banks once
            const float4* src = reinterpret_cast<const float4*>(smem + base) + (j >> 4) * 32 + 2 * (j & 15);
            const int sw = (j >> 2) & 1;
            const float4 a = src[sw], b = src[1 - sw];
            r4[i][0] = sw ? b : a;
            r4[i][1] = sw ? a : b;
          } else {
            const float4* src = reinterpret_cast<const float4*>(smem + base) + 2 * k * 256 + f;
            r4[i][0] = src[0];
            r4[i][1] = src[256];
          }
        }
        workers_sync();
        if (warp == 0) M3_TRACE(it, 46 + (tile == 1));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int j = tid + kWorkers * i;
          const uint32_t k = 2u * ((uint32_t)tid >> 8) + (uint32_t)i;
          const uint32_t l = stacked ? (uint32_t)j >> 4
                                     : 16u * (((uint32_t)f >> 5) & 3u) + ((uint32_t)f & 15u);
          const uint32_t qq = stacked ? (uint32_t)j & 15u
                                      : 8u * ((uint32_t)f >> 7) + 4u * (((uint32_t)f >> 4) & 1u) + k;
          const float2 cs = !stacked ? make_float2(1.f, 0.f)
                            : tile == 0 ? cmul2(rec.cis[l], p.crot) : rec.cis[l];
          const float rv[8] = {r4[i][0].x, r4[i][0].y, r4[i][0].z, r4[i][0].w,
                               r4[i][1].x, r4[i][1].y, r4[i][1].z, r4[i][1].w};
          float v[8];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            v[2 * u] = rv[2 * u] * cs.x - sg * (rv[2 * u + 1] * cs.y);
            v[2 * u + 1] = rv[2 * u] * cs.y + sg * (rv[2 * u + 1] * cs.x);
          }
          const uint32_t hi = stacked ? sb + base + (qq >> 3) * 16384u + swz(stack8(l, 0), qq & 7u)
                                      : sb + base + (qq >> 3) * 8192u + swz(l, qq & 7u);
          split8_store(hi, hi + (stacked ? 1024u : 16384u), v);
        }
        if (tile == 0) warp_arrive(&m.bar_opc, lane);   // Q may start
        if (tile == 1) warp_arrive(&m.bar_ops1, lane);  // G may start
        if (tile == 2) warp_arrive(&m.bar_oph, lane);   // dCb may start
        if (warp == 0) M3_TRACE(it, 4 + 2 * tile);
      }

      // ---- dS_z (fp32 in sDS, thread-major as the chunk z+1 ticket stored it: float4 i holds
      // row p = 16 sub + 8 (i/2) + lane/4, complex n = 16 grp + 4 k + lane%4 for k = 2 (i mod 2), +1)
      // -> dS'x hi | lo (K-major rows p: k-atom grp/2, 16-byte chunk 4 (grp mod 2) + k, 4 bytes
      // per complex)
      mbar_wait(&m.bar_ds, ph, p.err, kErrTmaWait);
      if (warp == 0) M3_TRACE(it, 9);
      float dsz[16];
      if (!q.last) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 v = ld_shared_f4(sb + OFF_DS + (uint32_t)(i * kWorkers + tid) * 16u);
          dsz[4 * i] = v.x;
          dsz[4 * i + 1] = v.y;
          dsz[4 * i + 2] = v.z;
          dsz[4 * i + 3] = v.w;
        }
      } else if (p.dhT != nullptr) {  // a chain's last chunk: dS = its end state's gradient, transposed
        const float2* src = p.dhT + (long long)q.sg * 64 * 64 + 16 * sub + (lane >> 2);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int n = 16 * grp + 4 * (2 * (i & 1) + u) + (lane & 3);
            const float2 v = __ldcg(src + n * 64 + 8 * (i >> 1));
            dsz[4 * i + 2 * u] = v.x;
            dsz[4 * i + 2 * u + 1] = v.y;
          }
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) dsz[c] = 0.f;
      }
      workers_sync();
      {
        const float2 ct = rec.ct;
        const uint32_t q4 = (uint32_t)lane & 3u, rr = (uint32_t)lane >> 2;
        const uint32_t db = sb + OFF_DS + ((uint32_t)grp >> 1) * 8192u + 4u * q4;
#pragma unroll
        for (int c = 0; c < 16; c += 2) {  // (Re, -Im) of conj(cis(theta_Gamma)) dS_z
          const uint32_t i = (uint32_t)c >> 2, k = 2u * (i & 1u) + (((uint32_t)c >> 1) & 1u);
          const uint32_t prow = 16u * (uint32_t)sub + 8u * (i >> 1) + rr;
          uint32_t whi, wlo;
          split2(dsz[c] * ct.x + dsz[c + 1] * ct.y, -(dsz[c + 1] * ct.x - dsz[c] * ct.y), whi, wlo);
          const uint32_t off = swz(prow, 4u * ((uint32_t)grp & 1u) + k);
          st_shared_u32(db + off, whi);
          st_shared_u32(db + 16384u + off, wlo);
        }
      }

      // ---- epilogue 1: Mr (over e dy, batch 1 done), dG' (two forms)
      if (warp == 0) M3_TRACE(it, 10);
      mbar_wait(&m.bar1, ph, p.err, kErrMmaWait);
      if (warp == 0) M3_TRACE(it, 11);
      tc_fence_after_sync();
      auto epilogue1 = [&]() {
        // 16x256b TMEM reads (hi / lo partial rows in one thread): rows 16 sub + 8 h + lane/4,
        // columns s = 16 grp + 8 k + 2 (lane%4), +1; each pair leaves as one 4-byte bf16x2 word
        // per split half and destination
        {
          const int q4 = lane & 3, rr = lane >> 2;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float g[8], dm[8];
            const uint32_t tl = tmem + lane_off + ((uint32_t)(16 * h) << 16) + 16u * grp;
            tmem_ld16x256_x2(tl + COL_G, g);
            tmem_ld16x256_x2(tl + COL_DM, dm);
            tmem_ld_wait();
            if (warp == 0) M3_TRACE(it, 40 + 2 * h);
            const int row = 16 * sub + 8 * h + rr;
            const float rl = rec.rho2[row];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              const int s0 = 16 * grp + 8 * k + 2 * q4;
              float mr2[2], dg2[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const float L = (s0 + e <= row) ? exp2f(rl - rec.rho2[s0 + e]) : 0.f;
                mr2[e] = L * (g[4 * k + e] + g[4 * k + 2 + e]);
                dg2[e] = L * (dm[4 * k + e] + dm[4 * k + 2 + e]);
              }
              uint32_t mrh, mrl, dgh, dgl;
              split2(mr2[0], mr2[1], mrh, mrl);
              split2(dg2[0], dg2[1], dgh, dgl);
              // MN-major (stacked s): k-atom s0/32, chunks 2 ((s0/8) mod 4) (hi) and +1 (lo)
              const uint32_t ch = 2u * (((uint32_t)s0 >> 3) & 3u), off = 4u * (uint32_t)q4;
              const uint32_t mnh = ((uint32_t)s0 >> 5) * 8192u + swz((uint32_t)row, ch) + off;
              const uint32_t mnl = ((uint32_t)s0 >> 5) * 8192u + swz((uint32_t)row, ch + 1u) + off;
              st_shared_u32(sb + OFF_DYT + mnh, mrh);
              st_shared_u32(sb + OFF_DYT + mnl, mrl);
              st_shared_u32(sb + OFF_DGM + mnh, dgh);
              st_shared_u32(sb + OFF_DGM + mnl, dgl);
              // K-major (stacked rows): chunk s0/8
              const uint32_t kc = (uint32_t)s0 >> 3;
              st_shared_u32(sb + OFF_DGK + swz(stack8((uint32_t)row, 0u), kc) + off, dgh);
              st_shared_u32(sb + OFF_DGK + swz(stack8((uint32_t)row, 1u), kc) + off, dgl);
            }
            if (warp == 0) M3_TRACE(it, 41 + 2 * h);
          }
        }
        warp_arrive(&m.bar_ops2, lane);
        if (warp == 0) M3_TRACE(it, 12);
      };
      auto carry = [&]() {
        // ---- carry: dS_{z-1} = Q + conj(e^Gamma) dS_z -> ring (thread-major, the layout above),
        // <dS_{z-1}, H_z>. Q in the 16x256b shape: rows p = 16 sub + 8 h + lane/4, complex
        // 16 grp + 4 k + lane%4 (k = 0..3), hi and lo partial rows added in registers.
        {
          const uint32_t q4 = (uint32_t)lane & 3u, rr = (uint32_t)lane >> 2;
          float qa[16], qb[16];
          tmem_ld16x256_x4(tmem + lane_off + COL_Q + 32u * grp, qa);
          tmem_ld16x256_x4(tmem + lane_off + (16u << 16) + COL_Q + 32u * grp, qb);
          tmem_ld_wait();
          float2 dg = make_float2(0.f, 0.f);
          if (!q.first) {
            const float2 g = rec.g;
            float4* slot = reinterpret_cast<float4*>(
                p.ring + ((long long)q.sg * kRingSlots + ((q.z - 1) % kRingSlots)) * 64 * 128);
            const uint32_t hb = sb + OFF_H + ((uint32_t)grp >> 1) * 8192u + 4u * q4;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float* qv = (i >> 1) ? qb : qa;
              const uint32_t prow = 16u * (uint32_t)sub + 8u * ((uint32_t)i >> 1) + rr;
              float o[4];
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int k = 2 * (i & 1) + u, c = 4 * i + 2 * u;
                const float qre = qv[4 * k] + qv[4 * k + 2], qim = qv[4 * k + 1] + qv[4 * k + 3];
                o[2 * u] = qre + g.x * dsz[c] + g.y * dsz[c + 1];
                o[2 * u + 1] = -qim + g.x * dsz[c + 1] - g.y * dsz[c];
                const uint32_t off = swz(prow, 4u * ((uint32_t)grp & 1u) + (uint32_t)k);
                const float2 h = unsplit2(ld_shared_u32(hb + off), ld_shared_u32(hb + 16384u + off));
                dg.x += o[2 * u] * h.x - o[2 * u + 1] * h.y;
                dg.y += o[2 * u] * h.y + o[2 * u + 1] * h.x;
              }
              __stcg(slot + i * kWorkers + tid, make_float4(o[0], o[1], o[2], o[3]));
            }
          } else if (p.dh0 != nullptr) {  // a chain's first chunk: dS_{z-1} is its entry state's gradient
            const float2 g = rec.g;
            float2* dst = p.dh0 + (long long)q.sg * 64 * 64 + 16 * sub + rr;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float* qv = (i >> 1) ? qb : qa;
#pragma unroll
              for (int u = 0; u < 2; ++u) {
                const int k = 2 * (i & 1) + u, c = 4 * i + 2 * u;
                const float qre = qv[4 * k] + qv[4 * k + 2], qim = qv[4 * k + 1] + qv[4 * k + 3];
                const int n = 16 * grp + 4 * k + (int)q4;
                __stcg(dst + n * 64 + 8 * (i >> 1),
                       make_float2(qre + g.x * dsz[c] + g.y * dsz[c + 1],
                                   -qim + g.x * dsz[c + 1] - g.y * dsz[c]));
              }
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) {
            dg.x += __shfl_xor_sync(0xffffffffu, dg.x, o);
            dg.y += __shfl_xor_sync(0xffffffffu, dg.y, o);
          }
          if (lane == 0) m.dgp[ph][warp] = dg;
        }
        // (back-pressure for the hand-off warp: it has finished the ticket before this one)
        if (warp == 0) M3_TRACE(it, 13);
        if (it > 0) mbar_wait(&m.bar_rel, (it - 1) & 1u, p.err, kErrMmaWait);
        warp_arrive(&m.bar_ops3, lane);
        if (warp == 0) M3_TRACE(it, 14);
      };
      if constexpr (kCarryFirst) {
        carry();
        epilogue1();
      } else {
        epilogue1();
        carry();
      }
      // the next ticket: its x and dy are prefetched at the top of the loop, during the epilogues
      mbar_wait(&m.bar_ctl, ph ^ 1u, p.err, kErrMmaWait);
      next = m.tick[(it + 1) & 1];
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

// dA[h] = sum over batch and chunks of the per-chunk partials: one CTA per head, fixed-order
// strided partial sums and a fixed tree, so the result is deterministic.
__global__ void __launch_bounds__(256) k_bwd_tc_dA(const float2* __restrict__ dapart, int Bsz,
                                                   int H, int nc, float2* __restrict__ dA,
                                                   int accum) {
  __shared__ float2 red[256];
  const int h = blockIdx.x;
  const int n = Bsz * nc;
  float2 acc = make_float2(0.f, 0.f);
  for (int i = threadIdx.x; i < n; i += 256) {
    const int b = i / nc, z = i - b * nc;
    const float2 v = dapart[((long long)b * H + h) * nc + z];
    acc.x += v.x;
    acc.y += v.y;
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) {
      red[threadIdx.x].x += red[threadIdx.x + o].x;
      red[threadIdx.x].y += red[threadIdx.x + o].y;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float2 prev = accum ? dA[h] : make_float2(0.f, 0.f);
    dA[h] = make_float2(prev.x + red[0].x, prev.y + red[0].y);
  }
}

// <dS_{nc-1}, conj(H_{nc})> of a sequence with a final-state gradient: the d Sigma term the last
// chunk's position 63 gets from its exit state (the other chunks take it from the chunk after
// them). One block per (b, h), (N, D) complex64 tiles of the final state and its gradient.
__global__ void __launch_bounds__(256) k_bwd_tc_dgam_last(const float2* __restrict__ hT,
                                                          const float2* __restrict__ dhT,
                                                          float2* __restrict__ out) {
  __shared__ float2 red[8];
  const long long base = (long long)blockIdx.x * 64 * 64;
  float2 acc = make_float2(0.f, 0.f);
  for (int i = threadIdx.x; i < 64 * 64; i += 256) {
    const float2 g = dhT[base + i], h = hT[base + i];
    acc.x += g.x * h.x + g.y * h.y;
    acc.y += g.y * h.x - g.x * h.y;
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
    out[blockIdx.x] = t;
  }
}

// ---------------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------------
namespace {

struct BwdLayout {
  size_t flags, ring, dgring, dapart, dglast, total;
};

// the ring, its <dS, H> slots and the end-state d Sigma terms are per chain (G per sequence)
BwdLayout bwd_layout(const Problem& p, int G) {
  const size_t bh = (size_t)p.Bsz * p.H, nc = (size_t)((p.T + 63) / 64), chains = bh * G;
  auto al = [](size_t v) { return (v + 255) & ~(size_t)255; };
  BwdLayout L;
  L.flags = 256;
  L.ring = al(L.flags + 4 * bh * nc);
  L.dgring = al(L.ring + chains * kRingSlots * 64 * 128 * sizeof(float));
  L.dapart = al(L.dgring + chains * kRingSlots * sizeof(float4));
  L.dglast = al(L.dapart + bh * nc * sizeof(float2));
  L.total = al(L.dglast + chains * sizeof(float2));
  return L;
}

}  // namespace

bool bwd_supported(const Problem& p) { return fwd_supported(p); }

size_t bwd_workspace_bytes(const Problem& p, int G) { return bwd_layout(p, G).total; }

BwdOut contiguous_bwd_out(const Problem& p, float* dx, float2* dA, float2* dB, float2* dC,
                          float* ddt) {
  (void)p;
  BwdOut o{};
  o.dx = dx;
  o.dA = dA;
  o.dB = reinterpret_cast<float*>(dB);
  o.dC = reinterpret_cast<float*>(dC);
  o.ddt = ddt;
  o.planar = 0;
  return o;
}

int run_bwd(const Problem& p, const void* dy, const long long dys[4], const void* states,
            const BwdOut& out, void* ws, cudaStream_t st, const void* hT, const void* dhT,
            void* dh0, int G, const void* dgam, bool clear_status, const void* recs_in,
            float2 crot, bool accum) {
  const BwdLayout L = bwd_layout(p, G);
  BwdParams bp{};
  bp.Bsz = p.Bsz;
  bp.T = p.T;
  bp.H = p.H;
  bp.nc = (p.T + 63) / 64;
  bp.total = p.Bsz * p.H * bp.nc;
  if (G < 1 || bp.nc % G != 0) return M3SSD_ERR_SHAPE;
  bp.G = G;
  bp.seg = bp.nc / G;
  bp.x = static_cast<const float*>(p.x);
  for (int i = 0; i < 4; ++i) bp.xs[i] = p.xs[i];
  bp.x_vec = (p.xs[3] == 1 && p.xs[0] % 4 == 0 && p.xs[1] % 4 == 0 && p.xs[2] % 4 == 0 &&
              reinterpret_cast<uintptr_t>(p.x) % 16 == 0)
                 ? 1
                 : 0;
  bp.dy = dy;
  bp.dy_bf16 = p.y_bf16;
  for (int i = 0; i < 4; ++i) bp.dys[i] = dys[i];
  // 8 values (32 or 16 bytes) per vector load
  const long long dv = p.y_bf16 ? 8 : 4;
  bp.dy_vec = (dys[3] == 1 && dys[0] % dv == 0 && dys[1] % dv == 0 && dys[2] % dv == 0 &&
               reinterpret_cast<uintptr_t>(dy) % 16 == 0)
                  ? 1
                  : 0;
  bp.A = p.A;
  bp.Bm = p.Bm;
  bp.Cm = p.Cm;
  for (int i = 0; i < 4; ++i) {
    bp.bs[i] = p.bs[i];
    bp.cs[i] = p.cs[i];
  }
  bp.states = static_cast<const float*>(states);
  bp.recs = recs_in != nullptr
                ? static_cast<const ChunkRec*>(recs_in)
                : reinterpret_cast<const ChunkRec*>(static_cast<const char*>(states) +
                                                    states_h_bytes(p));
  bp.crot = crot;
  bp.accum = accum ? 1 : 0;
  bp.ddt = out.ddt;
  // planar B / C in and planar dB / dC out go together (the in_proj entry points)
  if ((out.planar != 0) != (p.bc_planar != 0)) return M3SSD_ERR_SHAPE;
  bp.hp = out.planar ? p.H : 0;
  bp.ddt_sb = out.planar ? out.s_b : (long long)p.T * p.H;
  bp.ddt_st = out.planar ? out.s_t : (long long)p.H;
  char* base = static_cast<char*>(ws);
  bp.err = reinterpret_cast<uint32_t*>(base);
  bp.counter = reinterpret_cast<uint32_t*>(base) + 1;
  bp.flags = reinterpret_cast<uint32_t*>(base + L.flags);
  bp.ring = reinterpret_cast<float*>(base + L.ring);
  bp.dgring = reinterpret_cast<float4*>(base + L.dgring);
  bp.dapart = reinterpret_cast<float2*>(base + L.dapart);
  // state carry: with an end-state gradient the end state must come too (the chain's last chunk's
  // d Sigma term), unless that term is given ready-made; the entry-state gradient is written
  // whenever asked for
  if (dgam == nullptr && (dhT != nullptr) != (hT != nullptr)) return M3SSD_ERR_NULL;
  bp.dhT = static_cast<const float2*>(dhT);
  bp.dh0 = static_cast<float2*>(dh0);
  bp.dgam_last = dgam != nullptr  ? static_cast<const float2*>(dgam)
                 : dhT != nullptr ? reinterpret_cast<const float2*>(base + L.dglast)
                                  : nullptr;
  CUtensorMap tmB, tmC, tmDX, tmDB, tmDC;
  if (!encode_bc_tensor_map(&tmB, p.Bm, p, p.bs) || !encode_bc_tensor_map(&tmC, p.Cm, p, p.cs))
    return M3SSD_ERR_LAUNCH;
  if (out.planar) {
    // dx rows of D = 64 floats per head; dB, dC as (2H rows of N = 64 floats), Im rows after Re
    if (!encode_out_map_strided(&tmDX, out.dx, p, 64, p.H, 64, out.s_t, out.s_b) ||
        !encode_out_map_strided(&tmDB, out.dB, p, 64, 2 * p.H, 64, out.s_t, out.s_b) ||
        !encode_out_map_strided(&tmDC, out.dC, p, 64, 2 * p.H, 64, out.s_t, out.s_b))
      return M3SSD_ERR_LAUNCH;
  } else if (!encode_out_tensor_map(&tmDX, out.dx, p, 64) ||
             !encode_out_tensor_map(&tmDB, out.dB, p, 128) ||
             !encode_out_tensor_map(&tmDC, out.dC, p, 128)) {
    return M3SSD_ERR_LAUNCH;
  }
  const size_t keep = clear_status ? 0 : 4;  // an earlier pass of the same call reported here
  if (cudaMemsetAsync(base + keep, 0, L.ring - keep, st) != cudaSuccess) return M3SSD_ERR_LAUNCH;
  const int sms = sm_count();
  if (sms <= 0) return M3SSD_ERR_DEVICE;
  // few independent chains (sequences x chains per sequence): the chunk-to-chunk hand-offs, ~5.2 us
  // each, take longer than the tickets' throughput (~70 ns each), so the carry goes first
  const bool carry_first = (double)p.Bsz * p.H * G * 0.070 < 5.2;
  auto kern = carry_first
                  ? (out.planar ? (G > 1 ? k_bwd_tc<true, true, true> : k_bwd_tc<true, false, true>)
                                : (G > 1 ? k_bwd_tc<false, true, true> : k_bwd_tc<false, false, true>))
                  : (out.planar ? (G > 1 ? k_bwd_tc<true, true, false> : k_bwd_tc<true, false, false>)
                                : (G > 1 ? k_bwd_tc<false, true, false> : k_bwd_tc<false, false, false>));
  if (!ensure_smem_attr(reinterpret_cast<const void*>(kern), (int)kSmemBytes))
    return M3SSD_ERR_LAUNCH;
  const int grid = bp.total < sms ? bp.total : sms;
  if (dhT != nullptr && dgam == nullptr)
    k_bwd_tc_dgam_last<<<p.Bsz * p.H * G, 256, 0, st>>>(static_cast<const float2*>(hT),
                                                    bp.dhT, reinterpret_cast<float2*>(base + L.dglast));
  kern<<<grid, kThreads, kSmemBytes, st>>>(tmB, tmC, tmDX, tmDB, tmDC, bp);
  k_bwd_tc_dA<<<p.H, 256, 0, st>>>(bp.dapart, p.Bsz, p.H, bp.nc, out.dA, bp.accum);
  return cudaGetLastError() == cudaSuccess ? M3SSD_OK : M3SSD_ERR_LAUNCH;
}

}  // namespace tc
}  // namespace m3ssd

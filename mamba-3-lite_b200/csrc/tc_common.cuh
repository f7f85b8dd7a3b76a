// sm_100a building blocks for the tensor-core path: mbarriers, TMA, tcgen05 (TMEM allocation,
// MMA, commit, loads), shared-memory matrix descriptors and the split-bf16 operand format.
//
// Split-bf16 operands: every fp32 operand value v is stored as hi = bf16(v) and
// lo = bf16(v - hi), so hi + lo carries ~16 significant bits. A product A.B is formed from all
// four partial products (A_hi + A_lo)(B_hi + B_lo) with fp32 accumulation; for a GEMM whose
// natural M is 64 the hi and lo rows of A are stacked into one M = 128 operand (rows interleaved
// in groups of 16, see stack_row) so two tcgen05.mma passes (B_hi, B_lo) produce all four
// products, and the epilogue adds the hi-row and lo-row partial sums with one warp shuffle.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace m3ssd {
namespace tc {

// bounded waits: iterations before a wait gives up and records an error bit
// flag polls (each an L2 round trip plus a short sleep, well under 1 us) before a hand-off wait
// gives up: about a second, against tens of microseconds for the longest legitimate wait
constexpr uint32_t kSpinLimit = 1u << 21;
// mbarrier waits give up after this many sleeping attempts: ~1 s (an attempt that does not see
// the phase complete returns after several microseconds; one that does returns at once)
constexpr uint32_t kSpinLimitSleep = 1u << 17;

enum ErrorBits : uint32_t {
  kErrTmaWait = 1u << 0,  // M3SSD_DEVERR_* in include/m3ssd.h
  kErrMmaWait = 1u << 1,
  kErrFlagWait = 1u << 2,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase completes or
// about `ns` nanoseconds pass, instead of re-polling the barrier in shared memory
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
// The polling loop is out of line: inlined at every wait site, the compiler's peeling of its first
// iterations made the persistent kernels several times larger than the instruction cache. Each
// iteration sleeps in hardware rather than polling, which keeps 17 waiting warps from
// competing with the tensor core for shared-memory bandwidth.
static __device__ __noinline__ bool mbar_spin(uint64_t* bar, uint32_t parity, uint32_t* err,
                                              uint32_t code) {
  for (uint32_t i = 0; i < kSpinLimitSleep; ++i)
    if (mbar_try_wait_sleep(bar, parity, 1000u)) return true;
  atomicOr(err, code);
  return false;
}
// Waits for the phase with the given parity to complete. Gives up after kSpinLimitSleep attempts,
// records `code` in *err and returns false (the kernel then finishes with garbage results
// instead of hanging the GPU).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err,
                                          uint32_t code) {
  return mbar_try_wait(bar, parity) || mbar_spin(bar, parity, err, code);
}

// ----------------------------------------------------------------------------- proxies, fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ----------------------------------------------------------------------------- TMA
// 4-D tiled bulk tensor load global -> shared, completion counted on `bar` (no multicast).
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// tiled TMA store from shared memory (bulk-group completion); out-of-range elements are skipped
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// the same as a reduction: the tile is added (f32 add) to what global memory holds
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int c0,
                                                  int c1, int c2, int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group"
      " [%0, {%2, %3, %4, %5}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
// store (accumulate = false) or add (true) a tile
__device__ __forceinline__ void tma_put_4d(const CUtensorMap* map, const void* src, int c0, int c1,
                                           int c2, int c3, bool accumulate) {
  if (accumulate)
    tma_reduce_add_4d(map, src, c0, c1, c2, c3);
  else
    tma_store_4d(map, src, c0, c1, c2, c3);
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// the shared-memory sources of all committed bulk groups have been read
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// all committed bulk groups have completed (their global writes are done)
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ----------------------------------------------------------------------------- TMEM
// warp-wide; writes the allocated base address to *dst
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D(tmem) (+)= A(smem desc) x B(smem desc), kind::f16 (bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// mbarrier arrives once all previously issued tcgen05.mma of this thread have completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (base + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 16 consecutive 32-bit columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 16 TMEM lanes x 32 columns (shape 16x256b, 4 repeats): thread t receives, for k = 0..3,
// v[4k], v[4k+1] = (lane t/4, columns 8k + 2 (t%4), +1) and v[4k+2], v[4k+3] = the same columns of
// lane t/4 + 8 (lanes relative to the 16-lane base in taddr)
__device__ __forceinline__ void tmem_ld16x256_x4(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// the same over 16 columns (2 repeats): v[4k .. 4k+3] for k = 0, 1
__device__ __forceinline__ void tmem_ld16x256_x2(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, SWIZZLE_128B (Blackwell descriptor version 1).
// K-major: rows of 128 B, 8-row groups `sbo` bytes apart; MN-major: 64-element (128 B) groups
// `lbo` bytes apart, K-rows of 128 B, 8-K-row groups `sbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: kind::f16 with bf16 A/B, fp32 D, dense.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn_major, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn_major << 15) |
         ((uint32_t)b_mn_major << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ----------------------------------------------------------------------------- operand format
// 128-B-swizzled byte offset of 16-byte chunk `chunk` (0..7) in row `row` of a SW128 region
__device__ __forceinline__ uint32_t swz(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}
// stacked M = 128 row holding part (0 = hi, 1 = lo) of logical row r (0..63)
__device__ __forceinline__ uint32_t stack_row(uint32_t r, uint32_t part) {
  return ((r >> 4) << 5) | (part << 4) | (r & 15u);
}
// splits 8 floats into 8 hi and 8 lo bf16 packed in two uint4 (pairwise bf16x2 conversions)
__device__ __forceinline__ void split8(const float (&v)[8], uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 hp = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    const float2 hf = __bfloat1622float2(hp);
    const __nv_bfloat162 lp = __floats2bfloat162_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
    h[i] = *reinterpret_cast<const uint32_t*>(&hp);
    l[i] = *reinterpret_cast<const uint32_t*>(&lp);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}
__device__ __forceinline__ void st_shared_v4(uint32_t saddr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(saddr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// ----------------------------------------------------------------------------- global memory
__device__ __forceinline__ float4 ldg_nc_v4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// A probe that does not order anything by itself: pair a nonzero result with fence_acquire_gpu()
// before reading what the flag publishes (relaxed load + fence = acquire). Unlike an acquire
// load, the thread need not wait for the value until it uses it.
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acquire_gpu() {
  asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
// Waits until the hand-off flag at f is nonzero (acquire, gpu scope). Gives up after kSpinLimit
// polls and records kErrFlagWait in *err instead of hanging; returns whether the flag was seen.
__device__ __forceinline__ bool flag_wait(const uint32_t* f, uint32_t* err) {
#pragma unroll 1
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ld_acquire_gpu(f) != 0u) return true;
    __nanosleep(64);
  }
  atomicOr(err, kErrFlagWait);
  return false;
}
// flag_wait with relaxed polls: the caller follows it with fence_acquire_gpu()
__device__ __forceinline__ bool flag_wait_relaxed(const uint32_t* f, uint32_t* err) {
#pragma unroll 1
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (ld_relaxed_gpu(f) != 0u) return true;
    __nanosleep(64);
  }
  atomicOr(err, kErrFlagWait);
  return false;
}
__device__ __forceinline__ void st_release_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

}  // namespace tc
}  // namespace m3ssd

namespace m3ssd {
namespace tc {
// Stacked M = 128 row for part (0 = hi, 1 = lo) of logical row r (0..63), interleaved in groups
// of 8: rows 16g..16g+7 hold hi of r = 8g..8g+7 and rows 16g+8..16g+15 the lo. The hi (or lo)
// rows alone then form a regular 8-row-group layout with a 2048-byte group stride, so the same
// buffer is also a plain 64-row operand (B role, or K rows of an MN-major operand), and the hi
// and lo partial sums of one output row sit in TMEM lanes m and m ^ 8 of the same warp.
__device__ __forceinline__ uint32_t stack8(uint32_t r, uint32_t part) {
  return ((r >> 3) << 4) | (part << 3) | (r & 7u);
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t saddr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(saddr));
  return v;
}
__device__ __forceinline__ void st_shared_f2(uint32_t saddr, float x, float y) {
  asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(saddr), "f"(x), "f"(y) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t saddr, uint32_t x) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(saddr), "r"(x) : "memory");
}
// splits 2 floats into a bf16x2 hi word and a bf16x2 lo word (one pair of split8)
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 hp = __floats2bfloat162_rn(v0, v1);
  const float2 hf = __bfloat1622float2(hp);
  const __nv_bfloat162 lp = __floats2bfloat162_rn(v0 - hf.x, v1 - hf.y);
  hi = *reinterpret_cast<const uint32_t*>(&hp);
  lo = *reinterpret_cast<const uint32_t*>(&lp);
}
__device__ __forceinline__ void st_shared_f32(uint32_t saddr, float x) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(saddr), "f"(x) : "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(uint32_t saddr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(saddr));
  return v;
}
__device__ __forceinline__ uint4 ld_shared_u4(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(saddr));
  return v;
}
// hi + lo of a packed bf16 pair -> two floats
__device__ __forceinline__ float2 unsplit2(uint32_t hi, uint32_t lo) {
  const float h0 = __uint_as_float(hi << 16), h1 = __uint_as_float(hi & 0xFFFF0000u);
  const float l0 = __uint_as_float(lo << 16), l1 = __uint_as_float(lo & 0xFFFF0000u);
  return make_float2(h0 + l0, h1 + l1);
}
}  // namespace tc
}  // namespace m3ssd

namespace m3ssd {
namespace tc {
// Non-tensor bulk copy global -> shared (16-byte aligned, size a multiple of 16), counted on bar.
// pull the 128-byte line holding `ptr` into L2 (no register, nothing to wait for)
__device__ __forceinline__ void prefetch_l2_line(const void* ptr) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(ptr)));
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Per (sequence, chunk) decay quantities written by k_chunk_prep and bulk-copied by the forward
// and backward kernels. Position l of chunk z is t = 64 z + l; Sigma_l = rho_l + i theta_l is the
// within-chunk inclusive cumsum of a = softplus(dt) A (a = 0 for t >= T), Gamma = Sigma_63.
struct ChunkRec {
  float rho2[64];  // Re Sigma_l in log2 units (rho_l log2(e)): exp(rho_l - rho_s) = exp2(rho2_l - rho2_s)
  float el[64];    // exp(rho_l)
  float dec[64];   // exp(rho_Gamma - rho_l)
  float sp[64];    // softplus(dt_t) (0 past T)
  float dsp[64];   // softplus'(dt_t) (0 past T)
  float2 cis[64];  // (cos, sin)(theta_l)
  float2 g;        // e^Gamma
  float2 ct;       // cis(theta_Gamma)
  float2 pad[2];
};
static_assert(sizeof(ChunkRec) % 16 == 0, "bulk copy granularity");
}  // namespace tc
}  // namespace m3ssd

namespace m3ssd {
namespace tc {
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// orders this thread's generic-proxy view of global memory with its async-proxy (bulk copy)
// accesses: after acquiring data another CTA wrote with plain stores, before bulk-copying it
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// barrier among the first `count` threads of the CTA (ids 1..15; 0 is __syncthreads)
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
}  // namespace tc
}  // namespace m3ssd

// C ABI of the m3ssd operator (declared in include/m3ssd.h): argument validation, path
// selection and launch. No allocation, no synchronisation, no host-side compute fallback.
#include <cuda_runtime.h>
#include <limits.h>
#include <stdint.h>

#include <mutex>

#include "m3ssd.h"
#include "m3ssd_common.cuh"
#include "simt_path.h"
#include "tc_path.h"

using m3ssd::Problem;

namespace {

bool mul_ok(int64_t a, int64_t b, int64_t* out) {
  if (a < 0 || b < 0) return false;
  if (a != 0 && b > INT64_MAX / a) return false;
  *out = a * b;
  return true;
}

int check_problem(const m3ssd_problem* pr) {
  if (!pr) return M3SSD_ERR_NULL;
  if (pr->reserved != 0) return M3SSD_ERR_FLAGS;
  const uint32_t known = M3SSD_X_COMPLEX | M3SSD_PREC_MASK | M3SSD_Y_BF16;
  if (pr->flags & ~known) return M3SSD_ERR_FLAGS;
  if ((pr->flags & M3SSD_PREC_MASK) == M3SSD_PREC_MASK) return M3SSD_ERR_FLAGS;
  if (pr->batch <= 0 || pr->seqlen <= 0 || pr->nheads <= 0 || pr->headdim <= 0 || pr->dstate <= 0)
    return M3SSD_ERR_SHAPE;
  if (pr->chunk < 1 || pr->chunk > 256) return M3SSD_ERR_CHUNK;
  if (pr->headdim > 256 || pr->dstate > 256) return M3SSD_ERR_DIM_LIMIT;
  const int64_t nc = (pr->seqlen + pr->chunk - 1) / pr->chunk;
  int64_t bh, t1, t2;
  if (!mul_ok(pr->batch, pr->nheads, &bh)) return M3SSD_ERR_OVERFLOW;
  // grid limits of the chunk-parallel kernels (gridDim.y = chunks, gridDim.z = batch*heads)
  if (nc > 65535 || bh > 65535) return M3SSD_ERR_SHAPE;
  if (pr->seqlen > INT_MAX / 2) return M3SSD_ERR_SHAPE;
  // largest buffers: states (bh*nc*N*D complex) and the per-chunk C*C workspace
  if (!mul_ok(bh, nc, &t1) || !mul_ok(t1, pr->dstate * pr->headdim, &t2) || !mul_ok(t2, 8, &t2))
    return M3SSD_ERR_OVERFLOW;
  if (!mul_ok(t1, pr->chunk * pr->chunk, &t2) || !mul_ok(t2, 16, &t2)) return M3SSD_ERR_OVERFLOW;
  // a bf16 y is written (and its gradient read) only by the tensor-core kernels
  if ((pr->flags & M3SSD_Y_BF16) &&
      !(pr->headdim == 64 && pr->dstate == 64 && !(pr->flags & M3SSD_X_COMPLEX) &&
        (pr->flags & M3SSD_PREC_MASK) != M3SSD_PREC_FP32))
    return M3SSD_ERR_SHAPE;
  return M3SSD_OK;
}

// Problems the tensor-core path can take (by shape and precision) are blocked at 64 positions
// whichever path runs, so `states` written by either forward path is read correctly by either
// backward path. The result does not depend on the blocking. Complex x runs as two real-x passes
// (tc_complex.cu).
bool tc_shape(const m3ssd_problem* pr) {
  const uint32_t prec = pr->flags & M3SSD_PREC_MASK;
  return pr->headdim == 64 && pr->dstate == 64 && prec != M3SSD_PREC_FP32;
}

// whether the tensor-core kernels take this problem's operands (B / C through TMA); complex x is
// checked on the real-x view of its passes
bool tc_supported(const Problem& p) {
  return m3ssd::tc::fwd_supported(p.x_complex ? m3ssd::tc::real_part_view(p, 0) : p);
}

Problem make_problem(const m3ssd_problem* pr) {
  Problem p{};
  p.Bsz = (int)pr->batch;
  p.T = (int)pr->seqlen;
  p.H = (int)pr->nheads;
  p.D = (int)pr->headdim;
  p.N = (int)pr->dstate;
  p.C = (int)pr->chunk;
  p.nc = (int)((pr->seqlen + pr->chunk - 1) / pr->chunk);
  p.x_complex = (pr->flags & M3SSD_X_COMPLEX) ? 1 : 0;
  p.y_bf16 = (pr->flags & M3SSD_Y_BF16) ? 1 : 0;
  if (tc_shape(pr)) {
    p.C = m3ssd::tc::kChunk;
    p.nc = (int)((pr->seqlen + p.C - 1) / p.C);
  }
  return p;
}


// Scratch of a forward / backward call: the larger of the two paths' needs; the tensor-core path
// adds the chained-pass buffers when the shape runs as several chains per sequence.
size_t bwd_ws(const m3ssd_problem* pr, const Problem& p) {
  size_t a = m3ssd::simt::bwd_workspace_bytes(p), b = m3ssd::tc::bwd_workspace_bytes(p);
  if (tc_shape(pr) && p.x_complex) {
    b = m3ssd::tc::complex_bwd_workspace_bytes(p);
  } else if (tc_shape(pr)) {
    const int G = m3ssd::tc::chains_for(p, true);
    if (G > 1) b = m3ssd::tc::bwd_chains_workspace_bytes(p, G);
  }
  return a > b ? a : b;
}

size_t fwd_ws(const m3ssd_problem* pr, const Problem& p) {
  size_t a = m3ssd::simt::fwd_workspace_bytes(p), b = m3ssd::tc::fwd_workspace_bytes(p);
  if (tc_shape(pr)) {
    const int G = m3ssd::tc::chains_for(p, false);
    if (G > 1) b = m3ssd::tc::fwd_chains_workspace_bytes(p, G);
  }
  return a > b ? a : b;
}

// The tensor-core forward / backward, in one pass or as chains (m3ssd::tc::chains_for)
int tc_fwd(const Problem& p, void* y, void* states, void* ws, void* stream, const void* h0,
           void* hT) {
  const auto st = static_cast<cudaStream_t>(stream);
  const int G = m3ssd::tc::chains_for(p, false);
  if (G > 1) return m3ssd::tc::run_fwd_chains(p, y, states, ws, st, h0, hT, G);
  return m3ssd::tc::run_fwd(p, y, states, ws, st, h0, hT);
}

int tc_bwd(const Problem& p, const void* dy, const long long dys[4], const void* states,
           const m3ssd::tc::BwdOut& out, void* ws, void* stream, const void* hT, const void* dhT,
           void* dh0) {
  const auto st = static_cast<cudaStream_t>(stream);
  const int G = m3ssd::tc::chains_for(p, true);
  if (G > 1) return m3ssd::tc::run_bwd_chains(p, dy, dys, states, out, ws, st, hT, dhT, dh0, G);
  return m3ssd::tc::run_bwd(p, dy, dys, states, out, ws, st, hT, dhT, dh0);
}

bool aligned(const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

int check_device() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return M3SSD_ERR_DEVICE;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return M3SSD_ERR_DEVICE;
  if (major != 10) return M3SSD_ERR_DEVICE;
  return M3SSD_OK;
}

int fill_inputs(Problem& p, const void* x, const int64_t xs[4], const void* A, const void* B,
                const int64_t bs[4], const void* C, const int64_t cs[4], const float* dt,
                const int64_t dts[3]) {
  if (!x || !A || !B || !C || !dt) return M3SSD_ERR_NULL;
  const size_t xa = p.x_complex ? 8 : 4;
  if (!aligned(x, xa) || !aligned(A, 8) || !aligned(B, 8) || !aligned(C, 8) || !aligned(dt, 4))
    return M3SSD_ERR_ALIGN;
  p.x = x;
  p.A = static_cast<const float2*>(A);
  p.Bm = static_cast<const float2*>(B);
  p.Cm = static_cast<const float2*>(C);
  p.dt = dt;
  for (int i = 0; i < 4; ++i) {
    p.xs[i] = xs[i];
    p.bs[i] = bs[i];
    p.cs[i] = cs[i];
  }
  for (int i = 0; i < 3; ++i) p.dts[i] = dts[i];
  return M3SSD_OK;
}

// ---------------------------------------------------------------------------------------------
// Fixed device scratch for m3ssd_fwd_static_scratch. Some callers cannot allocate device memory
// when they call the operator: a serving runtime that plans every byte of device memory before
// it takes requests and forbids allocation on the request path, or code running inside another
// framework's step where no allocator is reachable. The tensor-core forward needs only a small
// scratch area (status word, ticket counter and one hand-off flag per chunk of each sequence), so
// that area lives in this file-scope device array instead. Every GPU that loads the library holds
// the array until the process exits.
constexpr int64_t kStaticMaxChunks = 32768;  // batch * heads * ceil(seqlen / 64) limit
constexpr size_t kStaticScratchBytes = 256 + 4 * (size_t)kStaticMaxChunks;  // 131,328 bytes
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_static_mu;
// per device: the array's device address and the context it was looked up in
void* g_static_scratch_addr[kMaxDevices] = {};
void* g_static_scratch_ctx[kMaxDevices] = {};

// The current context of the calling thread, through the driver entry point the runtime exposes
// (the library does not link libcuda). nullptr if it cannot be queried.
void* current_context() {
  using GetCtx = int (*)(void**);
  static GetCtx fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<GetCtx>(ptr);
    return static_cast<GetCtx>(nullptr);
  }();
  void* ctx = nullptr;
  if (fn == nullptr || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of g_static_scratch on the current device, looked up with that device current
// (the name is only a host-side stand-in for the device array). The lookup is cached per device
// and redone when the device's context has changed (cudaDeviceReset reloads the module, which
// can move the array).
int static_scratch_address(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return M3SSD_ERR_DEVICE;
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_scratch_addr[dev] || ctx == nullptr || ctx != g_static_scratch_ctx[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_static_scratch) != cudaSuccess || ptr == nullptr)
      return M3SSD_ERR_DEVICE;
    g_static_scratch_addr[dev] = ptr;
    // the lookup has made the device's primary context current if none was
    g_static_scratch_ctx[dev] = current_context();
  }
  *out = g_static_scratch_addr[dev];
  return M3SSD_OK;
}

// Column offsets (floats) of the in_proj output of one token, in the order the block slices it
// (models/mamba_block.py:74-84): x, Re B, Im B, Re C, Im C, dt
struct ProjCols {
  int64_t x, b_re, b_im, c_re, c_im, dt, width;
};
ProjCols proj_cols(const m3ssd_problem& pr) {
  const int64_t H = pr.nheads, D = pr.headdim, N = pr.dstate;
  ProjCols c;
  c.x = 0;
  c.b_re = H * D;
  c.b_im = c.b_re + H * N;
  c.c_re = c.b_im + H * N;
  c.c_im = c.c_re + H * N;
  c.dt = c.c_im + H * N;
  c.width = c.dt + H;
  return c;
}

// Problem view of the in_proj form: x, B, C, dt are column blocks of `proj`, B and C planar.
// Tensor-core shapes only; TMA reads the B and C blocks, so the projection must be 16-byte aligned
// with batch / time strides (and the column offsets) multiples of 4 floats.
int proj_problem(const m3ssd_problem* pr, const float* proj, const int64_t ps[2], const void* A,
                 Problem* out) {
  int rc = check_problem(pr);
  if (rc) return rc;
  if (!tc_shape(pr) || (pr->flags & M3SSD_X_COMPLEX)) return M3SSD_ERR_SHAPE;
  if (!proj || !A) return M3SSD_ERR_NULL;
  if (ps[0] <= 0 || ps[1] <= 0) return M3SSD_ERR_SHAPE;
  const ProjCols c = proj_cols(*pr);
  if (!aligned(proj, 16) || !aligned(A, 8) || ps[0] % 4 || ps[1] % 4 || c.b_re % 4)
    return M3SSD_ERR_ALIGN;
  Problem p = make_problem(pr);
  p.x = proj + c.x;
  p.xs[0] = ps[0];
  p.xs[1] = ps[1];
  p.xs[2] = pr->headdim;
  p.xs[3] = 1;
  p.A = static_cast<const float2*>(A);
  p.bc_planar = 1;
  p.Bm = reinterpret_cast<const float2*>(proj + c.b_re);
  p.Cm = reinterpret_cast<const float2*>(proj + c.c_re);
  p.bs[0] = p.cs[0] = ps[0];
  p.bs[1] = p.cs[1] = ps[1];
  p.bs[2] = p.cs[2] = pr->dstate;
  p.bs[3] = p.cs[3] = 1;
  p.dt = proj + c.dt;
  p.dts[0] = ps[0];
  p.dts[1] = ps[1];
  p.dts[2] = 1;
  if (!m3ssd::tc::fwd_supported(p)) return M3SSD_ERR_ALIGN;
  *out = p;
  return M3SSD_OK;
}

}  // namespace

extern "C" {

int m3ssd_abi_version(void) { return M3SSD_ABI_VERSION; }

const char* m3ssd_strerror(int status) {
  switch (status) {
    case M3SSD_OK: return "success";
    case M3SSD_ERR_NULL: return "m3ssd: a required pointer is NULL";
    case M3SSD_ERR_SHAPE: return "m3ssd: invalid or unsupported shape";
    case M3SSD_ERR_CHUNK: return "m3ssd: chunk_size must be in [1, 256]";
    case M3SSD_ERR_DIM_LIMIT: return "m3ssd: head_dim and state_dim must not exceed 256";
    case M3SSD_ERR_ALIGN: return "m3ssd: pointer not aligned to its element type";
    case M3SSD_ERR_WORKSPACE: return "m3ssd: workspace missing or too small";
    case M3SSD_ERR_LAUNCH: return "m3ssd: CUDA kernel launch failed";
    case M3SSD_ERR_DEVICE: return "m3ssd: current CUDA device is not an sm_100 GPU";
    case M3SSD_ERR_FLAGS: return "m3ssd: unknown flag bits";
    case M3SSD_ERR_OVERFLOW: return "m3ssd: problem size overflows 64-bit indexing";
    case M3SSD_ERR_SCRATCH_LIMIT:
      return "m3ssd: problem exceeds the fixed scratch of m3ssd_fwd_static_scratch "
             "(batch * heads * ceil(seqlen / 64) must be <= 32768)";
    default: return "m3ssd: unknown status";
  }
}

int m3ssd_check_problem(const m3ssd_problem* prob) { return check_problem(prob); }

size_t m3ssd_states_bytes(const m3ssd_problem* prob) {
  if (check_problem(prob) != M3SSD_OK) return 0;
  const Problem p = make_problem(prob);
  const size_t a = m3ssd::simt::states_bytes(p);
  const size_t b = !tc_shape(prob) ? 0
                   : p.x_complex   ? m3ssd::tc::complex_states_bytes(p)
                                   : m3ssd::tc::states_bytes(p);
  return a > b ? a : b;
}

size_t m3ssd_fwd_workspace_bytes(const m3ssd_problem* prob) {
  if (check_problem(prob) != M3SSD_OK) return 0;
  return fwd_ws(prob, make_problem(prob));
}

size_t m3ssd_bwd_workspace_bytes(const m3ssd_problem* prob) {
  if (check_problem(prob) != M3SSD_OK) return 0;
  return bwd_ws(prob, make_problem(prob));
}

const char* m3ssd_fwd_path(const m3ssd_problem* prob) {
  if (check_problem(prob) != M3SSD_OK) return "invalid";
  return tc_shape(prob) ? "tcgen05-bf16x2" : "simt-fp32";
}

const char* m3ssd_bwd_path(const m3ssd_problem* prob) {
  if (check_problem(prob) != M3SSD_OK) return "invalid";
  return tc_shape(prob) ? "tcgen05-bf16x2" : "simt-fp32";
}

int m3ssd_launch_count(const m3ssd_problem* prob, int backward) {
  if (check_problem(prob) != M3SSD_OK) return 0;
  if (!tc_shape(prob)) return backward ? m3ssd::simt::kBwdLaunches : m3ssd::simt::kFwdLaunches;
  // complex x: two passes of the real-x kernels (the forward's records once), and the backward's
  // dx interleave
  if (prob->flags & M3SSD_X_COMPLEX)
    return backward ? 2 * m3ssd::tc::kBwdLaunches + 1 : 2 * m3ssd::tc::kFwdLaunches - 1;
  // the chained forms: forward two passes (the records once) plus the segment chain; backward the
  // carry pass, the segment chain, the segments' end-state terms and the tensor-core pass
  const bool chained = m3ssd::tc::chains_for(make_problem(prob), backward != 0) > 1;
  if (backward) return chained ? m3ssd::tc::kBwdLaunches + 3 : m3ssd::tc::kBwdLaunches;
  return chained ? 2 * m3ssd::tc::kFwdLaunches : m3ssd::tc::kFwdLaunches;
}

int m3ssd_fwd(const m3ssd_fwd_args* a, void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  Problem p = make_problem(&a->prob);
  rc = fill_inputs(p, a->x, a->x_strides, a->A, a->B, a->b_strides, a->C, a->c_strides, a->dt,
                   a->dt_strides);
  if (rc) return rc;
  if (!a->y || !a->states) return M3SSD_ERR_NULL;
  if (!aligned(a->y, 4) || !aligned(a->states, 16)) return M3SSD_ERR_ALIGN;
  const size_t need = fwd_ws(&a->prob, p);
  if (!a->workspace || a->workspace_bytes < need) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 256)) return M3SSD_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  if (tc_shape(&a->prob) && tc_supported(p)) {
    // y leaves the tensor-core forward through TMA stores
    if (!aligned(a->y, 16)) return M3SSD_ERR_ALIGN;
    if (p.x_complex)
      return m3ssd::tc::run_fwd_complex(p, a->y, a->states, a->workspace,
                                        static_cast<cudaStream_t>(stream));
    return tc_fwd(p, a->y, a->states, a->workspace, stream, nullptr, nullptr);
  }
  if (p.y_bf16) return M3SSD_ERR_SHAPE;  // B / C strides the tensor-core path cannot take
  return m3ssd::simt::run_fwd(p, static_cast<float*>(a->y), a->states, a->workspace,
                              static_cast<cudaStream_t>(stream));
}

int m3ssd_bwd(const m3ssd_bwd_args* a, void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  Problem p = make_problem(&a->prob);
  rc = fill_inputs(p, a->x, a->x_strides, a->A, a->B, a->b_strides, a->C, a->c_strides, a->dt,
                   a->dt_strides);
  if (rc) return rc;
  if (!a->dy || !a->states || !a->dx || !a->dA || !a->dB || !a->dC || !a->ddt)
    return M3SSD_ERR_NULL;
  const size_t xa = p.x_complex ? 8 : 4;
  if (!aligned(a->dy, p.y_bf16 ? 2 : 4) || !aligned(a->states, 16) || !aligned(a->dx, xa) ||
      !aligned(a->dA, 8) ||
      !aligned(a->dB, 8) || !aligned(a->dC, 8) || !aligned(a->ddt, 4))
    return M3SSD_ERR_ALIGN;
  const size_t need = bwd_ws(&a->prob, p);
  if (!a->workspace || a->workspace_bytes < need) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 256)) return M3SSD_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  long long dys[4];
  for (int i = 0; i < 4; ++i) dys[i] = a->dy_strides[i];
  // the tensor-core backward reads the forward's private state layout and writes dx, dB, dC
  // with TMA stores: 16-byte aligned outputs
  if (tc_shape(&a->prob) && tc_supported(p)) {
    if (!aligned(a->dx, 16) || !aligned(a->dB, 16) || !aligned(a->dC, 16))
      return M3SSD_ERR_ALIGN;
    if (p.x_complex)
      return m3ssd::tc::run_bwd_complex(
          p, a->dy, dys, a->states, static_cast<float2*>(a->dx), static_cast<float2*>(a->dA),
          static_cast<float2*>(a->dB), static_cast<float2*>(a->dC), a->ddt, a->workspace,
          static_cast<cudaStream_t>(stream));
    const m3ssd::tc::BwdOut out = m3ssd::tc::contiguous_bwd_out(
        p, static_cast<float*>(a->dx), static_cast<float2*>(a->dA), static_cast<float2*>(a->dB),
        static_cast<float2*>(a->dC), a->ddt);
    return tc_bwd(p, a->dy, dys, a->states, out, a->workspace, stream, nullptr, nullptr, nullptr);
  }
  if (p.y_bf16) return M3SSD_ERR_SHAPE;
  return m3ssd::simt::run_bwd(p, static_cast<const float*>(a->dy), dys, a->states, a->dx,
                              static_cast<float2*>(a->dA),
                              static_cast<float2*>(a->dB), static_cast<float2*>(a->dC), a->ddt,
                              a->workspace, static_cast<cudaStream_t>(stream));
}

int m3ssd_fwd_static_scratch(const m3ssd_fwd_args* a, void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  if (!tc_shape(&a->prob)) return M3SSD_ERR_SHAPE;  // tensor-core forward shapes only
  Problem p = make_problem(&a->prob);
  rc = fill_inputs(p, a->x, a->x_strides, a->A, a->B, a->b_strides, a->C, a->c_strides, a->dt,
                   a->dt_strides);
  if (rc) return rc;
  if (!a->y || !a->states) return M3SSD_ERR_NULL;
  if (!aligned(a->y, 16) || !aligned(a->states, 16)) return M3SSD_ERR_ALIGN;
  if (!m3ssd::tc::fwd_supported(p)) return M3SSD_ERR_SHAPE;
  const int64_t chunks = a->prob.batch * a->prob.nheads * (int64_t)p.nc;
  if (chunks > kStaticMaxChunks || m3ssd::tc::fwd_workspace_bytes(p) > kStaticScratchBytes)
    return M3SSD_ERR_SCRATCH_LIMIT;
  rc = check_device();
  if (rc) return rc;
  // an optional caller buffer receives the device status word (4 bytes) after the forward
  if (a->workspace != nullptr && a->workspace_bytes < 4) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 4)) return M3SSD_ERR_ALIGN;
  void* scratch = nullptr;
  rc = static_scratch_address(&scratch);
  if (rc) return rc;
  const auto st = static_cast<cudaStream_t>(stream);
  // run_fwd clears the status word, ticket counter and flags it uses before its kernel runs; it
  // always runs the one-pass forward (the chained form needs more scratch than the array holds)
  rc = m3ssd::tc::run_fwd(p, a->y, a->states, scratch, st);
  if (rc != M3SSD_OK || a->workspace == nullptr) return rc;
  return cudaMemcpyAsync(a->workspace, scratch, 4, cudaMemcpyDeviceToDevice, st) == cudaSuccess
             ? M3SSD_OK
             : M3SSD_ERR_LAUNCH;
}

int m3ssd_fwd_proj(const m3ssd_proj_fwd_args* a, void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  Problem p;
  int rc = proj_problem(&a->prob, a->proj, a->proj_strides, a->A, &p);
  if (rc) return rc;
  if (!a->y || !a->states) return M3SSD_ERR_NULL;
  if (!aligned(a->y, 16) || !aligned(a->states, 16)) return M3SSD_ERR_ALIGN;
  const size_t need = fwd_ws(&a->prob, p);
  if (!a->workspace || a->workspace_bytes < need) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 256)) return M3SSD_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  return tc_fwd(p, a->y, a->states, a->workspace, stream, nullptr, nullptr);
}

int m3ssd_bwd_proj(const m3ssd_proj_bwd_args* a, void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  Problem p;
  int rc = proj_problem(&a->prob, a->proj, a->proj_strides, a->A, &p);
  if (rc) return rc;
  if (!a->dy || !a->states || !a->dproj || !a->dA) return M3SSD_ERR_NULL;
  if (!aligned(a->dy, p.y_bf16 ? 2 : 4) || !aligned(a->states, 16) || !aligned(a->dA, 8))
    return M3SSD_ERR_ALIGN;
  // dproj: same conditions as proj (its column blocks leave through TMA stores)
  const int64_t sb = a->dproj_strides[0], st = a->dproj_strides[1];
  if (sb <= 0 || st <= 0) return M3SSD_ERR_SHAPE;
  if (!aligned(a->dproj, 16) || sb % 4 || st % 4) return M3SSD_ERR_ALIGN;
  const size_t need = bwd_ws(&a->prob, p);
  if (!a->workspace || a->workspace_bytes < need) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 256)) return M3SSD_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  long long dys[4];
  for (int i = 0; i < 4; ++i) dys[i] = a->dy_strides[i];
  const ProjCols c = proj_cols(a->prob);
  m3ssd::tc::BwdOut out{};
  out.dx = a->dproj + c.x;
  out.dA = static_cast<float2*>(a->dA);
  out.dB = a->dproj + c.b_re;
  out.dC = a->dproj + c.c_re;
  out.ddt = a->dproj + c.dt;
  out.planar = 1;
  out.s_b = sb;
  out.s_t = st;
  return tc_bwd(p, a->dy, dys, a->states, out, a->workspace, stream, nullptr, nullptr, nullptr);
}

int m3ssd_fwd_state(const m3ssd_fwd_args* a, const void* h0, void* hT, void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  if (!tc_shape(&a->prob) || (a->prob.flags & M3SSD_X_COMPLEX) ||
      a->prob.seqlen % m3ssd::tc::kChunk)
    return M3SSD_ERR_SHAPE;
  Problem p = make_problem(&a->prob);
  rc = fill_inputs(p, a->x, a->x_strides, a->A, a->B, a->b_strides, a->C, a->c_strides, a->dt,
                   a->dt_strides);
  if (rc) return rc;
  if (!m3ssd::tc::fwd_supported(p)) return M3SSD_ERR_SHAPE;
  if (!a->y || !a->states) return M3SSD_ERR_NULL;
  if (!aligned(a->y, 16) || !aligned(a->states, 16) || !aligned(h0, 8) || !aligned(hT, 8))
    return M3SSD_ERR_ALIGN;
  const size_t need = fwd_ws(&a->prob, p);
  if (!a->workspace || a->workspace_bytes < need) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 256)) return M3SSD_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  return tc_fwd(p, a->y, a->states, a->workspace, stream, h0, hT);
}

int m3ssd_bwd_state(const m3ssd_bwd_args* a, const void* hT, const void* dhT, void* dh0,
                    void* stream) {
  if (!a) return M3SSD_ERR_NULL;
  int rc = check_problem(&a->prob);
  if (rc) return rc;
  if (!tc_shape(&a->prob) || (a->prob.flags & M3SSD_X_COMPLEX) ||
      a->prob.seqlen % m3ssd::tc::kChunk)
    return M3SSD_ERR_SHAPE;
  Problem p = make_problem(&a->prob);
  rc = fill_inputs(p, a->x, a->x_strides, a->A, a->B, a->b_strides, a->C, a->c_strides, a->dt,
                   a->dt_strides);
  if (rc) return rc;
  if (!m3ssd::tc::bwd_supported(p)) return M3SSD_ERR_SHAPE;
  if (!a->dy || !a->states || !a->dx || !a->dA || !a->dB || !a->dC || !a->ddt)
    return M3SSD_ERR_NULL;
  if ((hT != nullptr) != (dhT != nullptr)) return M3SSD_ERR_NULL;
  if (!aligned(a->dy, p.y_bf16 ? 2 : 4) || !aligned(a->states, 16) || !aligned(a->dx, 16) ||
      !aligned(a->dA, 8) || !aligned(a->dB, 16) || !aligned(a->dC, 16) || !aligned(a->ddt, 4) ||
      !aligned(hT, 8) || !aligned(dhT, 8) || !aligned(dh0, 8))
    return M3SSD_ERR_ALIGN;
  const size_t need = bwd_ws(&a->prob, p);
  if (!a->workspace || a->workspace_bytes < need) return M3SSD_ERR_WORKSPACE;
  if (!aligned(a->workspace, 256)) return M3SSD_ERR_ALIGN;
  rc = check_device();
  if (rc) return rc;
  long long dys[4];
  for (int i = 0; i < 4; ++i) dys[i] = a->dy_strides[i];
  const m3ssd::tc::BwdOut out = m3ssd::tc::contiguous_bwd_out(
      p, static_cast<float*>(a->dx), static_cast<float2*>(a->dA), static_cast<float2*>(a->dB),
      static_cast<float2*>(a->dC), a->ddt);
  return tc_bwd(p, a->dy, dys, a->states, out, a->workspace, stream, hT, dhT, dh0);
}

int m3ssd_selftest_bounded_waits(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < 256) return M3SSD_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return M3SSD_ERR_ALIGN;
  const int rc = check_device();
  if (rc) return rc;
  return m3ssd::tc::run_selftest_waits(workspace, static_cast<cudaStream_t>(stream));
}

}  // extern "C"

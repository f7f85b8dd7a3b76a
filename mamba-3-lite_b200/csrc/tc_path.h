// Host entry points of the tensor-core (tcgen05, split-bf16) path.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>

#include "m3ssd_common.cuh"
#include "tc_common.cuh"

namespace m3ssd {
namespace tc {

// The tensor-core path blocks the sequence in chunks of 64 positions internally.
constexpr int kChunk = 64;

// kernels enqueued by one run_fwd / run_bwd call (memsets of the flag areas are not kernels)
constexpr int kFwdLaunches = 2;  // k_chunk_prep, k_fwd_tc
constexpr int kBwdLaunches = 2;  // k_bwd_tc, k_bwd_tc_dA (records come from the forward)

// `states` of a tensor-core problem: the chunk-entry states H_z ([b*H+h][chunk][64 p][128] fp32)
// followed by the per-chunk decay records written by the forward and reused by the backward
size_t states_bytes(const Problem& p);
inline size_t states_h_bytes(const Problem& p) {
  return sizeof(float) * 64 * 128 * (size_t)p.Bsz * p.H * ((p.T + 63) / 64);
}

// per-chunk decay records (tc_prep.cu)
size_t chunk_prep_bytes(const Problem& p);
int run_chunk_prep(const Problem& p, ChunkRec* out, cudaStream_t st);

// TMA descriptor for a (B, T, H, N) complex64 tensor viewed as (B, T, H, 2N) fp32, box of
// 64 time steps x 2N floats of one head (zero fill past T); for planar B / C (p.bc_planar) a
// (B, T, 2H, N) fp32 view whose rows h and H + h are the real and imaginary parts of head h, box
// of 64 time steps x N floats
bool encode_bc_tensor_map(CUtensorMap* map, const void* ptr, const Problem& p,
                          const long long st[4]);
// 4D map over a contiguous (B, T, H, row_floats) fp32 output for TMA stores of 64-row tiles in
// 32-float (128-byte) column segments, 128-byte swizzled in shared memory. False if the pointer
// is not 16-byte aligned.
bool encode_out_tensor_map(CUtensorMap* map, void* ptr, const Problem& p, int row_floats);
// 4D map over a contiguous (B, T, H, 64) bfloat16 output, box of 64 rows x 64 values (128-byte
// rows, 128-byte swizzled in shared memory)
bool encode_out_map_bf16(CUtensorMap* map, void* ptr, const Problem& p);
// the same over a strided (B, T, rows, row_floats) fp32 output: strides of a row, a time step and
// a batch entry in floats, each a multiple of 4. False for a misaligned pointer or stride.
bool encode_out_map_strided(CUtensorMap* map, void* ptr, const Problem& p, int row_floats,
                            int rows, long long s_row, long long s_t, long long s_b);

// SM count of the current device (0 if it cannot be queried), cached per device
int sm_count();
// cudaFuncSetAttribute(func, MaxDynamicSharedMemorySize, bytes) once per kernel and device
bool ensure_smem_attr(const void* func, int bytes);

// head_dim = state_dim = 64, real x, B/C with contiguous state dim and 16-byte aligned strides
bool fwd_supported(const Problem& p);
size_t fwd_workspace_bytes(const Problem& p);
// h0 / hT (optional): initial and final state, (B, H, N, D) complex64 contiguous. With G > 1
// (a divisor of the chunk count) every sequence runs as G independent chains of nc / G chunks,
// h0 / hT then hold one state per (sequence, segment) ((b * H + h) * G + segment). `prep` = false
// reuses the chunk records a previous call left in `states`; `clear_status` = false keeps what an
// earlier pass of the same call reported in the status word.
// Complex x runs as two real passes (see run_fwd_complex); for those, `recs` gives the decay
// records' location when they do not follow the H tiles of `states`, `crot` multiplies C as it is
// read and `y_accum` adds y to what y holds instead of storing it.
int run_fwd(const Problem& p, void* y, void* states, void* ws, cudaStream_t st,
            const void* h0 = nullptr, void* hT = nullptr, int G = 1, bool prep = true,
            bool clear_status = true, const void* recs = nullptr, float2 crot = {1.f, 0.f},
            bool y_accum = false);

bool bwd_supported(const Problem& p);

// tc_selftest.cu: the bounded waits give up and report (status word in the first 256 bytes of ws)
int run_selftest_waits(void* ws, cudaStream_t st);
size_t bwd_workspace_bytes(const Problem& p, int G = 1);

// Where the backward writes its gradients. Contiguous (B, T, H, ...) tensors by default; the
// in_proj form (planar = 1) writes dx, dB, dC, ddt into one (B, T, H(D + 4N + 1)) fp32 gradient of
// the projection, strides s_b, s_t in floats, with dB and dC planar (Re, then Im H*N floats on).
struct BwdOut {
  float* dx;
  float2* dA;
  float* dB;      // real parts (planar) or interleaved complex64
  float* dC;
  float* ddt;
  int planar;
  long long s_b, s_t;  // planar: strides of the projection gradient (floats)
};
BwdOut contiguous_bwd_out(const Problem& p, float* dx, float2* dA, float2* dB, float2* dC,
                          float* ddt);
// dy: float32, or bfloat16 with p.y_bf16; strides in elements. State carry (optional, all
// (B, H, N, D) complex64 contiguous): hT the forward's final state and dhT its gradient (both or
// neither), dh0 receives the gradient of the initial state. With G > 1 (a divisor of the chunk
// count) every sequence runs as G independent chains (run_fwd): dhT / dh0 (and hT) then hold one
// state per chain, and `dgam` (one complex per chain: <dhT, conj(end state)>, the chain's last
// chunk's d Sigma term) may be passed ready-made instead of hT.
// recs / crot as for run_fwd; `accum` adds dB, dC, ddt and dA to what they hold (the complex-x
// second pass; dx is written as usual).
int run_bwd(const Problem& p, const void* dy, const long long dys[4], const void* states,
            const BwdOut& out, void* ws, cudaStream_t st, const void* hT = nullptr,
            const void* dhT = nullptr, void* dh0 = nullptr, int G = 1,
            const void* dgam = nullptr, bool clear_status = true, const void* recs = nullptr,
            float2 crot = {1.f, 0.f}, bool accum = false);

// Complex x (x = xr + i xi) through the real-x kernels: the operator is linear in x, so
// y = F(xr; A, B, C, dt) + F(xi; A, B, i C, dt). `states` holds both passes' H tiles and one set
// of decay records (complex_states_bytes). The backward runs both passes' backwards (the second
// one adding into dB, dC, ddt, dA, with dC taking conj(i) = -i of its C gradient) and
// interleaves the two real parts of dx; its workspace adds two real dx buffers
// (complex_bwd_workspace_bytes).
size_t complex_states_bytes(const Problem& p);
size_t complex_bwd_workspace_bytes(const Problem& p);
int run_fwd_complex(const Problem& p, void* y, void* states, void* ws, cudaStream_t st);
int run_bwd_complex(const Problem& p, const void* dy, const long long dys[4], const void* states,
                    float2* dx, float2* dA, float2* dB, float2* dC, float* ddt, void* ws,
                    cudaStream_t st);
// the real-x view of part 0 (real) or 1 (imaginary) of a complex-x problem
Problem real_part_view(const Problem& p, int part);

// Long sequences with few of them: the hand-off chain from chunk to chunk (a few microseconds per
// chunk) bounds the time, not the work. tc_long.cu then runs every sequence as G chains in two
// passes with a short chain over segments in between (forward: local end states, then the true
// entry states; backward: local entry-state gradients, then the true end-state gradients).
// chains_for picks G from the problem's shape alone (1 = the one-pass path), so a forward and a
// backward may pick differently: `states` is the same either way.
int chains_for(const Problem& p, bool backward);
size_t fwd_chains_workspace_bytes(const Problem& p, int G);
size_t bwd_chains_workspace_bytes(const Problem& p, int G);
// tc_chain_state.cu: the chained form's first passes on the tensor cores, one CTA per chain: the
// end state of every chain from a zero entry state (forward: W = B, R = x) or its entry-state
// gradient from a zero end-state gradient (backward: W = C, R = dy), written (n, p) per chain.
// 16-byte rows of B / C (interleaved or planar) and of x / dy only (chain_state_tc_ok).
bool chain_state_tc_ok(const Problem& p, bool forward, const void* r, const long long rs[4],
                       int r_bf16);
int run_chain_state(const Problem& p, bool forward, const void* r, const long long rs[4],
                    int r_bf16, const ChunkRec* recs, int G, float2* out, uint32_t* err,
                    cudaStream_t st);
// the forward / backward with G chains per sequence; h0, hT, dhT, dh0 as for run_fwd / run_bwd
// with G = 1 (one state per sequence, optional)
int run_fwd_chains(const Problem& p, void* y, void* states, void* ws, cudaStream_t st,
                   const void* h0, void* hT, int G);
int run_bwd_chains(const Problem& p, const void* dy, const long long dys[4], const void* states,
                   const BwdOut& out, void* ws, cudaStream_t st, const void* hT, const void* dhT,
                   void* dh0, int G);

}  // namespace tc
}  // namespace m3ssd

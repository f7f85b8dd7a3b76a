/*
 * m3ssd - complex64 chunkwise SSD operator for NVIDIA B200 (sm_100a). Stable C ABI.
 *
 * The operator is the one of models/ssd_complex.py:58-119 (ssd_complex_chunkwise) in
 * atandra2000/Mamba-3-Lite:
 *
 *   a[b,t,h]   = softplus(dt[b,t,h]) * A[h]                         (complex)
 *   s_t        = exp(a_t) s_{t-1} + B_t x_t^T                        (state N x D, complex)
 *   y[b,t,h,:] = Re( sum_n C[b,t,h,n] s_t[n,:] )                     (no conjugate on C)
 *
 * evaluated chunkwise with chunk length `chunk`. T need not be a multiple of `chunk` (the
 * reference's zero padding, models/ssd_complex.py:72-80, never influences t < T).
 *
 * Conventions shared by every entry point:
 *   - All pointers are device pointers on the current CUDA device, except the args structs.
 *   - Strides are in ELEMENTS of the tensor's own element type (float for dt/dy and real x,
 *     complex64 = two floats for A/B/C and complex x). Any strides are accepted; outputs are
 *     written contiguous (row-major in the documented shape).
 *   - `stream` is a cudaStream_t passed as void*; work is only enqueued, never synchronised.
 *   - The library never allocates, frees or synchronises. Scratch is caller-provided, sized by
 *     the *_bytes queries below. Calls are reentrant; concurrent calls need distinct scratch.
 *   - Return value 0 is success; anything else is an m3ssd_status (see m3ssd_strerror).
 *   - The first 4 bytes of each workspace receive a device status word once the enqueued work
 *     has run: 0 = ok, otherwise bits of M3SSD_DEVERR_*. Kernels never trap or spin forever;
 *     a wait that exceeds its bound sets a bit and the call completes with undefined outputs.
 *   - No CPU fallback exists: the only implementation is CUDA code built for sm_100a.
 */
#ifndef M3SSD_H_
#define M3SSD_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define M3SSD_ABI_VERSION 1

#if defined(__GNUC__)
#define M3SSD_API __attribute__((visibility("default")))
#else
#define M3SSD_API
#endif

typedef enum m3ssd_status {
  M3SSD_OK = 0,
  M3SSD_ERR_NULL = 1,          /* a required pointer is NULL */
  M3SSD_ERR_SHAPE = 2,         /* a size is <= 0 or inconsistent */
  M3SSD_ERR_CHUNK = 3,         /* chunk size outside [1, 256] */
  M3SSD_ERR_DIM_LIMIT = 4,     /* head_dim or state_dim above 256 (same cap as the reference's
                                  Triton wrapper, models/ssd_triton.py:27-28, 139-146) */
  M3SSD_ERR_ALIGN = 5,         /* pointer not aligned to its element type */
  M3SSD_ERR_WORKSPACE = 6,     /* scratch pointer NULL or smaller than required */
  M3SSD_ERR_LAUNCH = 7,        /* a kernel launch failed (cudaGetLastError) */
  M3SSD_ERR_DEVICE = 8,        /* current device is not sm_100 or cannot be queried */
  M3SSD_ERR_FLAGS = 9,         /* unknown flag bits */
  M3SSD_ERR_OVERFLOW = 10,     /* a size product overflows the 64-bit index space */
  M3SSD_ERR_SCRATCH_LIMIT = 11 /* problem too large for m3ssd_fwd_static_scratch */
} m3ssd_status;

/* device status bits (first word of the workspace) */
#define M3SSD_DEVERR_TMA_WAIT   0x1u  /* a TMA transfer did not complete within the bound */
#define M3SSD_DEVERR_MMA_WAIT   0x2u  /* a tcgen05.mma group did not complete within the bound */
#define M3SSD_DEVERR_FLAG_WAIT  0x4u  /* a chunk-state hand-off flag was not set within the bound */

/* problem flags */
#define M3SSD_X_COMPLEX      0x1u   /* x (and dx) are complex64; otherwise float32 */
#define M3SSD_PREC_AUTO      0x0u   /* fastest path supported for the shape */
#define M3SSD_PREC_FP32      0x10u  /* fp32 CUDA-core arithmetic everywhere */
#define M3SSD_PREC_TENSOR    0x20u  /* tcgen05 tensor-core tiles where the shape has them:
                                       split-bf16 operands (hi + lo), fp32 accumulation */
#define M3SSD_PREC_MASK      0x30u
#define M3SSD_Y_BF16         0x100u /* y (forward output) and dy (backward input) are bfloat16
                                       instead of float32: the output is rounded to nearest-even
                                       once, in the store; dy is widened exactly on load. For the
                                       block, whose next op (MIMO, models/mimo.py:27) runs in bf16
                                       under autocast. Tensor-core path only: with any other path
                                       the calls return M3SSD_ERR_SHAPE. */

typedef struct m3ssd_problem {
  int64_t batch;      /* B */
  int64_t seqlen;     /* T */
  int64_t nheads;     /* H */
  int64_t headdim;    /* D */
  int64_t dstate;     /* N */
  int64_t chunk;      /* chunk length C (problems the tensor-core path can take are blocked
                         at 64 internally; the result does not depend on the blocking) */
  uint32_t flags;     /* M3SSD_X_COMPLEX | one M3SSD_PREC_* | M3SSD_Y_BF16 */
  uint32_t reserved;  /* must be 0 */
} m3ssd_problem;

typedef struct m3ssd_fwd_args {
  m3ssd_problem prob;
  const void* x;   int64_t x_strides[4];   /* (B,T,H,D) float32 or complex64 */
  const void* A;                           /* (H,) complex64, contiguous */
  const void* B;   int64_t b_strides[4];   /* (B,T,H,N) complex64 */
  const void* C;   int64_t c_strides[4];   /* (B,T,H,N) complex64 */
  const float* dt; int64_t dt_strides[3];  /* (B,T,H) float32, pre-softplus */
  void* y;                                 /* out: (B,T,H,D) float32 contiguous (bfloat16 with
                                              M3SSD_Y_BF16) */
  void* states;                            /* out: m3ssd_states_bytes() bytes; chunk-entry states
                                              kept for m3ssd_bwd (layout internal) */
  void* workspace;                         /* scratch, m3ssd_fwd_workspace_bytes() bytes */
  size_t workspace_bytes;
} m3ssd_fwd_args;

typedef struct m3ssd_bwd_args {
  m3ssd_problem prob;                      /* identical to the forward call */
  const void* x;   int64_t x_strides[4];
  const void* A;
  const void* B;   int64_t b_strides[4];
  const void* C;   int64_t c_strides[4];
  const float* dt; int64_t dt_strides[3];
  const void* dy; int64_t dy_strides[4];   /* (B,T,H,D) float32 (bfloat16 with M3SSD_Y_BF16):
                                              gradient of y */
  const void* states;                      /* from the matching m3ssd_fwd call */
  void* dx;                                /* out: (B,T,H,D) float32 (complex64 if X_COMPLEX) */
  void* dA;                                /* out: (H,) complex64 */
  void* dB;                                /* out: (B,T,H,N) complex64 */
  void* dC;                                /* out: (B,T,H,N) complex64 */
  float* ddt;                              /* out: (B,T,H) float32 */
  void* workspace;                         /* scratch, m3ssd_bwd_workspace_bytes() bytes */
  size_t workspace_bytes;
} m3ssd_bwd_args;

/* ABI version of the loaded library (M3SSD_ABI_VERSION at build time). */
M3SSD_API int m3ssd_abi_version(void);

/* Human-readable text for a status code; never NULL. */
M3SSD_API const char* m3ssd_strerror(int status);

/* Validate a problem description without touching the device. Returns an m3ssd_status. */
M3SSD_API int m3ssd_check_problem(const m3ssd_problem* prob);

/* Bytes of the `states` buffer written by m3ssd_fwd and read by m3ssd_bwd (0 on bad input). */
M3SSD_API size_t m3ssd_states_bytes(const m3ssd_problem* prob);
/* Scratch bytes needed by m3ssd_fwd / m3ssd_bwd for this problem (0 on bad input). */
M3SSD_API size_t m3ssd_fwd_workspace_bytes(const m3ssd_problem* prob);
M3SSD_API size_t m3ssd_bwd_workspace_bytes(const m3ssd_problem* prob);

/* Forward. Replaces the body of ssd_complex_chunkwise (models/ssd_complex.py:69-119) and the
 * per-chunk kernel launch it dispatches to (models/ssd_triton.py:163-197). Writes y and states. */
M3SSD_API int m3ssd_fwd(const m3ssd_fwd_args* args, void* stream);

/* Backward. Replaces torch.autograd through models/ssd_complex.py:82-119 and the recompute
 * backward of the per-chunk kernel (models/ssd_triton.py:210-225). Writes dx, dA, dB, dC, ddt in
 * PyTorch's convention for complex tensors (grad = dL/dRe + i dL/dIm). dA is summed over
 * batch and time. */
M3SSD_API int m3ssd_bwd(const m3ssd_bwd_args* args, void* stream);

/* Name of the implementation m3ssd_fwd / m3ssd_bwd use for this problem ("tcgen05-bf16x2",
 * "simt-fp32"). The tensor-core path needs head_dim = state_dim = 64, real x, and B/C with a
 * contiguous state dimension and 16-byte aligned strides; otherwise the fp32 path runs. On the
 * tensor-core path y (forward) and dx, dB, dC (backward) must be 16-byte aligned (any allocator's
 * default), else the call returns M3SSD_ERR_ALIGN: its outputs leave through TMA stores and its
 * `states` layout is its own, so it has no fallback for them. Host-only query, no device work. */
M3SSD_API const char* m3ssd_fwd_path(const m3ssd_problem* prob);
M3SSD_API const char* m3ssd_bwd_path(const m3ssd_problem* prob);

/* Number of kernel launches one m3ssd_fwd (backward = 0) or m3ssd_bwd (backward = 1) call
 * enqueues for this problem (0 on bad input). Host-only query. */
M3SSD_API int m3ssd_launch_count(const m3ssd_problem* prob, int backward);

/* Forward that allocates nothing, for callers that cannot allocate device memory when they call
 * the operator (a serving runtime that plans all device memory up front and forbids allocation
 * on the request path, or code inside another framework's step with no allocator at hand).
 * No counterpart in the reference. Same arguments and results as m3ssd_fwd, except for the
 * workspace: the scratch this forward needs (status word, ticket counter, one hand-off flag per
 * chunk) is a fixed device array inside the library, 131,328 bytes, held on every GPU that loads
 * the library until exit.
 *   - `workspace` may be NULL (workspace_bytes ignored). If it is not NULL it must hold at least
 *     4 bytes (M3SSD_ERR_WORKSPACE) at a 4-byte aligned address (M3SSD_ERR_ALIGN): after the
 *     forward the call copies the device status word there (cudaMemcpyAsync on `stream`), so it
 *     reads as m3ssd_fwd's status word at offset 0 of its workspace. With NULL no status is
 *     reported.
 *   - Only the tensor-core forward: head_dim = state_dim = 64, real x, B/C with a contiguous
 *     state dimension and 16-byte aligned strides; otherwise M3SSD_ERR_SHAPE. y and states must
 *     be 16-byte aligned (M3SSD_ERR_ALIGN). It always runs the one-pass form: for few long
 *     sequences (where m3ssd_fwd splits each sequence into chains) it is several times slower
 *     than m3ssd_fwd, with the same results.
 *   - batch * nheads * ceil(seqlen / 64) must be <= 32768, otherwise M3SSD_ERR_SCRATCH_LIMIT.
 *   - The first call on a device looks up the array's device address (with that device
 *     current), and again after the device's context changed (cudaDeviceReset); make that first
 *     call before any stream capture.
 *   - Every call uses the same array and leaves its contents behind; each call clears what must
 *     start at zero before its kernel runs. Calls that overlap on the GPU (other streams, other
 *     host threads) race on the array: serialise them.
 *   - Calls no cudaMalloc/cudaFree and no allocating library routine. */
M3SSD_API int m3ssd_fwd_static_scratch(const m3ssd_fwd_args* args, void* stream);

/* ---- The block's input projection as the operator's input -------------------------------------
 * models/mamba_block.py:73-88 slices the in_proj output `proj` (B, T, H(D + 4N + 1)) into x, B, C
 * and dt, upcasts the slices and interleaves B and C into new complex64 tensors (torch.complex,
 * :78 and :82) before calling ssd_complex_chunkwise; its backward then assembles the projection's
 * gradient from six slice gradients. These two entry points take `proj` itself: columns, per
 * token, in the block's order
 *     x [H*D] | Re B [H*N] | Im B [H*N] | Re C [H*N] | Im C [H*N] | dt [H]
 * (head-major inside each block, float32, last dimension contiguous). The forward computes the same
 * y as m3ssd_fwd on the unpacked tensors and writes the same `states`; the backward writes dA and
 * the gradient of the whole projection, `dproj`, in the same column layout (every column written).
 *   - Tensor-core shapes only: head_dim = state_dim = 64, flags M3SSD_PREC_AUTO or
 *     M3SSD_PREC_TENSOR (no M3SSD_X_COMPLEX); otherwise M3SSD_ERR_SHAPE.
 *   - proj, dproj, y: 16-byte aligned; batch and time strides of proj and dproj (in floats)
 *     multiples of 4 and H*D a multiple of 4 (the B and C blocks are read and written by TMA);
 *     otherwise M3SSD_ERR_ALIGN.
 *   - states / workspace sizes: m3ssd_states_bytes, m3ssd_fwd_workspace_bytes,
 *     m3ssd_bwd_workspace_bytes of the same problem. No counterpart in the reference's API. */
typedef struct m3ssd_proj_fwd_args {
  m3ssd_problem prob;
  const float* proj; int64_t proj_strides[2];  /* (B, T, H(D+4N+1)) fp32; strides of b, t */
  const void* A;                               /* (H,) complex64 */
  void* y;                                     /* out: (B,T,H,D) float32 (bfloat16 with
                                                  M3SSD_Y_BF16) contiguous */
  void* states;                                /* out: as m3ssd_fwd */
  void* workspace;
  size_t workspace_bytes;
} m3ssd_proj_fwd_args;

typedef struct m3ssd_proj_bwd_args {
  m3ssd_problem prob;                          /* identical to the forward call */
  const float* proj; int64_t proj_strides[2];
  const void* A;
  const void* dy; int64_t dy_strides[4];       /* (B,T,H,D) float32 (bfloat16 with
                                                  M3SSD_Y_BF16): gradient of y */
  const void* states;                          /* from the matching m3ssd_fwd_proj / m3ssd_fwd */
  float* dproj; int64_t dproj_strides[2];      /* out: (B, T, H(D+4N+1)) fp32, proj's layout */
  void* dA;                                    /* out: (H,) complex64 */
  void* workspace;
  size_t workspace_bytes;
} m3ssd_proj_bwd_args;

M3SSD_API int m3ssd_fwd_proj(const m3ssd_proj_fwd_args* args, void* stream);
M3SSD_API int m3ssd_bwd_proj(const m3ssd_proj_bwd_args* args, void* stream);

/* ---- State carry -------------------------------------------------------------------------------
 * The operator over one segment of a longer sequence: the reference's recurrence
 * (models/ssd_complex.py:17-33) started from an initial state h0 instead of zero, returning the
 * state after the segment's last position. A sequence cut into segments of multiples of 64
 * positions, each call fed the previous call's hT, gives the same y as one call over the whole
 * sequence, and the backward chains the same way (dhT of a segment = dh0 of the next). No
 * counterpart in the reference's API (its operator always starts from zero and drops the state).
 * States are (B, H, N, D) complex64, contiguous: s[n, :] of the recurrence for every (b, h).
 *   - Tensor-core shapes only (as m3ssd_fwd_proj) and seqlen a multiple of 64; otherwise
 *     M3SSD_ERR_SHAPE. y, dx, dB, dC: 16-byte aligned; state pointers 8-byte aligned.
 *   - m3ssd_fwd_state: h0 NULL = zero initial state (m3ssd_fwd's result); hT NULL = not written.
 *   - m3ssd_bwd_state: `states` from the matching m3ssd_fwd_state (it carries h0 into the
 *     gradients). hT (the forward's final state) and dhT (its gradient) come together or both
 *     NULL (M3SSD_ERR_NULL otherwise); dh0 NULL = the initial state's gradient is not written.
 *     Gradients in the convention of m3ssd_bwd; dh0 = dL/dRe h0 + i dL/dIm h0. */
M3SSD_API int m3ssd_fwd_state(const m3ssd_fwd_args* args, const void* h0, void* hT, void* stream);
M3SSD_API int m3ssd_bwd_state(const m3ssd_bwd_args* args, const void* hT, const void* dhT,
                              void* dh0, void* stream);

/* Test aid, no counterpart in the reference: checks that the library's bounded waits end instead
 * of hanging. One thread waits on an mbarrier nobody arrives at and on a hand-off flag nobody
 * sets, with the same helpers the tensor-core kernels use; each gives up after about a second.
 * `workspace` (>= 256 device bytes) is cleared first; once the work has run its status word reads
 * M3SSD_DEVERR_MMA_WAIT | M3SSD_DEVERR_FLAG_WAIT and the CUDA context remains usable. Enqueues only.
 * Returns M3SSD_ERR_WORKSPACE for a missing or smaller workspace, M3SSD_ERR_DEVICE without an
 * sm_100 GPU. */
M3SSD_API int m3ssd_selftest_bounded_waits(void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* M3SSD_H_ */

"""Drop-in replacement for the reference's complex chunkwise SSD operator.

``ssd_complex_chunkwise(x, A, B_t, C_t, dt, chunk_size=64, ssd_dispatch=...)`` has the signature,
shapes, dtypes and return value of models/ssd_complex.py:58-119 (atandra2000/Mamba-3-Lite):

    x     (B, T, H, D) float32 (the block's real ``x_ssm``) or complex64 (the reference tests)
    A     (H,) complex64, one complex decay rate per head (models/mamba_block.py:41)
    B_t   (B, T, H, N) complex64
    C_t   (B, T, H, N) complex64
    dt    (B, T, H) float32, pre-softplus (the operator applies softplus itself)
    ->    (B, T, H, D) float32 = Re(Y)

It is differentiable with respect to all five inputs, with PyTorch's gradient convention for
complex tensors (grad = dL/dRe + i dL/dIm; dA summed over batch and time), and runs only on CUDA
through libm3ssd.so (include/m3ssd.h). There is no CPU fallback: CPU tensors raise.

Differences from the reference, all deliberate:
* ``exp`` is evaluated only inside the causal region, so strong decays that overflow the
  reference's exp-then-mask (models/ssd_complex.py:52, :107) to NaN stay finite here.
* The chunk-to-chunk carry is a sequential scan over chunks instead of the O(n_chunks^2) decay
  matrix (models/ssd_complex.py:98-111); it is the same sum with no long-range cumsum
  differences.
* ``ssd_dispatch`` is accepted for call-site compatibility (models/mamba_block.py:100-121 passes
  "triton" or nothing); every value runs the CUDA kernels here.
* ``precision`` (extra keyword) selects "auto" (default, same as "tensor"), "fp32" (CUDA cores,
  fp32 everywhere) or "tensor" (tcgen05 tensor-core tiles with split-bf16 operands and fp32
  accumulation where the shape has them: head_dim = state_dim = 64; complex x runs as two
  passes of the real-x kernels, y = F(Re x; C) + F(Im x; iC)).
* ``y_dtype`` (extra keyword): torch.float32 (default, the reference's output) or torch.bfloat16,
  for the block whose next op (MIMO, models/mimo.py:27) runs in bf16 under autocast. The
  tensor-core kernels then round y to bf16 in their store and read its gradient as bf16, which
  saves the cast kernels autocast would run on both sides; y is bit-identical to
  ``y_fp32.to(torch.bfloat16)``. Other shapes compute in fp32 and cast.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _lib

ctypes_ref = ctypes.byref

_PREC = {"auto": _lib.M3SSD_PREC_AUTO, "fp32": _lib.M3SSD_PREC_FP32,
         "tensor": _lib.M3SSD_PREC_TENSOR}


def _y_dtype(flags):
    return torch.bfloat16 if flags & _lib.M3SSD_Y_BF16 else torch.float32


def _problem(x, B_t, chunk, flags):
    Bsz, T, H, D = x.shape
    N = B_t.shape[-1]
    return _lib.Problem(Bsz, T, H, D, N, int(chunk), int(flags), 0)


_plans = {}


def _plan(x, B_t, chunk, flags):
    """Problem struct and buffer sizes of a call, validated once per (shape, chunk, flags)."""
    key = (tuple(x.shape), B_t.shape[-1], int(chunk), int(flags))
    plan = _plans.get(key)
    if plan is None:
        lib = _lib.load()
        prob = _problem(x, B_t, chunk, flags)
        _lib.check(lib.m3ssd_check_problem(ctypes_ref(prob)))
        plan = (prob, int(lib.m3ssd_states_bytes(ctypes_ref(prob))),
                int(lib.m3ssd_fwd_workspace_bytes(ctypes_ref(prob))),
                int(lib.m3ssd_bwd_workspace_bytes(ctypes_ref(prob))))
        if len(_plans) > 256:
            _plans.clear()
        _plans[key] = plan
    return plan


def _strides(t, n):
    s = t.stride()
    assert len(s) == n
    return s


def _stream_ptr(device):
    return torch.cuda.current_stream(device).cuda_stream


# Scratch of a call (status word, ticket counter, hand-off flags and rings) is reused per
# (device, current stream) up to this size: calls on one stream run in order, so they never use it
# at the same time. Larger scratch, and scratch during stream capture, is allocated per call.
_WS_CACHE_MAX = 64 << 20
_ws_cache = {}
_ws_lock = threading.Lock()


def _workspace(dev, nbytes):
    nbytes = max(int(nbytes), 256)
    if nbytes > _WS_CACHE_MAX or torch.cuda.is_current_stream_capturing():
        return torch.empty(nbytes, dtype=torch.uint8, device=dev)
    key = (dev.index, torch.cuda.current_stream(dev).cuda_stream)
    with _ws_lock:
        buf = _ws_cache.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            _ws_cache[key] = buf
    return buf


def _check_device_status(ws, what):
    """With M3SSD_CHECK=1 in the environment, synchronise and raise if a kernel reported a
    bounded-wait timeout in the workspace status word (a debugging aid; off by default)."""
    if os.environ.get("M3SSD_CHECK", "0") in ("", "0"):
        return
    torch.cuda.synchronize(ws.device)
    code = int(ws[:4].view(torch.int32).item())
    if code != 0:
        raise RuntimeError(f"m3ssd {what}: device status word {code:#x} (bounded wait expired)")


def _check_inputs(x, A, B_t, C_t, dt, chunk_size):
    for name, t in (("x", x), ("A", A), ("B_t", B_t), ("C_t", C_t), ("dt", dt)):
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if t.device.type != "cuda":
            raise RuntimeError(
                f"m3ssd: {name} is on {t.device}; the operator runs only on CUDA (sm_100a) "
                "and has no CPU fallback")
    if x.dim() != 4:
        raise ValueError(f"x must be (B, T, H, D), got shape {tuple(x.shape)}")
    Bsz, T, H, D = x.shape
    if B_t.dim() != 4 or C_t.dim() != 4:
        raise ValueError("B_t and C_t must be (B, T, H, N)")
    N = B_t.shape[-1]
    if tuple(B_t.shape) != (Bsz, T, H, N) or tuple(C_t.shape) != (Bsz, T, H, N):
        raise ValueError(f"B_t/C_t shapes {tuple(B_t.shape)}, {tuple(C_t.shape)} do not match "
                         f"x {tuple(x.shape)}")
    if tuple(dt.shape) != (Bsz, T, H):
        raise ValueError(f"dt must be (B, T, H) = {(Bsz, T, H)}, got {tuple(dt.shape)}")
    if tuple(A.shape) != (H,):
        raise ValueError(f"A must be (H,) = ({H},), got {tuple(A.shape)}")
    if x.dtype not in (torch.float32, torch.complex64):
        raise TypeError(f"x must be float32 or complex64, got {x.dtype}")
    for name, t in (("A", A), ("B_t", B_t), ("C_t", C_t)):
        if t.dtype != torch.complex64:
            raise TypeError(f"{name} must be complex64, got {t.dtype}")
    if dt.dtype != torch.float32:
        raise TypeError(f"dt must be float32, got {dt.dtype}")
    devs = {t.device for t in (x, A, B_t, C_t, dt)}
    if len(devs) != 1:
        raise RuntimeError(f"m3ssd: inputs are on different devices {devs}")
    if not (1 <= int(chunk_size) <= 256):
        raise ValueError(f"chunk_size {chunk_size} exceeds the supported range [1, 256]")
    if D > 256 or N > 256:
        raise ValueError(f"head_dim {D} / state_dim {N} exceeds the limit 256")


def _fwd_impl(x, A, B_t, C_t, dt, chunk, flags):
    lib = _lib.load()
    dev = x.device
    A = A.contiguous()
    prob, states_bytes, ws_bytes, _ = _plan(x, B_t, chunk, flags)
    y = torch.empty(x.shape, dtype=_y_dtype(flags), device=dev)
    states = torch.empty(states_bytes, dtype=torch.uint8, device=dev)
    ws = _workspace(dev, ws_bytes)
    args = _lib.FwdArgs()
    args.prob = prob
    args.x, args.x_strides = x.data_ptr(), _lib.I64x4(*_strides(x, 4))
    args.A = A.data_ptr()
    args.B, args.b_strides = B_t.data_ptr(), _lib.I64x4(*_strides(B_t, 4))
    args.C, args.c_strides = C_t.data_ptr(), _lib.I64x4(*_strides(C_t, 4))
    args.dt, args.dt_strides = dt.data_ptr(), _lib.I64x3(*_strides(dt, 3))
    args.y = y.data_ptr()
    args.states = states.data_ptr()
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
    with torch.cuda.device(dev):
        _lib.check(lib.m3ssd_fwd(ctypes_ref(args), _stream_ptr(dev)))
    _check_device_status(ws, "forward")
    return y, states


@torch.library.custom_op("m3ssd::ssd_fwd", mutates_args=(), device_types="cuda")
def ssd_fwd(x: torch.Tensor, A: torch.Tensor, B_t: torch.Tensor, C_t: torch.Tensor,
            dt: torch.Tensor, chunk: int, flags: int) -> tuple[torch.Tensor, torch.Tensor]:
    return _fwd_impl(x, A, B_t, C_t, dt, chunk, flags)


@ssd_fwd.register_fake
def _(x, A, B_t, C_t, dt, chunk, flags):
    lib = _lib.load()
    prob = _problem(x, B_t, chunk, flags)
    nbytes = int(lib.m3ssd_states_bytes(ctypes_ref(prob)))
    return (torch.empty(x.shape, dtype=_y_dtype(flags), device=x.device),
            torch.empty(nbytes, dtype=torch.uint8, device=x.device))


def _bwd_impl(dy, x, A, B_t, C_t, dt, states, chunk, flags):
    lib = _lib.load()
    dev = x.device
    A = A.contiguous()
    if dy.dtype != _y_dtype(flags):
        dy = dy.to(_y_dtype(flags))
    prob, _, _, ws_bytes = _plan(x, B_t, chunk, flags)
    dx = torch.empty(x.shape, dtype=x.dtype, device=dev)
    dA = torch.empty(A.shape, dtype=torch.complex64, device=dev)
    dB = torch.empty(B_t.shape, dtype=torch.complex64, device=dev)
    dC = torch.empty(C_t.shape, dtype=torch.complex64, device=dev)
    ddt = torch.empty(dt.shape, dtype=torch.float32, device=dev)
    ws = _workspace(dev, ws_bytes)
    args = _lib.BwdArgs()
    args.prob = prob
    args.x, args.x_strides = x.data_ptr(), _lib.I64x4(*_strides(x, 4))
    args.A = A.data_ptr()
    args.B, args.b_strides = B_t.data_ptr(), _lib.I64x4(*_strides(B_t, 4))
    args.C, args.c_strides = C_t.data_ptr(), _lib.I64x4(*_strides(C_t, 4))
    args.dt, args.dt_strides = dt.data_ptr(), _lib.I64x3(*_strides(dt, 3))
    args.dy, args.dy_strides = dy.data_ptr(), _lib.I64x4(*_strides(dy, 4))
    args.states = states.data_ptr()
    args.dx, args.dA, args.dB, args.dC, args.ddt = (dx.data_ptr(), dA.data_ptr(), dB.data_ptr(),
                                                    dC.data_ptr(), ddt.data_ptr())
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
    with torch.cuda.device(dev):
        _lib.check(lib.m3ssd_bwd(ctypes_ref(args), _stream_ptr(dev)))
    _check_device_status(ws, "backward")
    return dx, dA, dB, dC, ddt


@torch.library.custom_op("m3ssd::ssd_bwd", mutates_args=(), device_types="cuda")
def ssd_bwd(dy: torch.Tensor, x: torch.Tensor, A: torch.Tensor, B_t: torch.Tensor,
            C_t: torch.Tensor, dt: torch.Tensor, states: torch.Tensor, chunk: int,
            flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                 torch.Tensor]:
    return _bwd_impl(dy, x, A, B_t, C_t, dt, states, chunk, flags)


@ssd_bwd.register_fake
def _(dy, x, A, B_t, C_t, dt, states, chunk, flags):
    return (torch.empty(x.shape, dtype=x.dtype, device=x.device),
            torch.empty(A.shape, dtype=torch.complex64, device=x.device),
            torch.empty(B_t.shape, dtype=torch.complex64, device=x.device),
            torch.empty(C_t.shape, dtype=torch.complex64, device=x.device),
            torch.empty(dt.shape, dtype=torch.float32, device=x.device))


def _setup_context(ctx, inputs, output):
    x, A, B_t, C_t, dt, chunk, flags = inputs
    _, states = output
    ctx.save_for_backward(x, A, B_t, C_t, dt, states)
    ctx.chunk = chunk
    ctx.flags = flags
    ctx.mark_non_differentiable(states)
    # no zero-filled gradient for `states` (hundreds of MB at training sizes): unused grads
    # arrive as None
    ctx.set_materialize_grads(False)


def _backward(ctx, dy, _dstates):
    x, A, B_t, C_t, dt, states = ctx.saved_tensors
    if dy is None:
        dy = torch.zeros(x.shape, dtype=_y_dtype(ctx.flags), device=x.device)
    dx, dA, dB, dC, ddt = ssd_bwd(dy, x, A, B_t, C_t, dt, states, ctx.chunk, ctx.flags)
    return dx, dA, dB, dC, ddt, None, None


ssd_fwd.register_autograd(_backward, setup_context=_setup_context)


class _SsdFunction(torch.autograd.Function):
    """The eager path: the same kernels as the m3ssd::ssd_fwd / ssd_bwd custom ops without the
    op dispatch (the custom ops serve torch.compile, which traces them through register_fake)."""

    @staticmethod
    def forward(ctx, x, A, B_t, C_t, dt, chunk, flags):
        y, states = _fwd_impl(x, A, B_t, C_t, dt, chunk, flags)
        ctx.save_for_backward(x, A, B_t, C_t, dt, states)
        ctx.chunk = chunk
        ctx.flags = flags
        return y

    @staticmethod
    def backward(ctx, dy):
        x, A, B_t, C_t, dt, states = ctx.saved_tensors
        dx, dA, dB, dC, ddt = _bwd_impl(dy, x, A, B_t, C_t, dt, states, ctx.chunk, ctx.flags)
        return dx, dA, dB, dC, ddt, None, None


def ssd_complex_chunkwise(x: torch.Tensor, A: torch.Tensor, B_t: torch.Tensor,
                          C_t: torch.Tensor, dt: torch.Tensor, chunk_size: int = 64,
                          ssd_dispatch: str = "cuda", precision: str = "auto",
                          y_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Complex chunkwise SSD, forward and backward on the GPU (see the module docstring)."""
    del ssd_dispatch  # every dispatch value runs the CUDA kernels
    _check_inputs(x, A, B_t, C_t, dt, chunk_size)
    if precision not in _PREC:
        raise ValueError(f"precision must be one of {sorted(_PREC)}, got {precision!r}")
    if y_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"y_dtype must be torch.float32 or torch.bfloat16, got {y_dtype}")
    flags = _PREC[precision] | (_lib.M3SSD_X_COMPLEX if x.dtype == torch.complex64 else 0)
    bf16_in_kernel = y_dtype == torch.bfloat16 and _bf16_store_ok(x, B_t, C_t, flags)
    if bf16_in_kernel:
        flags |= _lib.M3SSD_Y_BF16
    with torch.autocast("cuda", enabled=False):
        if torch.compiler.is_compiling():
            y, _ = ssd_fwd(x, A, B_t, C_t, dt, int(chunk_size), int(flags))
        else:
            y = _SsdFunction.apply(x, A, B_t, C_t, dt, int(chunk_size), int(flags))
    return y.to(y_dtype) if y.dtype != y_dtype else y


def _bf16_store_ok(x, B_t, C_t, flags):
    """The tensor-core path runs for this call (so the kernels can store y as bf16)."""
    Bsz, T, H, D = x.shape
    N = B_t.shape[-1]
    if D != 64 or N != 64 or flags & (_lib.M3SSD_X_COMPLEX | _lib.M3SSD_PREC_FP32):
        return False
    # B / C operands through TMA: contiguous state dim, 16-byte aligned base and strides
    for t in (B_t, C_t):
        s = t.stride()
        if s[3] != 1 or any(v % 2 for v in s[:3]) or t.data_ptr() % 16:
            return False
    return True


def implementation(x_shape, N, chunk_size=64, complex_x=False, precision="auto"):
    """Names of the forward and backward implementations the library picks for a shape."""
    lib = _lib.load()
    Bsz, T, H, D = x_shape
    flags = _PREC[precision] | (_lib.M3SSD_X_COMPLEX if complex_x else 0)
    prob = _lib.Problem(Bsz, T, H, D, N, int(chunk_size), int(flags), 0)
    return (lib.m3ssd_fwd_path(ctypes_ref(prob)).decode(),
            lib.m3ssd_bwd_path(ctypes_ref(prob)).decode())

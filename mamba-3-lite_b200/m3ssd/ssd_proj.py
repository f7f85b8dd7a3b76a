"""The block's SSD input path fused into the operator (models/mamba_block.py:73-88).

``ssd_from_proj(proj, A, n_heads, head_dim, state_dim, chunk_size=64)`` takes the block's in_proj
output ``proj`` (B, T, H(D + 4N + 1)) and returns what the block computes from it:

    x_ssm = proj[..., :H*D].reshape(B, T, H, D).float()                         # :74
    B_t = torch.complex(Re B, Im B).reshape(B, T, H, N)  (columns H*D .. H*D+2HN) # :76-78
    C_t = torch.complex(Re C, Im C).reshape(B, T, H, N)  (the next 2HN columns)   # :80-82
    dt = proj[..., -H:].float()                                                   # :84
    y = ssd_complex_chunkwise(x_ssm, A, B_t, C_t, dt, chunk_size)                  # :86, :102

The forward kernels read x, the planar real and imaginary parts of B and C, and dt straight from
``proj`` (no complex64 copies of B and C), and the backward writes the gradient of the whole
projection in proj's column layout in one pass (autograd through the slices would build it from
six slice gradients). Results are identical to the composition above with the CUDA operator:
same kernels, same operand values, same order of arithmetic.

Shapes the tensor-core kernels take (head_dim = state_dim = 64) with a 16-byte aligned fp32
projection whose batch / time strides are multiples of 4 floats run fused; anything else runs the
composition above (still on the GPU). A bf16 / fp16 projection (the block under autocast) is
upcast once, as the block's ``.float()`` calls do.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .ssd_complex import (_check_device_status, _PREC, ssd_complex_chunkwise, _stream_ptr,
                          _workspace, _y_dtype)

ctypes_ref = ctypes.byref


def proj_width(n_heads: int, head_dim: int, state_dim: int) -> int:
    """Columns of the block's in_proj output (models/mamba_block.py:35)."""
    return n_heads * (head_dim + 4 * state_dim + 1)


def unpack_proj(proj: torch.Tensor, n_heads: int, head_dim: int, state_dim: int):
    """The block's own unpacking (models/mamba_block.py:74-84): x_ssm, B_t, C_t, dt."""
    Bsz, T, _ = proj.shape
    H, D, N = n_heads, head_dim, state_dim
    x_ssm = proj[..., :H * D].reshape(Bsz, T, H, D).float()
    b_re = proj[..., H * D:H * D + H * N].float()
    b_im = proj[..., H * D + H * N:H * D + 2 * H * N].float()
    B_t = torch.complex(b_re, b_im).reshape(Bsz, T, H, N)
    c_re = proj[..., H * D + 2 * H * N:H * D + 3 * H * N].float()
    c_im = proj[..., H * D + 3 * H * N:H * D + 4 * H * N].float()
    C_t = torch.complex(c_re, c_im).reshape(Bsz, T, H, N)
    dt = proj[..., -H:].float()
    return x_ssm, B_t, C_t, dt


def _problem(proj, H, D, N, chunk, flags):
    Bsz, T, _ = proj.shape
    return _lib.Problem(Bsz, T, H, D, N, int(chunk), int(flags), 0)


def fusable(proj: torch.Tensor, n_heads: int, head_dim: int, state_dim: int,
            precision: str = "auto") -> bool:
    """True when the fused kernels take this projection (the conditions of m3ssd_fwd_proj)."""
    if head_dim != 64 or state_dim != 64 or precision == "fp32":
        return False
    if proj.stride(-1) != 1 or (n_heads * head_dim) % 4:
        return False
    if proj.stride(0) % 4 or proj.stride(1) % 4:
        return False
    # dproj is allocated contiguous: its time stride is the width
    if proj_width(n_heads, head_dim, state_dim) % 4:
        return False
    return proj.dtype == torch.float32 and proj.data_ptr() % 16 == 0


@torch.library.custom_op("m3ssd::ssd_proj_fwd", mutates_args=(), device_types="cuda")
def ssd_proj_fwd(proj: torch.Tensor, A: torch.Tensor, H: int, D: int, N: int, chunk: int,
                 flags: int) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    dev = proj.device
    A = A.contiguous()
    prob = _problem(proj, H, D, N, chunk, flags)
    _lib.check(lib.m3ssd_check_problem(ctypes_ref(prob)))
    Bsz, T, _ = proj.shape
    y = torch.empty((Bsz, T, H, D), dtype=_y_dtype(flags), device=dev)
    states = torch.empty(int(lib.m3ssd_states_bytes(ctypes_ref(prob))), dtype=torch.uint8,
                         device=dev)
    ws_bytes = int(lib.m3ssd_fwd_workspace_bytes(ctypes_ref(prob)))
    ws = _workspace(dev, ws_bytes)
    args = _lib.ProjFwdArgs()
    args.prob = prob
    args.proj, args.proj_strides = proj.data_ptr(), _lib.I64x2(proj.stride(0), proj.stride(1))
    args.A = A.data_ptr()
    args.y = y.data_ptr()
    args.states = states.data_ptr()
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
    with torch.cuda.device(dev):
        _lib.check(lib.m3ssd_fwd_proj(ctypes_ref(args), _stream_ptr(dev)))
    _check_device_status(ws, "forward (in_proj form)")
    return y, states


@ssd_proj_fwd.register_fake
def _(proj, A, H, D, N, chunk, flags):
    lib = _lib.load()
    prob = _problem(proj, H, D, N, chunk, flags)
    nbytes = int(lib.m3ssd_states_bytes(ctypes_ref(prob)))
    Bsz, T, _ = proj.shape
    return (torch.empty((Bsz, T, H, D), dtype=_y_dtype(flags), device=proj.device),
            torch.empty(nbytes, dtype=torch.uint8, device=proj.device))


@torch.library.custom_op("m3ssd::ssd_proj_bwd", mutates_args=(), device_types="cuda")
def ssd_proj_bwd(dy: torch.Tensor, proj: torch.Tensor, A: torch.Tensor, states: torch.Tensor,
                 H: int, D: int, N: int, chunk: int,
                 flags: int) -> tuple[torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    dev = proj.device
    A = A.contiguous()
    if dy.dtype != _y_dtype(flags):
        dy = dy.to(_y_dtype(flags))
    prob = _problem(proj, H, D, N, chunk, flags)
    dproj = torch.empty(proj.shape, dtype=torch.float32, device=dev)
    dA = torch.empty(A.shape, dtype=torch.complex64, device=dev)
    ws_bytes = int(lib.m3ssd_bwd_workspace_bytes(ctypes_ref(prob)))
    ws = _workspace(dev, ws_bytes)
    args = _lib.ProjBwdArgs()
    args.prob = prob
    args.proj, args.proj_strides = proj.data_ptr(), _lib.I64x2(proj.stride(0), proj.stride(1))
    args.A = A.data_ptr()
    args.dy, args.dy_strides = dy.data_ptr(), _lib.I64x4(*dy.stride())
    args.states = states.data_ptr()
    args.dproj = dproj.data_ptr()
    args.dproj_strides = _lib.I64x2(dproj.stride(0), dproj.stride(1))
    args.dA = dA.data_ptr()
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
    with torch.cuda.device(dev):
        _lib.check(lib.m3ssd_bwd_proj(ctypes_ref(args), _stream_ptr(dev)))
    _check_device_status(ws, "backward (in_proj form)")
    return dproj, dA


@ssd_proj_bwd.register_fake
def _(dy, proj, A, states, H, D, N, chunk, flags):
    return (torch.empty(proj.shape, dtype=torch.float32, device=proj.device),
            torch.empty(A.shape, dtype=torch.complex64, device=proj.device))


def _setup_context(ctx, inputs, output):
    proj, A, H, D, N, chunk, flags = inputs
    _, states = output
    ctx.save_for_backward(proj, A, states)
    ctx.dims = (H, D, N, chunk, flags)
    ctx.mark_non_differentiable(states)
    ctx.set_materialize_grads(False)


def _backward(ctx, dy, _dstates):
    proj, A, states = ctx.saved_tensors
    H, D, N, chunk, flags = ctx.dims
    if dy is None:
        Bsz, T, _ = proj.shape
        dy = torch.zeros((Bsz, T, H, D), dtype=_y_dtype(flags), device=proj.device)
    dproj, dA = ssd_proj_bwd(dy, proj, A, states, H, D, N, chunk, flags)
    return dproj, dA, None, None, None, None, None


ssd_proj_fwd.register_autograd(_backward, setup_context=_setup_context)


def ssd_from_proj(proj: torch.Tensor, A: torch.Tensor, n_heads: int, head_dim: int,
                  state_dim: int, chunk_size: int = 64, precision: str = "auto",
                  y_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """y (B, T, H, D) from the block's in_proj output (see the module docstring); float32, or
    bfloat16 stored by the kernels themselves with ``y_dtype=torch.bfloat16`` (as
    ``ssd_complex_chunkwise``)."""
    if not isinstance(proj, torch.Tensor) or not isinstance(A, torch.Tensor):
        raise TypeError("proj and A must be torch.Tensor")
    if proj.device.type != "cuda" or A.device.type != "cuda":
        raise RuntimeError("m3ssd: the operator runs only on CUDA (sm_100a) and has no CPU "
                           "fallback")
    if proj.dim() != 3:
        raise ValueError(f"proj must be (B, T, H(D+4N+1)), got shape {tuple(proj.shape)}")
    H, D, N = int(n_heads), int(head_dim), int(state_dim)
    if proj.shape[-1] != proj_width(H, D, N):
        raise ValueError(f"proj has {proj.shape[-1]} columns; H={H}, D={D}, N={N} need "
                         f"{proj_width(H, D, N)}")
    if A.dtype != torch.complex64 or tuple(A.shape) != (H,):
        raise TypeError(f"A must be complex64 of shape ({H},)")
    if precision not in _PREC:
        raise ValueError(f"precision must be one of {sorted(_PREC)}, got {precision!r}")
    if not (1 <= int(chunk_size) <= 256):
        raise ValueError(f"chunk_size {chunk_size} exceeds the supported range [1, 256]")
    if proj.dtype in (torch.bfloat16, torch.float16):
        proj = proj.float()  # the block's .float() on every slice, done once
    elif proj.dtype != torch.float32:
        raise TypeError(f"proj must be float32, bfloat16 or float16, got {proj.dtype}")
    if y_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"y_dtype must be torch.float32 or torch.bfloat16, got {y_dtype}")
    if not fusable(proj, H, D, N, precision):
        return ssd_complex_chunkwise(*_interleave(proj, A, H, D, N), chunk_size=chunk_size,
                                     precision=precision, y_dtype=y_dtype)
    flags = _PREC[precision] | (_lib.M3SSD_Y_BF16 if y_dtype == torch.bfloat16 else 0)
    with torch.autocast("cuda", enabled=False):
        y, _ = ssd_proj_fwd(proj, A, H, D, N, int(chunk_size), int(flags))
    return y


def _interleave(proj, A, H, D, N):
    x_ssm, B_t, C_t, dt = unpack_proj(proj, H, D, N)
    return x_ssm, A, B_t, C_t, dt

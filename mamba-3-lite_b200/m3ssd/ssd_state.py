"""The operator over one segment of a longer sequence: an initial state in, the final state out.

``ssd_complex_chunkwise_state(x, A, B_t, C_t, dt, initial_state=None, chunk_size=64)`` returns
``(y, final_state)``. ``y`` is what ``ssd_complex_chunkwise`` returns when the reference's
recurrence (models/ssd_complex.py:17-33)

    s_t = exp(softplus(dt_t) A) s_{t-1} + B_t x_t^T,   y_t = Re(sum_n C_t,n s_t,n)

starts from ``s_{-1} = initial_state`` instead of zero; ``final_state`` is ``s_{T-1}``. Both
states are (B, H, N, D) complex64, ``s[n, :]`` for every (b, h). A sequence cut into segments,
each call fed the previous call's final state, gives the y of one call over the whole sequence;
the backward chains the same way, and autograd carries gradients through both states
(PyTorch's convention for complex tensors, as everywhere in this package).

The reference's operator always starts from zero and drops its state, so this has no counterpart
there; it is what a caller needs to run sequences longer than one call's memory, or a stream of
segments, through the same kernels. It runs on the tensor-core kernels only (through
m3ssd_fwd_state / m3ssd_bwd_state): head_dim = state_dim = 64, float32 x, B_t / C_t with a
contiguous state dimension and 16-byte aligned strides, and T a multiple of 64. Anything else
raises ValueError.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib
from .ssd_complex import (_bf16_store_ok, _check_device_status, _check_inputs, _PREC, _problem,
                          _stream_ptr, _strides, _workspace, _y_dtype)

ctypes_ref = ctypes.byref

STATE_CHUNK = 64  # sequence blocking of the tensor-core kernels; T must be a multiple of it


def _state_shape(x, B_t):
    Bsz, _, H, D = x.shape
    return (Bsz, H, B_t.shape[-1], D)


def _fill_common(args, x, A, B_t, C_t, dt, prob):
    args.prob = prob
    args.x, args.x_strides = x.data_ptr(), _lib.I64x4(*_strides(x, 4))
    args.A = A.data_ptr()
    args.B, args.b_strides = B_t.data_ptr(), _lib.I64x4(*_strides(B_t, 4))
    args.C, args.c_strides = C_t.data_ptr(), _lib.I64x4(*_strides(C_t, 4))
    args.dt, args.dt_strides = dt.data_ptr(), _lib.I64x3(*_strides(dt, 3))


@torch.library.custom_op("m3ssd::ssd_state_fwd", mutates_args=(), device_types="cuda")
def ssd_state_fwd(x: torch.Tensor, A: torch.Tensor, B_t: torch.Tensor, C_t: torch.Tensor,
                  dt: torch.Tensor, h0: Optional[torch.Tensor], chunk: int,
                  flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    dev = x.device
    A = A.contiguous()
    prob = _problem(x, B_t, chunk, flags)
    _lib.check(lib.m3ssd_check_problem(ctypes_ref(prob)))
    y = torch.empty(x.shape, dtype=_y_dtype(flags), device=dev)
    states = torch.empty(int(lib.m3ssd_states_bytes(ctypes_ref(prob))), dtype=torch.uint8,
                         device=dev)
    hT = torch.empty(_state_shape(x, B_t), dtype=torch.complex64, device=dev)
    ws_bytes = int(lib.m3ssd_fwd_workspace_bytes(ctypes_ref(prob)))
    ws = _workspace(dev, ws_bytes)
    args = _lib.FwdArgs()
    _fill_common(args, x, A, B_t, C_t, dt, prob)
    args.y = y.data_ptr()
    args.states = states.data_ptr()
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
    h0_ptr = None if h0 is None else h0.contiguous().data_ptr()
    with torch.cuda.device(dev):
        _lib.check(lib.m3ssd_fwd_state(ctypes_ref(args), h0_ptr, hT.data_ptr(), _stream_ptr(dev)))
    _check_device_status(ws, "forward (state carry)")
    return y, states, hT


@ssd_state_fwd.register_fake
def _(x, A, B_t, C_t, dt, h0, chunk, flags):
    lib = _lib.load()
    prob = _problem(x, B_t, chunk, flags)
    nbytes = int(lib.m3ssd_states_bytes(ctypes_ref(prob)))
    return (torch.empty(x.shape, dtype=_y_dtype(flags), device=x.device),
            torch.empty(nbytes, dtype=torch.uint8, device=x.device),
            torch.empty(_state_shape(x, B_t), dtype=torch.complex64, device=x.device))


@torch.library.custom_op("m3ssd::ssd_state_bwd", mutates_args=(), device_types="cuda")
def ssd_state_bwd(dy: torch.Tensor, x: torch.Tensor, A: torch.Tensor, B_t: torch.Tensor,
                  C_t: torch.Tensor, dt: torch.Tensor, states: torch.Tensor, hT: torch.Tensor,
                  dhT: Optional[torch.Tensor], chunk: int,
                  flags: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                       torch.Tensor, torch.Tensor]:
    lib = _lib.load()
    dev = x.device
    A = A.contiguous()
    if dy.dtype != _y_dtype(flags):
        dy = dy.to(_y_dtype(flags))
    prob = _problem(x, B_t, chunk, flags)
    dx = torch.empty(x.shape, dtype=x.dtype, device=dev)
    dA = torch.empty(A.shape, dtype=torch.complex64, device=dev)
    dB = torch.empty(B_t.shape, dtype=torch.complex64, device=dev)
    dC = torch.empty(C_t.shape, dtype=torch.complex64, device=dev)
    ddt = torch.empty(dt.shape, dtype=torch.float32, device=dev)
    dh0 = torch.empty(_state_shape(x, B_t), dtype=torch.complex64, device=dev)
    ws_bytes = int(lib.m3ssd_bwd_workspace_bytes(ctypes_ref(prob)))
    ws = _workspace(dev, ws_bytes)
    args = _lib.BwdArgs()
    _fill_common(args, x, A, B_t, C_t, dt, prob)
    args.dy, args.dy_strides = dy.data_ptr(), _lib.I64x4(*_strides(dy, 4))
    args.states = states.data_ptr()
    args.dx, args.dA, args.dB, args.dC, args.ddt = (dx.data_ptr(), dA.data_ptr(), dB.data_ptr(),
                                                    dC.data_ptr(), ddt.data_ptr())
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws_bytes
    if dhT is None:
        hT_ptr = dhT_ptr = None
    else:
        dhT = dhT.to(torch.complex64).contiguous()
        hT_ptr, dhT_ptr = hT.contiguous().data_ptr(), dhT.data_ptr()
    with torch.cuda.device(dev):
        _lib.check(lib.m3ssd_bwd_state(ctypes_ref(args), hT_ptr, dhT_ptr, dh0.data_ptr(),
                                       _stream_ptr(dev)))
    _check_device_status(ws, "backward (state carry)")
    return dx, dA, dB, dC, ddt, dh0


@ssd_state_bwd.register_fake
def _(dy, x, A, B_t, C_t, dt, states, hT, dhT, chunk, flags):
    return (torch.empty(x.shape, dtype=x.dtype, device=x.device),
            torch.empty(A.shape, dtype=torch.complex64, device=x.device),
            torch.empty(B_t.shape, dtype=torch.complex64, device=x.device),
            torch.empty(C_t.shape, dtype=torch.complex64, device=x.device),
            torch.empty(dt.shape, dtype=torch.float32, device=x.device),
            torch.empty(_state_shape(x, B_t), dtype=torch.complex64, device=x.device))


def _setup_context(ctx, inputs, output):
    x, A, B_t, C_t, dt, h0, chunk, flags = inputs
    _, states, hT = output
    ctx.save_for_backward(x, A, B_t, C_t, dt, states, hT)
    ctx.chunk = chunk
    ctx.flags = flags
    ctx.has_h0 = h0 is not None
    ctx.mark_non_differentiable(states)
    ctx.set_materialize_grads(False)


def _backward(ctx, dy, _dstates, dhT):
    x, A, B_t, C_t, dt, states, hT = ctx.saved_tensors
    if dy is None:
        dy = torch.zeros(x.shape, dtype=_y_dtype(ctx.flags), device=x.device)
    dx, dA, dB, dC, ddt, dh0 = ssd_state_bwd(dy, x, A, B_t, C_t, dt, states, hT, dhT, ctx.chunk,
                                             ctx.flags)
    return dx, dA, dB, dC, ddt, (dh0 if ctx.has_h0 else None), None, None


ssd_state_fwd.register_autograd(_backward, setup_context=_setup_context)


def ssd_complex_chunkwise_state(x: torch.Tensor, A: torch.Tensor, B_t: torch.Tensor,
                                C_t: torch.Tensor, dt: torch.Tensor,
                                initial_state: Optional[torch.Tensor] = None,
                                chunk_size: int = 64, precision: str = "auto",
                                y_dtype: torch.dtype = torch.float32):
    """(y, final_state) of the recurrence started from ``initial_state`` (see the module
    docstring). ``chunk_size``, ``precision`` and ``y_dtype`` mean what they mean for
    ``ssd_complex_chunkwise``; ``precision="fp32"`` is not available with a state carry."""
    _check_inputs(x, A, B_t, C_t, dt, chunk_size)
    if precision not in _PREC:
        raise ValueError(f"precision must be one of {sorted(_PREC)}, got {precision!r}")
    if y_dtype not in (torch.float32, torch.bfloat16):
        raise TypeError(f"y_dtype must be torch.float32 or torch.bfloat16, got {y_dtype}")
    flags = _PREC[precision] | (_lib.M3SSD_X_COMPLEX if x.dtype == torch.complex64 else 0)
    Bsz, T, H, D = x.shape
    if not _bf16_store_ok(x, B_t, C_t, flags):
        raise ValueError("the state carry runs on the tensor-core kernels only: head_dim = "
                         "state_dim = 64, float32 x, precision 'auto' or 'tensor', B_t / C_t with "
                         "a contiguous state dimension and 16-byte aligned strides")
    if T % STATE_CHUNK:
        raise ValueError(f"the state carry needs T a multiple of {STATE_CHUNK}, got T = {T}")
    if initial_state is not None:
        shape = _state_shape(x, B_t)
        if tuple(initial_state.shape) != shape:
            raise ValueError(f"initial_state must be (B, H, N, D) = {shape}, got "
                             f"{tuple(initial_state.shape)}")
        if initial_state.dtype != torch.complex64:
            raise TypeError(f"initial_state must be complex64, got {initial_state.dtype}")
        if initial_state.device != x.device:
            raise RuntimeError("initial_state is on another device than x")
    if y_dtype == torch.bfloat16:
        flags |= _lib.M3SSD_Y_BF16
    with torch.autocast("cuda", enabled=False):
        y, _, hT = ssd_state_fwd(x, A, B_t, C_t, dt, initial_state, int(chunk_size), int(flags))
    return y, hT

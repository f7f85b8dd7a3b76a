"""The forward entry point that allocates nothing (m3ssd_fwd_static_scratch).

It exists for callers that cannot allocate device memory when they call the operator, for
example a serving runtime that plans all device memory up front and forbids allocation on the
request path. Its scratch is a fixed device array inside libm3ssd.so. Here it is called through
the C ABI twice in a row on different inputs, so the second call must clear what the first left
in the shared array, and each result is compared with the regular m3ssd_fwd on the same inputs.
The device status word it copies to the caller's 4-byte buffer must read 0 after each call. At a
shape m3ssd_fwd runs as chains (few long sequences) the static entry still runs one pass: its y
and states must match, and the regular backward must give the same gradients from either states.
This file is collected last so that a run stopping at the first failure has run everything else.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import cases
from tolerances import TOL

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(cuda_device):
    from m3ssd import _lib
    return _lib.load()


def _inputs(dev, seed, B=3, T=1000, H=5):
    inp = cases.block_inputs(seed, B, T, H, 64, 64)
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in inp.items()}


def _args(t, y, states, ws):
    from m3ssd import _lib
    x = t["x"]
    Bsz, T, H, D = x.shape
    a = _lib.FwdArgs()
    a.prob = _lib.Problem(Bsz, T, H, D, t["B_t"].shape[-1], 64, 0, 0)
    a.x, a.x_strides = x.data_ptr(), _lib.I64x4(*x.stride())
    a.A = t["A"].data_ptr()
    a.B, a.b_strides = t["B_t"].data_ptr(), _lib.I64x4(*t["B_t"].stride())
    a.C, a.c_strides = t["C_t"].data_ptr(), _lib.I64x4(*t["C_t"].stride())
    a.dt, a.dt_strides = t["dt"].data_ptr(), _lib.I64x3(*t["dt"].stride())
    a.y, a.states = y.data_ptr(), states.data_ptr()
    a.workspace = ws.data_ptr() if ws is not None else None
    a.workspace_bytes = ws.numel() if ws is not None else 0
    return a


def _run(lib, t, static):
    """One forward through the C ABI; returns y, states (as float32) and the status word (the
    static entry copies it to a 4-byte caller buffer, m3ssd_fwd leaves it in its workspace)."""
    dev = t["x"].device
    a0 = _args(t, t["x"], t["x"], None)
    nstates = lib.m3ssd_states_bytes(ctypes.byref(a0.prob))
    y = torch.full(t["x"].shape, float("nan"), device=dev)
    states = torch.empty(nstates, dtype=torch.uint8, device=dev)
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    if static:
        status = torch.full((1,), -1, dtype=torch.int32, device=dev)
        a = _args(t, y, states, None)
        a.workspace, a.workspace_bytes = status.data_ptr(), 4
        rc = lib.m3ssd_fwd_static_scratch(ctypes.byref(a), stream)
    else:
        ws = torch.empty(lib.m3ssd_fwd_workspace_bytes(ctypes.byref(a0.prob)), dtype=torch.uint8,
                         device=dev)
        rc = lib.m3ssd_fwd(ctypes.byref(_args(t, y, states, ws)), stream)
        status = ws[:4].view(torch.int32)
    assert rc == 0, lib.m3ssd_strerror(rc).decode()
    torch.cuda.synchronize(dev)
    return y, states, int(status.item())


def _bwd(lib, t, states, dy):
    """The regular backward through the C ABI from a given forward's states."""
    from m3ssd import _lib
    dev = t["x"].device
    x = t["x"]
    Bsz, T, H, D = x.shape
    a = _lib.BwdArgs()
    a.prob = _lib.Problem(Bsz, T, H, D, t["B_t"].shape[-1], 64, 0, 0)
    a.x, a.x_strides = x.data_ptr(), _lib.I64x4(*x.stride())
    a.A = t["A"].data_ptr()
    a.B, a.b_strides = t["B_t"].data_ptr(), _lib.I64x4(*t["B_t"].stride())
    a.C, a.c_strides = t["C_t"].data_ptr(), _lib.I64x4(*t["C_t"].stride())
    a.dt, a.dt_strides = t["dt"].data_ptr(), _lib.I64x3(*t["dt"].stride())
    a.dy, a.dy_strides = dy.data_ptr(), _lib.I64x4(*dy.stride())
    a.states = states.data_ptr()
    g = {"dx": torch.empty_like(x), "dA": torch.empty_like(t["A"]),
         "dB": torch.empty_like(t["B_t"]), "dC": torch.empty_like(t["C_t"]),
         "ddt": torch.empty_like(t["dt"])}
    a.dx, a.dA, a.dB, a.dC, a.ddt = (g[k].data_ptr() for k in ("dx", "dA", "dB", "dC", "ddt"))
    ws = torch.empty(lib.m3ssd_bwd_workspace_bytes(ctypes.byref(a.prob)), dtype=torch.uint8,
                     device=dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    rc = lib.m3ssd_bwd(ctypes.byref(a), stream)
    assert rc == 0, lib.m3ssd_strerror(rc).decode()
    torch.cuda.synchronize(dev)
    assert int(ws[:4].view(torch.int32).item()) == 0
    return g


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max()).item()


def test_static_scratch_forward_matches_regular_forward_twice(lib, cuda_device):
    tol = TOL["tensor"]["y_normwise"]
    for seed in (1, 2):  # two calls in a row through the same static scratch
        t = _inputs(cuda_device, seed)
        y_s, st_s, status_s = _run(lib, t, static=True)
        y_r, st_r, status_r = _run(lib, t, static=False)
        assert status_s == 0 and status_r == 0
        assert torch.isfinite(y_s).all()
        assert _rel(y_s, y_r) < tol
        assert _rel(st_s.view(torch.float32), st_r.view(torch.float32)) < tol


def test_static_scratch_at_a_chained_shape(lib, cuda_device):
    """B1 T4096 H2: m3ssd_fwd runs each sequence as chains, the static entry in one pass."""
    from m3ssd import _lib
    prob = _lib.Problem(1, 4096, 2, 64, 64, 64, 0, 0)
    assert lib.m3ssd_launch_count(ctypes.byref(prob), 0) > 2  # the regular forward chains here
    tol, gtol = TOL["tensor"]["y_normwise"], TOL["tensor"]["g_normwise"]
    t = _inputs(cuda_device, 4, B=1, T=4096, H=2)
    dy = torch.from_numpy(cases.upstream_grad(4, 1, 4096, 2, 64)).to(cuda_device)
    y_s, st_s, status_s = _run(lib, t, static=True)
    y_r, st_r, status_r = _run(lib, t, static=False)
    assert status_s == 0 and status_r == 0
    assert _rel(y_s, y_r) < tol
    assert _rel(st_s.view(torch.float32), st_r.view(torch.float32)) < tol
    g_s = _bwd(lib, t, st_s, dy)
    g_r = _bwd(lib, t, st_r, dy)
    for k in g_r:
        a, b = torch.view_as_real(g_s[k]) if g_s[k].is_complex() else g_s[k], \
            torch.view_as_real(g_r[k]) if g_r[k].is_complex() else g_r[k]
        assert _rel(a, b) < gtol, k


def test_static_scratch_limits(lib, cuda_device):
    from m3ssd import _lib
    t = _inputs(cuda_device, 3, B=1, T=64, H=1)
    # more chunks than the fixed scratch holds: rejected before any device work
    a = _args(t, t["x"], t["x"], None)
    a.prob = _lib.Problem(1, 64 * 40000, 1, 64, 64, 64, 0, 0)
    assert lib.m3ssd_fwd_static_scratch(ctypes.byref(a), None) == 11
    assert "32768" in lib.m3ssd_strerror(11).decode()
    # shapes without the tensor-core forward are rejected
    a.prob = _lib.Problem(1, 64, 1, 32, 64, 64, 0, 0)
    assert lib.m3ssd_fwd_static_scratch(ctypes.byref(a), None) == 2

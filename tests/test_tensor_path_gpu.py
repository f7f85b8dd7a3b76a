"""GPU checks of the tcgen05 (split-bf16) path against the reference algorithm in complex128 on
the same GPU and against the fp32 CUDA-core path. Every call runs with M3SSD_CHECK=1, so a
bounded wait that expired inside a kernel fails the test."""
import numpy as np
import pytest
import torch

from oracle import cases
from oracle.ssd_torch_cpu import ssd_chunkwise_torch
from tolerances import TOL

pytestmark = pytest.mark.gpu
KEYS = ("x", "A", "B_t", "C_t", "dt")
GRAD_KEYS = ("dx", "dA", "dB", "dC", "ddt")


@pytest.fixture(autouse=True)
def _device_status_checks(monkeypatch):
    monkeypatch.setenv("M3SSD_CHECK", "1")


@pytest.fixture(scope="module")
def m3(cuda_device):
    import m3ssd
    m3ssd.load()
    return m3ssd


def _inputs(dev, B, T, H, seed=0, dt_mode="raw", slow=False, complex_x=False):
    inp = cases.block_inputs(seed, B, T, H, 64, 64, dt_mode=dt_mode, slow_decay=slow,
                             complex_x=complex_x)
    dy = cases.upstream_grad(seed, B, T, H, 64)
    t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in inp.items()}
    return t, torch.from_numpy(dy).to(dev)


def _f64(t):
    return {k: (v.to(torch.complex128) if v.is_complex() else v.double()) for k, v in t.items()}


def _up(a):
    return a.to(torch.complex128) if a.is_complex() else a.double()


def _rel(a, b):
    a, b = _up(a), _up(b)
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-300)).item()


def _floored(a, b, floor=1e-3):
    a, b = _up(a), _up(b)
    den = torch.maximum(b.abs(), floor * b.abs().max())
    return ((a - b).abs() / den).max().item()


def test_path_selection(m3):
    assert m3.implementation((16, 2048, 16, 64), 64)[0] == "tcgen05-bf16x2"
    assert m3.implementation((16, 2048, 16, 64), 64, precision="fp32")[0] == "simt-fp32"
    assert m3.implementation((2, 64, 2, 32), 64)[0] == "simt-fp32"
    # complex x: two passes of the real-x tensor-core kernels; fp32 precision stays on CUDA cores
    assert m3.implementation((2, 64, 2, 64), 64, complex_x=True)[0] == "tcgen05-bf16x2"
    assert m3.implementation((2, 64, 2, 64), 64, complex_x=True, precision="fp32")[0] == "simt-fp32"


@pytest.mark.parametrize("B,T,H,dt_mode,slow", [
    (1, 64, 1, "raw", False), (1, 1, 1, "raw", False), (1, 130, 2, "raw", False),
    (2, 256, 4, "literal", False), (3, 1000, 5, "raw", True), (16, 2048, 16, "raw", False),
    (16, 2048, 16, "literal", False), (1, 16384, 4, "raw", True),
])
def test_forward_vs_fp64(m3, cuda_device, B, T, H, dt_mode, slow):
    tol = TOL["tensor"]
    t, _ = _inputs(cuda_device, B, T, H, dt_mode=dt_mode, slow=slow)
    y = m3.ssd_complex_chunkwise(*(t[k] for k in KEYS), chunk_size=64, precision="tensor")
    with torch.no_grad():
        y64 = ssd_chunkwise_torch(*(_f64(t)[k] for k in KEYS), chunk_size=64,
                                  cdtype=torch.complex128)
    assert torch.isfinite(y).all()
    e, f = _rel(y, y64), _floored(y, y64)
    print(f"B{B} T{T} H{H} {dt_mode} slow={slow}: normwise {e:.2e} floored {f:.2e}")
    assert e < tol["y_normwise"]
    assert f < tol["y_floored"]


def test_tensor_matches_fp32_path(m3, cuda_device):
    t, _ = _inputs(cuda_device, 4, 777, 6, seed=3)
    args = [t[k] for k in KEYS]
    y_tc = m3.ssd_complex_chunkwise(*args, chunk_size=64, precision="tensor")
    y_fp = m3.ssd_complex_chunkwise(*args, chunk_size=64, precision="fp32")
    assert _rel(y_tc, y_fp) < 5e-5


def test_user_chunk_size_does_not_change_result(m3, cuda_device):
    t, _ = _inputs(cuda_device, 2, 300, 3, seed=4)
    args = [t[k] for k in KEYS]
    y64 = m3.ssd_complex_chunkwise(*args, chunk_size=64)
    for c in (16, 128, 256):
        assert torch.equal(m3.ssd_complex_chunkwise(*args, chunk_size=c), y64)


def test_strided_x_scalar_loads(m3, cuda_device):
    t, _ = _inputs(cuda_device, 2, 200, 3, seed=5)
    big = torch.zeros(2, 200, 3, 128, device=cuda_device)
    big[..., ::2] = t["x"]
    xs = big[..., ::2]
    assert xs.stride(-1) == 2
    y_s = m3.ssd_complex_chunkwise(xs, t["A"], t["B_t"], t["C_t"], t["dt"])
    y_c = m3.ssd_complex_chunkwise(t["x"], t["A"], t["B_t"], t["C_t"], t["dt"])
    assert torch.equal(y_s, y_c)


def test_states_handoff_many_sequences(m3, cuda_device):
    """More sequences than SMs and many chunks: every chunk waits for its predecessor's state."""
    t, _ = _inputs(cuda_device, 40, 640, 8, seed=6)
    args = [t[k] for k in KEYS]
    y_tc = m3.ssd_complex_chunkwise(*args, precision="tensor")
    y_fp = m3.ssd_complex_chunkwise(*args, precision="fp32")
    assert _rel(y_tc, y_fp) < 5e-5


@pytest.mark.parametrize("B,T,H,dt_mode,slow", [
    (1, 64, 1, "raw", False), (2, 300, 3, "raw", False), (2, 256, 4, "literal", False),
    (3, 1000, 5, "raw", True), (16, 2048, 16, "raw", False), (1, 16384, 4, "raw", True),
])
def test_grads_vs_fp64(m3, cuda_device, B, T, H, dt_mode, slow):
    tol = TOL["tensor"]
    assert m3.implementation((B, T, H, 64), 64)[1] == "tcgen05-bf16x2"
    t, dy = _inputs(cuda_device, B, T, H, seed=7, dt_mode=dt_mode, slow=slow)
    xs = [t[k].clone().requires_grad_(True) for k in KEYS]
    y = m3.ssd_complex_chunkwise(*xs, precision="tensor")
    (y * dy).sum().backward()
    x64 = [_f64(t)[k].clone().requires_grad_(True) for k in KEYS]
    y64 = ssd_chunkwise_torch(*x64, chunk_size=64, cdtype=torch.complex128)
    (y64 * dy.double()).sum().backward()
    for k, a, b in zip(GRAD_KEYS, xs, x64):
        assert torch.isfinite(a.grad).all(), k
        e = _rel(a.grad, b.grad)
        print(f"B{B} T{T} H{H} {dt_mode} slow={slow} {k}: normwise {e:.2e}")
        assert e < tol["g_normwise"], (k, e)


def test_grads_tensor_vs_fp32_many_sequences(m3, cuda_device):
    t, dy = _inputs(cuda_device, 40, 640, 8, seed=9)

    def grads(prec):
        xs = [t[k].clone().requires_grad_(True) for k in KEYS]
        y = m3.ssd_complex_chunkwise(*xs, precision=prec)
        (y * dy).sum().backward()
        return [v.grad for v in xs]

    for k, a, b in zip(GRAD_KEYS, grads("tensor"), grads("fp32")):
        assert _rel(a, b) < 1e-4, k


def test_backward_deterministic(m3, cuda_device):
    t, dy = _inputs(cuda_device, 8, 512, 8, seed=10)

    def grads():
        xs = [t[k].clone().requires_grad_(True) for k in KEYS]
        y = m3.ssd_complex_chunkwise(*xs)
        (y * dy).sum().backward()
        return [v.grad for v in xs]

    g1, g2 = grads(), grads()
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_deterministic(m3, cuda_device):
    t, _ = _inputs(cuda_device, 8, 512, 8, seed=8)
    args = [t[k] for k in KEYS]
    ys = [m3.ssd_complex_chunkwise(*args) for _ in range(3)]
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[0], ys[2])


# ---- complex x: y = F(xr; C) + F(xi; i C) through the real-x kernels, dx = dxr + i dxi

@pytest.mark.parametrize("B,T,H,dt_mode,slow", [
    (1, 64, 1, "raw", False), (2, 300, 3, "raw", False), (2, 256, 4, "literal", False),
    (3, 1000, 5, "raw", True), (4, 2048, 16, "raw", False),
])
def test_complex_x_vs_fp64(m3, cuda_device, B, T, H, dt_mode, slow):
    """Forward and all six gradients (dx complex) against the reference algorithm in complex128,
    at the tensor-core tolerances."""
    tol = TOL["tensor"]
    t, dy = _inputs(cuda_device, B, T, H, seed=11, dt_mode=dt_mode, slow=slow, complex_x=True)
    assert t["x"].dtype == torch.complex64
    assert m3.implementation((B, T, H, 64), 64, complex_x=True) == ("tcgen05-bf16x2",) * 2
    xs = [t[k].clone().requires_grad_(True) for k in KEYS]
    y = m3.ssd_complex_chunkwise(*xs, precision="tensor")
    (y * dy).sum().backward()
    x64 = [_f64(t)[k].clone().requires_grad_(True) for k in KEYS]
    y64 = ssd_chunkwise_torch(*x64, chunk_size=64, cdtype=torch.complex128)
    (y64 * dy.double()).sum().backward()
    assert torch.isfinite(y).all()
    e, f = _rel(y, y64), _floored(y, y64)
    print(f"complex x B{B} T{T} H{H} {dt_mode} slow={slow} y: normwise {e:.2e} floored {f:.2e}")
    assert e < tol["y_normwise"] and f < tol["y_floored"]
    for k, a, b in zip(GRAD_KEYS, xs, x64):
        assert torch.isfinite(torch.view_as_real(a.grad) if a.grad.is_complex() else a.grad).all()
        assert a.grad.dtype == (torch.complex64 if k in ("dx", "dA", "dB", "dC") else torch.float32)
        e = _rel(a.grad, b.grad)
        print(f"complex x B{B} T{T} H{H} {k}: normwise {e:.2e}")
        assert e < tol["g_normwise"], (k, e)


def test_complex_x_tensor_matches_fp32_path(m3, cuda_device):
    """The two tensor-core passes against the CUDA-core complex-x path on the same inputs."""
    t, dy = _inputs(cuda_device, 4, 777, 6, seed=12, complex_x=True)

    def run(prec):
        xs = [t[k].clone().requires_grad_(True) for k in KEYS]
        y = m3.ssd_complex_chunkwise(*xs, precision=prec)
        (y * dy).sum().backward()
        return [y.detach()] + [v.grad for v in xs]

    for k, a, b in zip(("y",) + GRAD_KEYS, run("tensor"), run("fp32")):
        assert _rel(a, b) < (5e-5 if k == "y" else 1e-4), k


def test_complex_x_real_part_only_equals_real_x(m3, cuda_device):
    """A complex x with zero imaginary part gives the real-x result for y and every gradient."""
    t, dy = _inputs(cuda_device, 2, 500, 3, seed=13)

    def run(x):
        xs = [x.clone().requires_grad_(True)] + [t[k].clone().requires_grad_(True)
                                                 for k in KEYS[1:]]
        y = m3.ssd_complex_chunkwise(*xs)
        (y * dy).sum().backward()
        return [y.detach()] + [v.grad for v in xs]

    got = run(t["x"].to(torch.complex64))
    ref = run(t["x"])
    assert _rel(got[0], ref[0]) < 1e-6
    assert _rel(got[1].real, ref[1]) < 1e-6  # dx real part
    for a, b in zip(got[2:], ref[2:]):
        assert _rel(a, b) < 1e-5


def test_chained_ragged_bf16_dy_vs_fp64(m3, cuda_device):
    """B2 L4090 H4 runs as chains with a ragged last chunk; with y in bf16 the backward's carry pass
    reads dy as bf16 through its plain-load kernel. Gradients against the complex128 reference fed
    the same (bf16-valued) upstream gradient."""
    B, T, H = 2, 4090, 4
    from m3ssd import _lib
    import ctypes
    prob = _lib.Problem(B, T, H, 64, 64, 64, _lib.M3SSD_Y_BF16, 0)
    assert _lib.load().m3ssd_launch_count(ctypes.byref(prob), 1) > 2  # chained backward
    tol = TOL["tensor"]
    t, dy = _inputs(cuda_device, B, T, H, seed=14, slow=True)
    dy16 = dy.to(torch.bfloat16)
    xs = [t[k].clone().requires_grad_(True) for k in KEYS]
    y = m3.ssd_complex_chunkwise(*xs, y_dtype=torch.bfloat16)
    assert y.dtype == torch.bfloat16
    y.backward(dy16)
    x64 = [_f64(t)[k].clone().requires_grad_(True) for k in KEYS]
    y64 = ssd_chunkwise_torch(*x64, chunk_size=64, cdtype=torch.complex128)
    (y64 * dy16.double()).sum().backward()
    for k, a, b in zip(GRAD_KEYS, xs, x64):
        e = _rel(a.grad, b.grad)
        print(f"chained ragged bf16 dy {k}: normwise {e:.2e}")
        assert e < tol["g_normwise"], (k, e)


def test_sequence_alone_equals_its_slice_of_a_large_batch(m3, cuda_device):
    """Sequences are independent, so the first sequence of a batch of 32 (128 sequences: the
    kernels' default order) and the same sequence alone (4 sequences: the order for few chains,
    the forward's state first and the backward's carry first) get the same y, dx, dB, dC and ddt,
    bit for bit (dA sums over the batch)."""
    t, dy = _inputs(cuda_device, 32, 256, 4, seed=21)

    def run(sl):
        xs = [t[k][sl].detach().clone().requires_grad_(True) if k != "A" else
              t[k].detach().clone().requires_grad_(True) for k in KEYS]
        y = m3.ssd_complex_chunkwise(*xs, chunk_size=64)
        y.backward(dy[sl])
        return [y.detach()] + [xs[i].grad for i in (0, 2, 3, 4)]

    full = run(slice(0, 32))
    one = run(slice(0, 1))
    for name, a, b in zip(("y", "dx", "dB", "dC", "ddt"), one, full):
        assert torch.equal(a, b[0:1]), name

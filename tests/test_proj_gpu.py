"""GPU checks of the in_proj form (m3ssd_fwd_proj / m3ssd_bwd_proj through ``ssd_from_proj``).

* Fused vs the block's composition (slices, torch.complex, then the operator): the same kernels on
  the same operand values, so y, d(proj) and dA must be BIT-identical.
* Fused vs the reference block's own outputs (fixture proj_block, made by the reference) at the
  tensor-path tolerances, wherever the reference is finite.
* Fused vs the fp64 evaluation of the reference algorithm at the block shape.
Every call runs with M3SSD_CHECK=1 (a bounded wait that expired fails the test).
"""
import os

import numpy as np
import pytest
import torch

from oracle import block_proj, cases
from oracle.ssd_torch_cpu import ssd_chunkwise_torch
from tolerances import TOL

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(autouse=True)
def _device_status_checks(monkeypatch):
    monkeypatch.setenv("M3SSD_CHECK", "1")


@pytest.fixture(scope="module")
def m3(cuda_device):
    import m3ssd
    m3ssd.load()
    return m3ssd


def _case(dev, B, T, H, seed=0, dt_mode="raw"):
    proj, A = cases.proj_inputs(seed, B, T, H, 64, 64, dt_mode=dt_mode)
    dy = cases.upstream_grad(seed, B, T, H, 64)
    return (torch.from_numpy(proj).to(dev), torch.from_numpy(A).to(dev),
            torch.from_numpy(dy).to(dev))


def _fused(m3, proj, A, dy, H, chunk=64, clone=True):
    # (clone() of a projection with gaps between rows would compact it)
    p = (proj.detach().clone() if clone else proj.detach()).requires_grad_(True)
    a = A.detach().clone().requires_grad_(True)
    y = m3.ssd_from_proj(p, a, H, 64, 64, chunk_size=chunk)
    y.backward(dy)
    return y.detach(), p.grad, a.grad


def _composed(m3, proj, A, dy, H, chunk=64):
    """The block's own path: unpack by slices and torch.complex, then the operator."""
    p = proj.detach().clone().requires_grad_(True)
    a = A.detach().clone().requires_grad_(True)
    x, Bt, Ct, dt = m3.unpack_proj(p, H, 64, 64)
    y = m3.ssd_complex_chunkwise(x, a, Bt, Ct, dt, chunk_size=chunk)
    y.backward(dy)
    return y.detach(), p.grad, a.grad


@pytest.mark.parametrize("B,T,H,chunk", [
    (2, 2048, 16, 64),   # block shape, two sequences per head
    (3, 200, 4, 64),     # T not a multiple of the chunk
    (1, 64, 4, 128),     # chunk 128 (the kernels block at 64; the result does not depend on it)
    (2, 1000, 8, 64),
    (1, 4096, 2, 64),    # few long sequences: both directions run as chains (planar C in the carry pass)
    (8, 256, 16, 64),    # 128 sequences: the default kernel order (fewer run the latency-bound variants)
])
def test_fused_equals_composition_bitwise(m3, cuda_device, B, T, H, chunk):
    proj, A, dy = _case(cuda_device, B, T, H, seed=B * 1000 + T)
    yf, gpf, gaf = _fused(m3, proj, A, dy, H, chunk)
    yc, gpc, gac = _composed(m3, proj, A, dy, H, chunk)
    assert torch.equal(yf, yc)
    assert torch.equal(gpf, gpc)
    assert torch.equal(gaf, gac)


def test_fused_strided_projection(m3, cuda_device):
    """proj as a column slice of a wider buffer (row stride > width) and the reverse order of
    batch and time in memory."""
    B, T, H = 2, 300, 4
    proj, A, dy = _case(cuda_device, B, T, H, seed=5)
    W = proj.shape[-1]
    wide = torch.randn(B, T, W + 60, device=cuda_device)
    wide[..., 20:20 + W] = proj
    view = wide[..., 20:20 + W]          # offset 80 bytes: 16-byte aligned
    tmaj = proj.transpose(0, 1).contiguous().transpose(0, 1)  # time-major storage
    yc, gpc, gac = _composed(m3, proj, A, dy, H)
    for p in (view, tmaj):
        assert m3.ssd_proj.fusable(p, H, 64, 64)
        yf, gpf, gaf = _fused(m3, p, A, dy, H, clone=False)
        assert torch.equal(yf, yc) and torch.equal(gpf, gpc) and torch.equal(gaf, gac)


def test_fallback_composition_for_other_shapes(m3, cuda_device):
    """head_dim 32: not a tensor-core shape, so ssd_from_proj runs the composition (fp32 path)."""
    B, T, H, D, N = 1, 100, 2, 32, 16
    proj_np, A_np = cases.proj_inputs(7, B, T, H, D, N)
    proj = torch.from_numpy(proj_np).to(cuda_device).requires_grad_(True)
    A = torch.from_numpy(A_np).to(cuda_device)
    assert not m3.ssd_proj.fusable(proj, H, D, N)
    y = m3.ssd_from_proj(proj, A, H, D, N, chunk_size=16)
    y_ref = block_proj.ssd_from_proj(proj_np, A_np, H, D, N, 16)
    assert np.abs(y.detach().cpu().numpy() - y_ref).max() / np.abs(y_ref).max() < 2e-5
    y.sum().backward()
    assert proj.grad.shape == proj.shape and torch.isfinite(proj.grad).all()


def test_bf16_projection(m3, cuda_device):
    """A bf16 projection (the block under autocast) is upcast once, like the block's .float()."""
    B, T, H = 1, 256, 4
    proj, A, dy = _case(cuda_device, B, T, H, seed=9)
    p16 = proj.to(torch.bfloat16)
    yf, gpf, gaf = _fused(m3, p16, A, dy, H)
    yc, gpc, gac = _composed(m3, p16, A, dy, H)
    assert gpf.dtype == torch.bfloat16 and torch.equal(yf, yc) and torch.equal(gpf, gpc)


def test_fused_matches_reference_block_fixture(m3, cuda_device):
    """proj_block: the reference block's own y, d(proj) and dA at sampled entries (finite ones)."""
    g = dict(np.load(os.path.join(GOLDEN, "proj_block.npz")))
    proj_np, A_np, dy_np, chunk, (H, D, N) = cases.make_proj_case("proj_block")
    proj = torch.from_numpy(proj_np).to(cuda_device)
    A = torch.from_numpy(A_np).to(cuda_device)
    dy = torch.from_numpy(dy_np).to(cuda_device)
    y, gp, ga = _fused(m3, proj, A, dy, H, chunk)
    tol = TOL["tensor"]
    for got, key, bar in ((y, "y", tol["y_normwise"]), (gp, "dproj", tol["g_normwise"]),
                          (ga, "dA", tol["g_normwise"])):
        ref = g[key]
        v = got.detach().cpu().numpy().reshape(-1)[g["idx_" + key]]
        m = np.isfinite(ref)
        assert m.mean() > 0.5
        err = np.abs(v[m] - ref[m]).max() / np.abs(ref[m]).max()
        assert err < bar, (key, err)


# B4 L2048 H16 runs in one pass; B2 L4090 H4 as chains with a ragged last chunk (the backward's
# carry pass then reads planar C with its plain-load kernel)
@pytest.mark.parametrize("B,T,H", [(4, 2048, 16), (2, 4090, 4)])
def test_fused_against_fp64_block_shape(m3, cuda_device, B, T, H):
    """y, d(proj) and dA against the reference algorithm in complex128 on the GPU."""
    proj, A, dy = _case(cuda_device, B, T, H, seed=11)
    y, gp, ga = _fused(m3, proj, A, dy, H)
    p64 = proj.double().requires_grad_(True)
    a64 = A.to(torch.complex128).requires_grad_(True)
    hd, hn = H * 64, H * 64  # the block's column blocks (models/mamba_block.py:74-84), in fp64
    x = p64[..., :hd].reshape(B, T, H, 64)
    Bt = torch.complex(p64[..., hd:hd + hn], p64[..., hd + hn:hd + 2 * hn]).reshape(B, T, H, 64)
    Ct = torch.complex(p64[..., hd + 2 * hn:hd + 3 * hn],
                       p64[..., hd + 3 * hn:hd + 4 * hn]).reshape(B, T, H, 64)
    dt = p64[..., -H:]
    y64 = ssd_chunkwise_torch(x, a64, Bt, Ct, dt, chunk_size=64, cdtype=torch.complex128)
    (y64 * dy.double()).sum().backward()
    tol = TOL["tensor"]

    def rel(a, b):
        return ((a.to(b.dtype) - b).abs().max() / b.abs().max()).item()

    assert rel(y, y64.detach()) < tol["y_normwise"]
    assert rel(gp, p64.grad) < tol["g_normwise"]
    assert rel(ga, a64.grad) < tol["g_normwise"]


# T = 4096 and 4090 (8 sequences of 64 chunks) run as chains: the carry pass reads dy as bf16 (and,
# fused, C as planar tiles) with the plain-load carry kernel, 4090 with a ragged last chunk
@pytest.mark.parametrize("T,fused", [(2048, True), (200, True), (200, False), (4096, True),
                                     (4090, True), (4090, False)])
def test_bf16_readout(m3, cuda_device, T, fused):
    """y_dtype=bfloat16: the kernels round y in their store and read dy as bf16. y is bit-equal to
    the fp32 result rounded, and the gradients equal those of the fp32 path fed the same (bf16)
    upstream gradient."""
    B, H = 2, 4
    proj, A, dy = _case(cuda_device, B, T, H, seed=T)
    dy16 = dy.to(torch.bfloat16)

    def run(y_dtype, g):
        p = proj.detach().clone().requires_grad_(True)
        a = A.detach().clone().requires_grad_(True)
        if fused:
            y = m3.ssd_from_proj(p, a, H, 64, 64, y_dtype=y_dtype)
            grads = lambda: (p.grad, a.grad)  # noqa: E731
        else:
            x, Bt, Ct, dt = m3.unpack_proj(p, H, 64, 64)
            y = m3.ssd_complex_chunkwise(x, a, Bt, Ct, dt, y_dtype=y_dtype)
            grads = lambda: (p.grad, a.grad)  # noqa: E731
        y.backward(g)
        return (y.detach(),) + grads()

    y16, gp16, ga16 = run(torch.bfloat16, dy16)
    y32, gp32, ga32 = run(torch.float32, dy16.float())
    assert y16.dtype == torch.bfloat16
    assert torch.equal(y16, y32.to(torch.bfloat16))
    assert torch.equal(gp16, gp32) and torch.equal(ga16, ga32)

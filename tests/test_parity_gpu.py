"""GPU parity of the CUDA operator against the reference's own outputs (golden fixtures), the
fp64 recurrence (oracle) and, at full block size, the torch restatement on the same GPU.

All calls go through the public drop-in, which calls libm3ssd.so through the C ABI.
"""
import os

import numpy as np
import pytest
import torch

from oracle import cases, metrics
from oracle import ssd_oracle as O
from oracle.ssd_torch_cpu import ssd_chunkwise_torch
from tolerances import TOL

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
PRECISIONS = ["fp32", "tensor"]
GRAD_KEYS = ("dx", "dA", "dB", "dC", "ddt")


@pytest.fixture(scope="module")
def m3(cuda_device):
    import m3ssd
    m3ssd.load()
    return m3ssd


def to_dev(inp, dev):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in inp.items()}


def run_op(m3, inp, dy, chunk, precision, dev, grads=True):
    t = to_dev(inp, dev)
    xs = [t[k].clone().requires_grad_(grads) for k in ("x", "A", "B_t", "C_t", "dt")]
    y = m3.ssd_complex_chunkwise(*xs, chunk_size=chunk, precision=precision)
    out = {"y": y.detach().cpu().numpy()}
    if grads:
        (y * torch.from_numpy(dy).to(dev)).sum().backward()
        for k, v in zip(GRAD_KEYS, xs):
            out[k] = v.grad.detach().cpu().numpy()
    return out


def pick(g, name, key, a):
    a = np.asarray(a)
    if name in cases.SAMPLED_CASES:
        return a.reshape(-1)[g["idx_" + key]]
    return a


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("name", list(cases.CASES))
def test_forward_and_grads_vs_reference_and_oracle(m3, cuda_device, name, precision):
    tol = TOL[precision]
    inp, dy, chunk = cases.make_case(name)
    g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    got = run_op(m3, inp, dy, chunk, precision, cuda_device)
    assert got["y"].dtype == np.float32 and got["y"].shape == inp["x"].shape
    assert np.isfinite(got["y"]).all()
    # vs the reference's own output where it is finite
    ref = g["y"]
    fin = np.isfinite(ref)
    if fin.any():
        assert metrics.normwise(pick(g, name, "y", got["y"]), ref, fin) < tol["y_normwise"]
    # vs the exact recurrence everywhere
    yn = O.ssd_naive(**inp).real
    assert metrics.normwise(got["y"], yn) < tol["y_normwise"]
    assert metrics.floored(got["y"], yn) < tol["y_floored"]
    # gradients vs the reference's autograd (where finite) and vs the fp64 adjoint
    ng = dict(zip(GRAD_KEYS, O.ssd_naive_grads(**inp, dy=dy)))
    for k in GRAD_KEYS:
        assert got[k].dtype == np.asarray(g[k]).dtype, k
        assert np.isfinite(got[k]).all(), k
        r = g[k]
        f = np.isfinite(r)
        if f.any():
            assert metrics.normwise(pick(g, name, k, got[k]), r, f) < tol["g_normwise"], k
        assert metrics.normwise(got[k], ng[k]) < tol["g_normwise"], k


@pytest.mark.parametrize("name", ["ref_dt0", "ref_tv_dt"])
def test_reference_test_criterion(m3, cuda_device, name):
    """The reference tests' own check (tests/test_ssd.py:17-22, :38-40): float32 output of shape
    (B, T, H, D), allclose to the complex64 naive recurrence at atol 1e-4."""
    inp, dy, chunk = cases.make_case(name)
    got = run_op(m3, inp, dy, chunk, "fp32", cuda_device, grads=False)
    yn = O.ssd_naive(**inp, dtype=np.complex64).real
    assert got["y"].dtype == np.float32 and got["y"].shape == inp["x"].shape
    np.testing.assert_allclose(got["y"], yn, atol=1e-4, rtol=0)


@pytest.mark.parametrize("name", ["ref_T20", "ref_T_eq_C", "pad_T18_C4"])
def test_reference_shape_checks(m3, cuda_device, name):
    """tests/test_ssd.py:43-66: T a multiple of C, T == C and (here) a padded T keep the shape and
    stay finite."""
    inp, dy, chunk = cases.make_case(name)
    got = run_op(m3, inp, dy, chunk, "fp32", cuda_device, grads=False)
    assert got["y"].shape == inp["x"].shape
    assert np.isfinite(got["y"]).all()


def _block_tensors(dev, B, T, H, D, N, seed=0, dt_mode="raw", slow=False, complex_x=False):
    inp = cases.block_inputs(seed, B, T, H, D, N, dt_mode=dt_mode, slow_decay=slow,
                             complex_x=complex_x)
    dy = cases.upstream_grad(seed, B, T, H, D)
    return to_dev(inp, dev), torch.from_numpy(dy).to(dev)


def _grads(fn, t, dy, **kw):
    xs = [t[k].clone().requires_grad_(True) for k in ("x", "A", "B_t", "C_t", "dt")]
    y = fn(*xs, **kw)
    (y * dy).sum().backward()
    return y.detach(), [v.grad.detach() for v in xs]


def _rel(a, b):
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


def _f64(t):
    return {k: (v.to(torch.complex128) if v.is_complex() else v.double()) for k, v in t.items()}


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape,chunk,dt_mode,slow", [
    ((16, 2048, 16, 64, 64), 64, "raw", False),       # block shape, raw dt
    ((16, 2048, 16, 64, 64), 64, "literal", False),   # block shape, literal softplus(dt)
    ((1, 16384, 4, 64, 64), 128, "raw", True),        # long sequence, slow decay, chunk 128
    ((1, 16384, 4, 64, 64), 64, "raw", True),
])
def test_full_size_vs_fp64_restatement_on_gpu(m3, cuda_device, shape, chunk, dt_mode, slow,
                                              precision):
    """Full-size parity against the reference algorithm (masked before exp) evaluated in
    complex128 on the same GPU; the fp32 restatement's own error is checked to be no smaller
    than ours by more than the tolerance."""
    tol = TOL[precision]
    t, dy = _block_tensors(cuda_device, *shape, dt_mode=dt_mode, slow=slow)
    y, g = _grads(m3.ssd_complex_chunkwise, t, dy, chunk_size=chunk, precision=precision)
    y64, g64 = _grads(ssd_chunkwise_torch, _f64(t), dy.double(), chunk_size=chunk,
                      cdtype=torch.complex128)
    y32, g32 = _grads(ssd_chunkwise_torch, t, dy, chunk_size=chunk)
    assert torch.isfinite(y).all()
    e_ours, e_ref = _rel(y.double(), y64), _rel(y32.double(), y64)
    print(f"y normwise vs fp64: ours {e_ours:.2e}, fp32 reference algorithm {e_ref:.2e}")
    assert e_ours < tol["y_normwise"]
    for k, a, b, c in zip(GRAD_KEYS, g, g64, g32):
        assert torch.isfinite(a).all(), k
        ea = _rel(a.to(b.dtype), b)
        print(f"{k} normwise vs fp64: ours {ea:.2e}, fp32 reference algorithm "
              f"{_rel(c.to(b.dtype), b):.2e}")
        assert ea < tol["g_normwise"], (k, ea)


def test_chunk_size_invariance(m3, cuda_device):
    """The result is the same function of the inputs for every chunk length."""
    t, dy = _block_tensors(cuda_device, 2, 500, 4, 64, 64, seed=3)
    base, gb = _grads(m3.ssd_complex_chunkwise, t, dy, chunk_size=64, precision="fp32")
    for c in (1, 7, 16, 32, 100, 128, 256):
        y, g = _grads(m3.ssd_complex_chunkwise, t, dy, chunk_size=c, precision="fp32")
        assert _rel(y, base) < 2e-5, c
        for a, b in zip(g, gb):
            assert _rel(a, b) < 1e-4, c


def test_causality_and_prefix(m3, cuda_device):
    t, _ = _block_tensors(cuda_device, 2, 300, 3, 32, 16, seed=4)
    y = m3.ssd_complex_chunkwise(*(t[k] for k in ("x", "A", "B_t", "C_t", "dt")), chunk_size=64)
    t2 = dict(t)
    x2 = t["x"].clone()
    x2[:, 150:] += 1.0
    t2["x"] = x2
    y2 = m3.ssd_complex_chunkwise(*(t2[k] for k in ("x", "A", "B_t", "C_t", "dt")), chunk_size=64)
    assert torch.equal(y[:, :150], y2[:, :150])
    assert not torch.equal(y[:, 150:], y2[:, 150:])
    tp = {k: (v[:, :137] if v.dim() > 1 else v) for k, v in t.items()}
    yp = m3.ssd_complex_chunkwise(*(tp[k] for k in ("x", "A", "B_t", "C_t", "dt")), chunk_size=64)
    torch.testing.assert_close(yp, y[:, :137], rtol=0, atol=1e-6)


def test_linearity_in_x(m3, cuda_device):
    t, _ = _block_tensors(cuda_device, 2, 256, 4, 64, 64, seed=5)
    args = lambda xx: (xx, t["A"], t["B_t"], t["C_t"], t["dt"])
    x1 = t["x"]
    x2 = torch.randn_like(x1)
    y12 = m3.ssd_complex_chunkwise(*args(x1 + 2 * x2))
    y1 = m3.ssd_complex_chunkwise(*args(x1))
    y2 = m3.ssd_complex_chunkwise(*args(x2))
    assert _rel(y12, y1 + 2 * y2) < 1e-5


def test_strided_inputs_match_contiguous(m3, cuda_device):
    """Views into one projection buffer, as the block passes them (models/mamba_block.py:73-84)."""
    B, T, H, D, N = 2, 130, 4, 16, 8
    g = torch.Generator(device=cuda_device).manual_seed(0)
    in_dim = H * (D + 4 * N + 1)
    proj = torch.randn(B, T, in_dim, device=cuda_device, generator=g)
    x = proj[..., :H * D].reshape(B, T, H, D)
    Bt = torch.complex(proj[..., H * D:H * D + H * N], proj[..., H * D + H * N:H * D + 2 * H * N]
                       ).reshape(B, T, H, N) * 0.3
    Ct = torch.complex(proj[..., H * D + 2 * H * N:H * D + 3 * H * N],
                       proj[..., H * D + 3 * H * N:H * D + 4 * H * N]).reshape(B, T, H, N) * 0.3
    dt = (proj - 3.0)[..., -H:]
    A = torch.complex(-torch.rand(H, device=cuda_device) - 0.5, torch.randn(H, device=cuda_device))
    assert not x.is_contiguous() and not dt.is_contiguous()
    Bs = Bt[:, :, :, ::2]  # strided complex view as well
    Cs = Ct[:, :, :, ::2]
    y_s = m3.ssd_complex_chunkwise(x, A, Bs, Cs, dt, chunk_size=32)
    y_c = m3.ssd_complex_chunkwise(x.contiguous(), A, Bs.contiguous(), Cs.contiguous(),
                                   dt.contiguous(), chunk_size=32)
    assert torch.equal(y_s, y_c)


def test_deterministic(m3, cuda_device):
    t, dy = _block_tensors(cuda_device, 2, 256, 4, 64, 64, seed=6)
    y1, g1 = _grads(m3.ssd_complex_chunkwise, t, dy)
    y2, g2 = _grads(m3.ssd_complex_chunkwise, t, dy)
    assert torch.equal(y1, y2)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


@pytest.mark.parametrize("shape,chunk", [
    ((1, 1, 1, 1, 1), 1), ((1, 1, 2, 3, 5), 64), ((1, 5, 1, 2, 2), 8), ((3, 33, 2, 40, 24), 16),
    ((1, 300, 1, 64, 64), 256), ((2, 64, 3, 256, 8), 64), ((1, 40, 2, 8, 256), 32),
])
def test_edge_shapes_vs_oracle(m3, cuda_device, shape, chunk):
    B, T, H, D, N = shape
    inp = cases.ref_style_inputs(9, B, T, H, D, N, dt_scale=0.5, complex_x=False)
    dy = cases.upstream_grad(9, B, T, H, D)
    got = run_op(m3, inp, dy, chunk, "fp32", cuda_device)
    yn = O.ssd_naive(**inp).real
    assert metrics.normwise(got["y"], yn) < 2e-5
    for k, ref in zip(GRAD_KEYS, O.ssd_naive_grads(**inp, dy=dy)):
        assert metrics.normwise(got[k], ref) < 1e-4, k


def test_input_validation(m3, cuda_device):
    dev = cuda_device
    x = torch.randn(1, 8, 2, 4, device=dev)
    A = torch.randn(2, dtype=torch.complex64, device=dev)
    B = torch.randn(1, 8, 2, 4, dtype=torch.complex64, device=dev)
    dt = torch.randn(1, 8, 2, device=dev)
    f = m3.ssd_complex_chunkwise
    with pytest.raises(TypeError):
        f(x.double(), A, B, B, dt, chunk_size=4)
    with pytest.raises(TypeError):
        f(x, A, B.to(torch.complex128), B, dt, chunk_size=4)
    with pytest.raises(ValueError, match="exceeds"):
        f(x, A, B, B, dt, chunk_size=512)
    with pytest.raises(ValueError, match="exceeds"):
        f(x, A, B, B, dt, chunk_size=0)
    with pytest.raises(ValueError):
        f(x, A[:1], B, B, dt, chunk_size=4)
    with pytest.raises(ValueError):
        f(x, A, B[:, :4], B, dt, chunk_size=4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        f(x.cpu(), A, B, B, dt, chunk_size=4)


def test_autograd_plumbing_checkpoint_and_compile(m3, cuda_device):
    """None-safe backward, non-reentrant checkpoint re-execution (models/mamba_block.py:57-61) and
    torch.compile(fullgraph=False) (training/pretrain.py:216-220) all run the custom op."""
    t, dy = _block_tensors(cuda_device, 1, 96, 2, 16, 8, seed=8)
    xs = [t[k].clone().requires_grad_(True) for k in ("x", "A", "B_t", "C_t", "dt")]

    def fn(*a):
        return m3.ssd_complex_chunkwise(*a, chunk_size=32) * 2.0

    y_ref, g_ref = _grads(fn, t, dy)
    y = torch.utils.checkpoint.checkpoint(fn, *xs, use_reentrant=False)
    (y * dy).sum().backward()
    for v, r in zip(xs, g_ref):
        torch.testing.assert_close(v.grad, r, rtol=0, atol=0)
    cfn = torch.compile(fn, fullgraph=False)
    y_c, g_c = _grads(cfn, t, dy)
    torch.testing.assert_close(y_c, y_ref, rtol=0, atol=0)
    for a, b in zip(g_c, g_ref):
        torch.testing.assert_close(a, b, rtol=1e-6, atol=1e-6)
    # a loss that ignores y still backpropagates zeros through the op
    xs2 = [t[k].clone().requires_grad_(True) for k in ("x", "A", "B_t", "C_t", "dt")]
    y2 = m3.ssd_complex_chunkwise(*xs2, chunk_size=32)
    (y2.sum() * 0.0).backward()
    assert all(v.grad is not None and torch.count_nonzero(v.grad) == 0 for v in xs2)


@pytest.mark.parametrize("precision", PRECISIONS)
def test_plain_per_element_error_vs_reference(m3, cuda_device, precision):
    """The plain per-element relative error |got - ref| / |ref| of y (no floor), against the
    reference's own output and against the exact recurrence, beside the reference's own plain
    error against the exact recurrence, over every golden case whose reference output is finite
    (the block-shape cases on their stored sample of entries). The fp32 path must be no less
    accurate than the reference algorithm itself on that measure. The split-bf16 tensor path is
    reported only: its relative error near y = 0 has no bound of that form (it is held to the
    floored per-element bar and the normwise bars in the other tests)."""
    rows = []
    for name in cases.CASES:
        inp, dy, chunk = cases.make_case(name)
        g = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
        ref = np.asarray(g["y"], dtype=np.float64)
        if not np.isfinite(ref).all():
            continue
        got = run_op(m3, inp, dy, chunk, precision, cuda_device, grads=False)["y"]
        got = pick(g, name, "y", got).astype(np.float64)
        exact = pick(g, name, "y", O.ssd_naive(**inp).real)
        nz = (ref != 0) & (exact != 0)
        plain = lambda a, b: float(np.max(np.abs(a[nz] - b[nz]) / np.abs(b[nz])))
        rows.append((name, plain(got, ref), plain(got, exact), plain(ref, exact)))
    assert rows
    print(f"\n{precision}: case, plain rel. error vs reference, vs exact, reference vs exact")
    for r in rows:
        print(f"  {r[0]:14s} {r[1]:.2e} {r[2]:.2e} {r[3]:.2e}")
    worst_ours = max(r[2] for r in rows)
    worst_ref = max(r[3] for r in rows)
    if precision == "fp32":
        assert worst_ours <= worst_ref

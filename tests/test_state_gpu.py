"""GPU checks of the state carry (m3ssd_fwd_state / m3ssd_bwd_state through
ssd_complex_chunkwise_state): the fp64 recurrence with an initial state and a final-state
gradient (oracle), segment chaining against one call over the whole sequence, and the zero-state
case against the plain operator. Every call runs with M3SSD_CHECK=1."""
import numpy as np
import pytest
import torch

from oracle import cases, metrics
from oracle import ssd_oracle as O
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


def _case(B, T, H, seed):
    inp = cases.block_inputs(seed, B, T, H, 64, 64, dt_mode="raw")
    dy = cases.upstream_grad(seed, B, T, H, 64)
    rng = np.random.default_rng(seed + 1000)
    shape = (B, H, 64, 64)
    h0 = (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(np.complex64)
    dhT = (0.1 * (rng.standard_normal(shape) + 1j * rng.standard_normal(shape))).astype(np.complex64)
    return inp, dy, h0, dhT


def _dev(a, dev, grad=False):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev).requires_grad_(grad)


def _state_loss(hT, dhT):
    """Re(sum conj(dhT) hT): its gradient with respect to hT is dhT."""
    return (torch.view_as_real(hT) * torch.view_as_real(dhT)).sum()


def _chained(B, T, H):
    """Whether the library runs this shape as several chains per sequence (two passes)."""
    import ctypes
    from m3ssd import _lib
    p = _lib.Problem(B, T, H, 64, 64, 64, 0, 0)
    lib = _lib.load()
    return (lib.m3ssd_launch_count(ctypes.byref(p), 0) > 2,
            lib.m3ssd_launch_count(ctypes.byref(p), 1) > 2)


# (2, 64, 3): first and last chunk in one ticket; (1, 1024, 2): few long sequences, run as chains
@pytest.mark.parametrize("B,T,H", [(2, 64, 3), (2, 256, 3), (1, 1024, 2)])
def test_state_carry_vs_fp64_recurrence(m3, cuda_device, B, T, H):
    tol = TOL["tensor"]
    assert _chained(B, T, H) == ((True, True) if T == 1024 else (False, False))
    inp, dy, h0, dhT = _case(B, T, H, seed=T)
    xs = [_dev(inp[k], cuda_device, True) for k in KEYS]
    h0_t = _dev(h0, cuda_device, True)
    y, hT = m3.ssd_complex_chunkwise_state(*xs, initial_state=h0_t)
    assert hT.shape == (B, H, 64, 64) and hT.dtype == torch.complex64
    loss = (y * _dev(dy, cuda_device)).sum() + _state_loss(hT, _dev(dhT, cuda_device))
    loss.backward()

    yn, sn = O.ssd_naive(**inp, s0=h0, return_state=True)
    got_y = y.detach().cpu().numpy()
    assert metrics.normwise(got_y, yn.real) < tol["y_normwise"]
    assert metrics.floored(got_y, yn.real) < tol["y_floored"]
    got_h = hT.detach().cpu().numpy()
    assert metrics.normwise(got_h, sn) < tol["y_normwise"]

    ref = O.ssd_naive_grads(**inp, dy=dy, s0=h0, dsT=dhT)
    for k, v, r in zip(GRAD_KEYS, xs, ref[:5]):
        g = v.grad.detach().cpu().numpy()
        assert np.isfinite(g).all(), k
        assert metrics.normwise(g, r) < tol["g_normwise"], k
    g0 = h0_t.grad.detach().cpu().numpy()
    assert metrics.normwise(g0, ref[5]) < tol["g_normwise"]


def test_segments_chain_like_one_call(m3, cuda_device):
    """A sequence of 512 cut at 192 and 320: y, the final state and every gradient of the chained
    calls match one call over the whole sequence (the forward bit for bit: the carried state is
    the same fp32 tile either way)."""
    inp, dy, _, dhT = _case(2, 512, 3, seed=7)
    dy_t, dhT_t = _dev(dy, cuda_device), _dev(dhT, cuda_device)
    full = [_dev(inp[k], cuda_device, True) for k in KEYS]
    y_full, h_full = m3.ssd_complex_chunkwise_state(*full)
    ((y_full * dy_t).sum() + _state_loss(h_full, dhT_t)).backward()

    cuts = [(0, 192), (192, 320), (320, 512)]
    segs, ys, h = [], [], None
    for a, b in cuts:
        seg = [_dev(inp[k][:, a:b] if k != "A" else inp[k], cuda_device, True) for k in KEYS]
        y, h = m3.ssd_complex_chunkwise_state(*seg, initial_state=h)
        segs.append(seg)
        ys.append(y)
    loss = sum((y * dy_t[:, a:b]).sum() for y, (a, b) in zip(ys, cuts)) + _state_loss(h, dhT_t)
    loss.backward()

    assert torch.equal(torch.cat(ys, dim=1), y_full)
    assert torch.equal(h, h_full)
    for i, k in enumerate(GRAD_KEYS):
        want = full[i].grad
        if k == "dA":
            got = sum(s[1].grad for s in segs)
        else:
            got = torch.cat([s[i].grad for s in segs], dim=1)
        rel = ((got - want).abs().max() / want.abs().max()).item()
        assert rel < 1e-5, (k, rel)


@pytest.mark.parametrize("B,T,H", [(2, 256, 2), (1, 2048, 2)])
def test_zero_state_is_the_plain_operator(m3, cuda_device, B, T, H):
    """No initial state and no final-state gradient: the same kernels and results as
    ssd_complex_chunkwise, bit for bit (one pass, and as chains); an explicit zero initial state
    gives the same y."""
    inp, dy, _, _ = _case(B, T, H, seed=3)
    dy_t = _dev(dy, cuda_device)
    a = [_dev(inp[k], cuda_device, True) for k in KEYS]
    b = [_dev(inp[k], cuda_device, True) for k in KEYS]
    y_plain = m3.ssd_complex_chunkwise(*a)
    (y_plain * dy_t).sum().backward()
    y_state, hT = m3.ssd_complex_chunkwise_state(*b)
    (y_state * dy_t).sum().backward()
    assert torch.equal(y_plain, y_state)
    for k, u, v in zip(GRAD_KEYS, a, b):
        assert torch.equal(u.grad, v.grad), k
    z = torch.zeros(hT.shape, dtype=torch.complex64, device=cuda_device)
    y_zero, h_zero = m3.ssd_complex_chunkwise_state(*[t.detach() for t in b], initial_state=z)
    assert torch.equal(y_zero, y_plain)
    assert torch.equal(h_zero, hT)


def test_state_carry_rejects_what_it_cannot_take(m3, cuda_device):
    inp, _, h0, _ = _case(1, 128, 2, seed=1)
    xs = [_dev(inp[k], cuda_device) for k in KEYS]
    with pytest.raises(ValueError, match="multiple of 64"):
        m3.ssd_complex_chunkwise_state(*[t[:, :100] if t.dim() > 1 else t for t in xs])
    with pytest.raises(ValueError, match="initial_state"):
        m3.ssd_complex_chunkwise_state(*xs, initial_state=_dev(h0[:, :, :32], cuda_device))
    with pytest.raises(ValueError, match="tensor-core"):
        m3.ssd_complex_chunkwise_state(*xs, precision="fp32")

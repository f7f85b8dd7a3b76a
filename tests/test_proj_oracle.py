"""CPU checks of the in_proj form (the block's SSD input path, models/mamba_block.py:73-88).

The fixtures proj_*.npz were made by the reference block itself (tests/golden/make_golden.py,
``run_reference_block``): its own slicing / torch.complex unpacking of a given projection, the
reference operator on the unpacked tensors, and torch.autograd back to the projection.
"""
import os

import numpy as np
import torch

from oracle import block_proj, cases
from oracle.ssd_oracle import ssd_naive_grads
from oracle.ssd_torch_cpu import ssd_chunkwise_torch

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


def _rel(a, b):
    a, b = np.asarray(a), np.asarray(b)
    m = np.isfinite(b)
    return float(np.abs(a[m] - b[m]).max() / np.abs(b[m]).max())


def test_fixture_inputs_regenerate():
    for name in cases.PROJ_CASES:
        g = _load(name)
        proj, A, dy, chunk, dims = cases.make_proj_case(name)
        assert np.allclose(g["sum_proj"][0], np.abs(proj).astype(np.float64).sum(), rtol=1e-12)
        assert np.allclose(g["sum_dy"][0], np.abs(dy).astype(np.float64).sum(), rtol=1e-12)
        assert int(g["chunk"]) == chunk and tuple(g["dims"]) == dims


def test_unpack_matches_reference_block():
    """oracle.block_proj.unpack_proj is bit-identical to the block's own unpacking."""
    g = _load("proj_small")
    H, D, N = (int(v) for v in g["dims"])
    x, Bt, Ct, dt = block_proj.unpack_proj(g["in_proj"], H, D, N)
    for got, key in ((x, "x"), (Bt, "B_t"), (Ct, "C_t"), (dt, "dt")):
        ref = g["unpacked_" + key]
        assert got.shape == ref.shape and got.dtype == ref.dtype
        np.testing.assert_array_equal(got, ref)


def test_package_unpack_matches_reference_block():
    """The package's torch unpacking (the fallback composition) equals the block's, on CPU."""
    import m3ssd.ssd_proj as sp
    g = _load("proj_small")
    H, D, N = (int(v) for v in g["dims"])
    out = sp.unpack_proj(torch.from_numpy(g["in_proj"]), H, D, N)
    for got, key in zip(out, ("x", "B_t", "C_t", "dt")):
        np.testing.assert_array_equal(got.numpy(), g["unpacked_" + key])
    assert sp.proj_width(H, D, N) == g["in_proj"].shape[-1]


def test_projection_gradient_assembly():
    """pack_proj_grad of the operator's gradients equals the block's autograd d(proj): exactly for
    gradients taken through the torch restatement (bit-identical to the reference where finite),
    and to ~1e-6 for the hand-derived fp64 adjoint."""
    g = _load("proj_small")
    H, D, N = (int(v) for v in g["dims"])
    chunk = int(g["chunk"])
    x, Bt, Ct, dt = block_proj.unpack_proj(g["in_proj"], H, D, N)
    ts = [torch.from_numpy(np.ascontiguousarray(v)).requires_grad_(True)
          for v in (x, g["in_A"], Bt, Ct, dt)]
    y = ssd_chunkwise_torch(*ts, chunk_size=chunk)
    (y * torch.from_numpy(g["in_dy"])).sum().backward()
    dx, dA, dB, dC, ddt = (t.grad.numpy() for t in ts)
    np.testing.assert_array_equal(block_proj.pack_proj_grad(dx, dB, dC, ddt, H, D, N), g["dproj"])
    np.testing.assert_array_equal(dA, g["dA"])
    gx, gA, gB, gC, gdt = ssd_naive_grads(x, g["in_A"], Bt, Ct, dt, g["in_dy"])
    assert _rel(block_proj.pack_proj_grad(gx, gB, gC, gdt, H, D, N), g["dproj"]) < 1e-5
    assert _rel(gA, g["dA"]) < 1e-5


def test_oracle_forward_small():
    g = _load("proj_small")
    H, D, N = (int(v) for v in g["dims"])
    y = block_proj.ssd_from_proj(g["in_proj"], g["in_A"], H, D, N, int(g["chunk"]))
    assert _rel(y, g["y"]) < 5e-6


def test_oracle_forward_block_shape_sampled():
    """Block shape (H4 D64 N64, T = 160 not a multiple of the chunk): the oracle's y at the
    fixture's sampled entries, wherever the reference is finite (its exp-then-mask overflow
    leaves ~25% of this strong-decay case NaN)."""
    g = _load("proj_block")
    proj, A, dy, chunk, (H, D, N) = cases.make_proj_case("proj_block")
    y = block_proj.ssd_from_proj(proj, A, H, D, N, chunk).reshape(-1)[g["idx_y"]]
    assert 0.0 < g["nonfinite_y"] < 0.5
    assert _rel(y, g["y"]) < 5e-6


def test_abi_rejects_bad_proj_arguments():
    """Argument checks of m3ssd_fwd_proj / m3ssd_bwd_proj run before any device work."""
    import ctypes
    from m3ssd import _lib
    lib = _lib.load()
    a = _lib.ProjFwdArgs()
    assert lib.m3ssd_fwd_proj(None, None) == 1                       # ERR_NULL
    a.prob = _lib.Problem(2, 100, 16, 64, 64, 64, 0, 0)
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 1            # proj NULL
    a.proj, a.A = 4096, 4096
    a.proj_strides = _lib.I64x2(100 * 5136, 5136)
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 1            # y / states NULL
    a.prob = _lib.Problem(2, 100, 16, 32, 64, 64, 0, 0)              # not a tensor-core shape
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 2
    a.prob = _lib.Problem(2, 100, 16, 64, 64, 64, _lib.M3SSD_PREC_FP32, 0)
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 2
    a.prob = _lib.Problem(2, 100, 16, 64, 64, 64, 0, 0)
    a.proj_strides = _lib.I64x2(100 * 5136, 5135)                    # time stride not 4-aligned
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 5
    a.proj_strides = _lib.I64x2(100 * 5136, 5136)
    a.proj = 4100                                                     # proj not 16-byte aligned
    assert lib.m3ssd_fwd_proj(ctypes.byref(a), None) == 5
    b = _lib.ProjBwdArgs()
    b.prob = _lib.Problem(2, 100, 16, 64, 64, 64, 0, 0)
    b.proj, b.A = 4096, 4096
    b.proj_strides = _lib.I64x2(100 * 5136, 5136)
    assert lib.m3ssd_bwd_proj(ctypes.byref(b), None) == 1            # dy, states, dproj NULL
    b.dy, b.states, b.dproj, b.dA = 4096, 4096, 4096, 4096
    b.dproj_strides = _lib.I64x2(100 * 5136, 5134)
    assert lib.m3ssd_bwd_proj(ctypes.byref(b), None) == 5            # dproj stride
    b.dproj_strides = _lib.I64x2(100 * 5136, 5136)
    assert lib.m3ssd_bwd_proj(ctypes.byref(b), None) == 6            # no workspace

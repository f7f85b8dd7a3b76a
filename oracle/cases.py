"""Seeded inputs for parity cases (test infrastructure).

Shapes and distributions:
* ``ref_*`` cases mirror the reference's own SSD tests (tests/test_ssd.py:9-14, 30-35, 45-50,
  58-63; tests/test_ssd_triton.py:322-327; tests/e2e_gpu_smoke.py:164-169): complex x,
  ``A = randn - 1``, randn B_t/C_t, dt zero or randn (scaled 0.1 where the reference scales it).
* ``block_*`` cases use the block-shape distributions: x ~ N(0,1) fp32 real,
  A = complex(-exp(U(log 1, log 16)), U(-pi, pi)) with ONE complex scalar per head (the operator's
  A is (H,), models/mamba_block.py:41), B_t/C_t re and im each N(0, 1/(2N)), and dt either raw
  N(-4, 0.5) (the operator applies softplus itself, step ~ 0.018) or the literal
  softplus(N(-4, 0.5)) (softplus applied twice, step ~ 0.70).
* ``slow_decay`` uses A_real = -exp(U(log 0.01, log 1)) (long-sequence stress distribution).

All draws use numpy's PCG64 generator so fixtures regenerate bit-for-bit on any host with the
same numpy.
"""
from __future__ import annotations

import numpy as np

from .ssd_oracle import softplus_f32


def _cn(rng, shape, scale=1.0):
    """complex64 with independent N(0, scale^2) real and imaginary parts."""
    re = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
    im = rng.standard_normal(shape, dtype=np.float32) * np.float32(scale)
    return (re + 1j * im).astype(np.complex64)


def ref_style_inputs(seed, B, T, H, D, N, dt_mode="randn", dt_scale=1.0, complex_x=True):
    """Inputs shaped like the reference's own unit tests (randn everywhere, A = randn - 1)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if complex_x:
        # torch.randn(dtype=complex64) draws each part with variance 1/2
        x = _cn(rng, (B, T, H, D), scale=np.sqrt(0.5))
    else:
        x = rng.standard_normal((B, T, H, D), dtype=np.float32)
    A = (_cn(rng, (H,), scale=np.sqrt(0.5)) - np.complex64(1.0)).astype(np.complex64)
    Bt = _cn(rng, (B, T, H, N), scale=np.sqrt(0.5))
    Ct = _cn(rng, (B, T, H, N), scale=np.sqrt(0.5))
    if dt_mode == "zero":
        dt = np.zeros((B, T, H), np.float32)
    else:
        dt = (rng.standard_normal((B, T, H), dtype=np.float32) * np.float32(dt_scale))
    return dict(x=x, A=A, B_t=Bt, C_t=Ct, dt=dt.astype(np.float32))


def block_inputs(seed, B, T, H, D, N, dt_mode="raw", slow_decay=False, complex_x=False):
    """Block-shape distributions (see module docstring)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    if complex_x:
        x = _cn(rng, (B, T, H, D), scale=np.sqrt(0.5))
    else:
        x = rng.standard_normal((B, T, H, D), dtype=np.float32)
    if slow_decay:
        a_re = -np.exp(rng.uniform(np.log(0.01), np.log(1.0), size=H))
    else:
        a_re = -np.exp(rng.uniform(np.log(1.0), np.log(16.0), size=H))
    a_im = rng.uniform(-np.pi, np.pi, size=H)
    A = (a_re + 1j * a_im).astype(np.complex64)
    s = np.sqrt(1.0 / (2 * N))
    Bt = _cn(rng, (B, T, H, N), scale=s)
    Ct = _cn(rng, (B, T, H, N), scale=s)
    z = (rng.standard_normal((B, T, H), dtype=np.float32) * np.float32(0.5) - np.float32(4.0))
    dt = softplus_f32(z) if dt_mode == "literal" else z
    return dict(x=x, A=A, B_t=Bt, C_t=Ct, dt=dt.astype(np.float32))


def upstream_grad(seed, B, T, H, D):
    rng = np.random.Generator(np.random.PCG64(seed + 7919))
    return rng.standard_normal((B, T, H, D), dtype=np.float32)


# name -> (generator kwargs, chunk size). Small enough for pure numpy/torch CPU in seconds.
CASES = {
    "ref_dt0":        (dict(kind="ref", seed=0, B=2, T=16, H=2, D=4, N=4, dt_mode="zero"), 4),
    "ref_tv_dt":      (dict(kind="ref", seed=3, B=2, T=16, H=2, D=4, N=4), 4),
    "ref_T20":        (dict(kind="ref", seed=1, B=1, T=20, H=2, D=4, N=4), 4),
    "ref_T_eq_C":     (dict(kind="ref", seed=2, B=1, T=4, H=2, D=4, N=4), 4),
    "pad_T18_C4":     (dict(kind="ref", seed=11, B=1, T=18, H=2, D=4, N=4), 4),
    "pad_T70_C16":    (dict(kind="ref", seed=12, B=2, T=70, H=3, D=8, N=8, dt_scale=0.5), 16),
    "ref_grad_c8":    (dict(kind="ref", seed=7, B=2, T=32, H=2, D=8, N=8, dt_scale=0.1), 8),
    "ref_e2e_c16":    (dict(kind="ref", seed=5, B=1, T=16, H=2, D=16, N=16, dt_scale=0.1), 16),
    "real_x_c16":     (dict(kind="ref", seed=21, B=2, T=40, H=3, D=8, N=8, dt_scale=0.5,
                            complex_x=False), 16),
    "block_small_raw":  (dict(kind="block", seed=31, B=1, T=160, H=2, D=64, N=64), 64),
    "block_small_lit":  (dict(kind="block", seed=32, B=1, T=128, H=2, D=64, N=64,
                              dt_mode="literal"), 64),
    "block_c32":        (dict(kind="block", seed=33, B=1, T=96, H=2, D=32, N=16), 32),
    "block_c128":       (dict(kind="block", seed=34, B=1, T=256, H=2, D=64, N=64,
                              slow_decay=True), 128),
    "block_cplx_x":     (dict(kind="block", seed=35, B=1, T=128, H=2, D=64, N=64,
                              complex_x=True), 64),
    # the B2 L256 H4 D64 N64 chunk-64 CPU correctness shape
    "cfg0_raw":         (dict(kind="block", seed=0, B=2, T=256, H=4, D=64, N=64), 64),
    "cfg0_literal":     (dict(kind="block", seed=0, B=2, T=256, H=4, D=64, N=64,
                              dt_mode="literal"), 64),
}

# cases whose fixtures store input checksums and sampled entries (full tensors would be megabytes)
SAMPLED_CASES = ("block_small_raw", "block_small_lit", "block_c32", "block_c128", "block_cplx_x",
                 "cfg0_raw", "cfg0_literal")


def make_case(name):
    """Return (inputs dict, dy, chunk_size) for a named case."""
    kw, chunk = CASES[name]
    kw = dict(kw)
    kind = kw.pop("kind")
    if kind == "ref":
        inp = ref_style_inputs(**kw)
    else:
        inp = block_inputs(**kw)
    Bsz, T, H, D = inp["x"].shape
    dy = upstream_grad(kw["seed"], Bsz, T, H, D)
    return inp, dy, chunk


# ------------------------------------------------------------------ in_proj form of the inputs
def proj_inputs(seed, B, T, H, D, N, dt_mode="raw"):
    """(proj, A): block-shape draws (``block_inputs``) laid out as the block's in_proj output,
    columns x | Re B | Im B | Re C | Im C | dt (models/mamba_block.py:74-84)."""
    inp = block_inputs(seed, B, T, H, D, N, dt_mode=dt_mode)
    hn = H * N
    proj = np.concatenate([
        inp["x"].reshape(B, T, H * D),
        inp["B_t"].real.reshape(B, T, hn), inp["B_t"].imag.reshape(B, T, hn),
        inp["C_t"].real.reshape(B, T, hn), inp["C_t"].imag.reshape(B, T, hn),
        inp["dt"].reshape(B, T, H)], axis=-1).astype(np.float32)
    return np.ascontiguousarray(proj), inp["A"]


# name -> (proj_inputs kwargs, chunk size)
PROJ_CASES = {
    "proj_small":  (dict(seed=41, B=2, T=20, H=2, D=8, N=8), 8),
    "proj_block":  (dict(seed=42, B=1, T=160, H=4, D=64, N=64), 64),
}
PROJ_SAMPLED = ("proj_block",)


def make_proj_case(name):
    """Return (proj, A, dy, chunk, (H, D, N)) for a named in_proj case."""
    kw, chunk = PROJ_CASES[name]
    proj, A = proj_inputs(**kw)
    H, D, N = kw["H"], kw["D"], kw["N"]
    dy = upstream_grad(kw["seed"], kw["B"], kw["T"], H, D)
    return proj, A, dy, chunk, (H, D, N)

"""numpy restatement of the block's SSD input path (test infrastructure; CPU only).

Reference: models/mamba_block.py in atandra2000/Mamba-3-Lite.

* ``proj_width``   - in_proj output width H(D + 4N + 1) (models/mamba_block.py:35).
* ``unpack_proj``  - models/mamba_block.py:73-84: x_ssm = proj[..., :HD] as (B,T,H,D);
                     B_t = Re B + i Im B from columns [HD, HD+HN) and [HD+HN, HD+2HN);
                     C_t likewise from the next 2HN columns; dt = the last H columns.
* ``pack_proj_grad`` - the adjoint of ``unpack_proj``: the gradient of the whole projection
                     from the operator's gradients, as torch.autograd assembles it through the
                     slices and torch.complex (for z = complex(a, b), dL/da = Re g and
                     dL/db = Im g with g = dL/dRe z + i dL/dIm z).
* ``ssd_from_proj`` - unpack, then ``ssd_oracle.ssd_chunkwise`` (models/ssd_complex.py:58-119).
"""
from __future__ import annotations

import numpy as np

from .ssd_oracle import ssd_chunkwise


def proj_width(H, D, N):
    return H * (D + 4 * N + 1)


def unpack_proj(proj, H, D, N):
    """(x_ssm, B_t, C_t, dt) from proj (B, T, H(D+4N+1)) float32 (models/mamba_block.py:74-84)."""
    proj = np.asarray(proj, dtype=np.float32)
    Bsz, T, W = proj.shape
    assert W == proj_width(H, D, N)
    hd, hn = H * D, H * N
    x = proj[..., :hd].reshape(Bsz, T, H, D).copy()
    Bt = (proj[..., hd:hd + hn] + 1j * proj[..., hd + hn:hd + 2 * hn]).astype(np.complex64)
    Ct = (proj[..., hd + 2 * hn:hd + 3 * hn] + 1j * proj[..., hd + 3 * hn:hd + 4 * hn]).astype(
        np.complex64)
    dt = proj[..., W - H:].copy()
    return x, Bt.reshape(Bsz, T, H, N), Ct.reshape(Bsz, T, H, N), dt


def pack_proj_grad(dx, dB, dC, ddt, H, D, N):
    """d(proj) (B, T, H(D+4N+1)) from the operator's gradients (adjoint of ``unpack_proj``)."""
    dx = np.asarray(dx)
    Bsz, T = dx.shape[:2]
    hd, hn = H * D, H * N
    out = np.zeros((Bsz, T, proj_width(H, D, N)), dtype=np.result_type(dx.real.dtype, np.float32))
    out[..., :hd] = np.real(dx).reshape(Bsz, T, hd)
    dB = np.asarray(dB).reshape(Bsz, T, hn)
    dC = np.asarray(dC).reshape(Bsz, T, hn)
    out[..., hd:hd + hn] = dB.real
    out[..., hd + hn:hd + 2 * hn] = dB.imag
    out[..., hd + 2 * hn:hd + 3 * hn] = dC.real
    out[..., hd + 3 * hn:hd + 4 * hn] = dC.imag
    out[..., hd + 4 * hn:] = np.asarray(ddt).reshape(Bsz, T, H)
    return out


def ssd_from_proj(proj, A, H, D, N, chunk):
    """y (B, T, H, D) float32: the block's unpacking followed by the operator."""
    x, Bt, Ct, dt = unpack_proj(proj, H, D, N)
    return ssd_chunkwise(x, A, Bt, Ct, dt, chunk)

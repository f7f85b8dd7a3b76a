"""numpy restatement of the complex chunkwise SSD operator (test infrastructure; CPU only).

Reference: models/ssd_complex.py in atandra2000/Mamba-3-Lite.

* ``softplus_f32``      - torch.nn.functional.softplus(beta=1, threshold=20), used at
                           models/ssd_complex.py:14 and :82.
* ``ssd_chunkwise``     - models/ssd_complex.py:58-119 (``ssd_complex_chunkwise``) together with
                           :36-55 (``per_chunk_ssd_pytorch``) in complex64, with one deliberate
                           change: the causal masks at :52 and :107 are applied BEFORE ``exp``
                           (``exp(where(mask, seg, -inf))``). The reference multiplies
                           ``exp(seg)`` by the mask, and ``exp`` of the masked-out triangle
                           overflows to inf for strong decays, so ``inf * 0`` turns whole heads into
                           NaN. Where the reference is finite the two agree (checked against the
                           reference's own outputs in tests/test_oracle.py).
* ``ssd_naive``         - models/ssd_complex.py:17-33 (``ssd_naive_complex``): the O(T) recurrence
                           ``s_t = exp(softplus(dt_t) A) s_{t-1} + B_t x_t^T``,
                           ``y_t = sum_n C_t,n s_t,n`` (no conjugate on C), in complex128 by default.
* ``ssd_naive_grads``   - the adjoint of that recurrence: gradients of ``sum(dy * Re(y))`` for
                           x, A, B_t, C_t, dt in PyTorch's convention for complex leaves
                           (grad = dL/dRe + i dL/dIm). This is an independent derivation of what
                           torch.autograd returns through models/ssd_complex.py:58-119. Both take
                           an optional initial state (and final-state gradient) for the state
                           carry of segmented calls.

Shapes follow the reference: x (B,T,H,D) real or complex, A (H,) complex, B_t/C_t (B,T,H,N)
complex, dt (B,T,H) real and pre-softplus.
"""
from __future__ import annotations

import numpy as np

_SOFTPLUS_THRESHOLD = 20.0


def softplus_f32(z):
    """torch softplus with beta=1, threshold=20 (models/ssd_complex.py:14, :82), float32."""
    z = np.asarray(z, dtype=np.float32)
    with np.errstate(over="ignore"):
        soft = np.log1p(np.exp(z)).astype(np.float32)
    return np.where(z > _SOFTPLUS_THRESHOLD, z, soft).astype(np.float32)


def softplus_f64(z):
    z = np.asarray(z, dtype=np.float64)
    with np.errstate(over="ignore"):
        soft = np.log1p(np.exp(z))
    return np.where(z > _SOFTPLUS_THRESHOLD, z, soft)


def softplus_grad_f64(z):
    """Derivative torch uses for softplus: sigmoid(z) below the threshold, 1 above it."""
    z = np.asarray(z, dtype=np.float64)
    sig = 1.0 / (1.0 + np.exp(-np.clip(z, -700.0, 700.0)))
    return np.where(z > _SOFTPLUS_THRESHOLD, 1.0, sig)


def _pad_time(t, pad):
    if pad == 0:
        return t
    widths = [(0, 0)] * t.ndim
    widths[1] = (0, pad)
    return np.pad(t, widths)


def ssd_chunkwise(x, A, B_t, C_t, dt, chunk_size=64):
    """Chunkwise SSD forward in complex64, masked before exp. Returns float32 (B,T,H,D).

    Follows models/ssd_complex.py:69-119 step by step (padding :72-80, A_log :82, chunk views
    :84-87, cumsum and decay_states :89-90, the per-chunk pass :36-55, the inter-chunk decay
    matrix :98-111, Y_off :115, real part and slice :117-119). The four-operand einsums are
    contracted pairwise from the left, the order torch.einsum uses without opt_einsum.
    """
    x = np.asarray(x)
    Bsz, T, H, D = x.shape
    N = B_t.shape[-1]
    C = int(chunk_size)
    pad = (C - T % C) % C
    xp = _pad_time(x, pad)
    Bp = _pad_time(np.asarray(B_t, np.complex64), pad)
    Cp = _pad_time(np.asarray(C_t, np.complex64), pad)
    dtp = _pad_time(np.asarray(dt, np.float32), pad)
    nc = (T + pad) // C

    a = softplus_f32(dtp) * np.asarray(A, np.complex64)  # (B,Tp,H) complex64
    a = a.astype(np.complex64)

    Xc = xp.reshape(Bsz, nc, C, H, D).astype(np.complex64)
    Bc = Bp.reshape(Bsz, nc, C, H, N)
    Cc = Cp.reshape(Bsz, nc, C, H, N)
    Ac = a.reshape(Bsz, nc, C, H)

    cs = np.cumsum(Ac, axis=2, dtype=np.complex64)                  # (b,c,l,h)
    decay_states = np.exp(cs[:, :, -1:, :] - cs).astype(np.complex64)

    # per-chunk pass (models/ssd_complex.py:47-55), masked before exp
    cs_h = np.cumsum(Ac.transpose(0, 1, 3, 2), axis=-1, dtype=np.complex64)   # (b,c,h,l)
    seg = cs_h[..., :, None] - cs_h[..., None, :]                             # (b,c,h,l,s)
    causal = np.tril(np.ones((C, C), dtype=bool))
    with np.errstate(over="ignore", invalid="ignore"):
        L = np.exp(np.where(causal, seg, np.complex64(-np.inf))).astype(np.complex64)
    G = np.einsum("bclhn,bcshn->bclhs", Cc, Bc)                    # sum over n
    GL = G * L.transpose(0, 1, 3, 2, 4)                            # (b,c,l,h,s)
    Y_diag = np.einsum("bclhs,bcshp->bclhp", GL, Xc)
    BD = Bc * decay_states[..., None]                              # (b,c,l,h,n)
    states = np.einsum("bclhn,bclhp->bchpn", BD, Xc)

    # inter-chunk (models/ssd_complex.py:98-111), masked before exp
    cd = cs[:, :, -1, :].transpose(0, 2, 1)                       # (b,h,c)
    cd_cum = np.cumsum(cd, axis=-1, dtype=np.complex64)
    cd_shift = np.concatenate([np.zeros_like(cd_cum[..., :1]), cd_cum[..., :-1]], axis=-1)
    cd_seg = cd_shift[..., :, None] - cd_cum[..., None, :]          # (b,h,z,c)
    strict = np.tril(np.ones((nc, nc), dtype=bool), k=-1)
    with np.errstate(over="ignore", invalid="ignore"):
        decay_chunk = np.exp(np.where(strict, cd_seg, np.complex64(-np.inf))).astype(np.complex64)
    states = np.einsum("bhzc,bchpn->bzhpn", decay_chunk, states)

    with np.errstate(over="ignore", invalid="ignore"):
        ecs = np.exp(cs).astype(np.complex64)
    Y_off = np.einsum("bclhn,bchpn->bclhp", Cc, states) * ecs[..., None]
    Y = (Y_diag + Y_off).real.astype(np.float32)
    return Y.reshape(Bsz, T + pad, H, D)[:, :T]


def ssd_naive(x, A, B_t, C_t, dt, dtype=np.complex128, s0=None, return_state=False):
    """The O(T) recurrence of models/ssd_complex.py:17-33; returns complex (B,T,H,D).

    With ``dtype=np.complex64`` it follows the reference's precision; the default complex128 is
    the ground truth used for error reports. ``s0`` (B,H,N,D) is an initial state (zero in the
    reference); with ``return_state`` the final state s_T is returned as well (the state carry
    of an operator call split into segments: no counterpart in the reference's code).
    """
    real_t = np.float64 if dtype == np.complex128 else np.float32
    sp = softplus_f64(dt) if real_t is np.float64 else softplus_f32(dt)
    Abar = np.exp(sp.astype(real_t) * np.asarray(A).astype(dtype)).astype(dtype)   # (B,T,H)
    x = np.asarray(x).astype(dtype)
    Bt = np.asarray(B_t).astype(dtype)
    Ct = np.asarray(C_t).astype(dtype)
    Bsz, T, H, D = x.shape
    N = Bt.shape[-1]
    s = np.zeros((Bsz, H, N, D), dtype=dtype) if s0 is None else np.asarray(s0).astype(dtype)
    ys = np.empty((Bsz, T, H, D), dtype=dtype)
    for t in range(T):
        s = Abar[:, t, :, None, None] * s + Bt[:, t, :, :, None] * x[:, t, :, None, :]
        ys[:, t] = np.einsum("bhn,bhnd->bhd", Ct[:, t], s)
    return (ys, s) if return_state else ys


def ssd_naive_grads(x, A, B_t, C_t, dt, dy, s0=None, dsT=None):
    """Gradients of L = sum(dy * Re(ssd_naive(...))) in complex128, PyTorch's convention.

    With an initial state ``s0`` and/or an upstream gradient ``dsT`` of the final state
    (L += Re(sum conj(dsT) s_T)), a sixth result is returned: ds0, the gradient of s0.

    Returns ``(dx, dA, dB, dC, ddt)``: dx real when x is real, complex otherwise; dA (H,) complex;
    dB/dC (B,T,H,N) complex; ddt (B,T,H) real. The adjoint state runs backwards in time:
    ``g_t = conj(C_t) dy_t + conj(Abar_{t+1}) g_{t+1}``; then dB_t = g_t conj(x_t),
    dx_t = conj(B_t)^T g_t, d(Abar_t) = <g_t, s_{t-1}>, da_t = d(Abar_t) conj(Abar_t),
    dA = sum_{b,t} da softplus(dt), ddt = Re(da conj(A)) softplus'(dt).
    """
    x_is_complex = np.iscomplexobj(x)
    sp = softplus_f64(dt)
    dsp = softplus_grad_f64(dt)
    A = np.asarray(A).astype(np.complex128)
    Abar = np.exp(sp * A)                                           # (B,T,H)
    X = np.asarray(x).astype(np.complex128)
    Bt = np.asarray(B_t).astype(np.complex128)
    Ct = np.asarray(C_t).astype(np.complex128)
    dy = np.asarray(dy, dtype=np.float64)
    Bsz, T, H, D = X.shape
    N = Bt.shape[-1]

    states = np.empty((Bsz, T, H, N, D), dtype=np.complex128)
    s0c = (np.zeros((Bsz, H, N, D), dtype=np.complex128) if s0 is None
           else np.asarray(s0).astype(np.complex128))
    s = s0c
    for t in range(T):
        s = Abar[:, t, :, None, None] * s + Bt[:, t, :, :, None] * X[:, t, :, None, :]
        states[:, t] = s

    dX = np.empty_like(X)
    dB = np.empty_like(Bt)
    dC = np.empty_like(Ct)
    da = np.empty((Bsz, T, H), dtype=np.complex128)
    g = (np.zeros((Bsz, H, N, D), dtype=np.complex128) if dsT is None
         else np.asarray(dsT).astype(np.complex128))
    for t in range(T - 1, -1, -1):
        g = g + np.conj(Ct[:, t])[..., None] * dy[:, t, :, None, :]
        dC[:, t] = np.einsum("bhd,bhnd->bhn", dy[:, t], np.conj(states[:, t]))
        dB[:, t] = np.einsum("bhnd,bhd->bhn", g, np.conj(X[:, t]))
        dX[:, t] = np.einsum("bhnd,bhn->bhd", g, np.conj(Bt[:, t]))
        prev = states[:, t - 1] if t > 0 else s0c
        dAbar = np.einsum("bhnd,bhnd->bh", g, np.conj(prev))
        da[:, t] = dAbar * np.conj(Abar[:, t])
        g = np.conj(Abar[:, t])[..., None, None] * g

    dA = np.einsum("bth,bth->h", da, sp)
    ddt = np.real(da * np.conj(A)[None, None, :]) * dsp
    dx = dX if x_is_complex else dX.real
    if s0 is not None or dsT is not None:
        return dx, dA, dB, dC, ddt, g
    return dx, dA, dB, dC, ddt

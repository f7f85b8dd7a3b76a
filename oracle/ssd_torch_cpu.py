"""torch-on-CPU restatement of the reference chunkwise SSD (test infrastructure and CPU baseline).

Reference: models/ssd_complex.py:36-119 in atandra2000/Mamba-3-Lite. The reference module cannot
travel with this repository, so this file restates its operator with the same torch ops in the
same order, so that its CPU cost and its autograd graph match the reference's. The only change
is the masking order at models/ssd_complex.py:52 and :107: the causal masks are applied before
``exp`` (``exp(where(mask, seg, -inf))``) so strong decays no longer turn into ``inf * 0 = NaN``.

It is used (1) by tests as a torch fp32/complex64 reference with autograd, and (2) by
``bench.py`` as the timed CPU baseline (kind "port") of the reference's PyTorch dispatch.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _chunk_local_pass(Bc, Cc, Xc, A_log, decay_states):
    """models/ssd_complex.py:36-55 (per_chunk_ssd_pytorch), masked before exp."""
    C = Bc.shape[2]
    causal = torch.tril(torch.ones(C, C, device=Bc.device, dtype=torch.bool))
    cs = A_log.permute(0, 1, 3, 2).cumsum(dim=-1)                 # (b,c,h,l)
    seg = cs.unsqueeze(-1) - cs.unsqueeze(-2)                      # (b,c,h,l,s)
    neg_inf = torch.full((), float("-inf"), dtype=seg.dtype, device=seg.device)
    L = torch.exp(torch.where(causal, seg, neg_inf))
    y_diag = torch.einsum("bclhn,bcshn,bchls,bcshp->bclhp", Cc, Bc, L, Xc)
    chunk_state = torch.einsum("bclhn,bclh,bclhp->bchpn", Bc, decay_states, Xc)
    return y_diag, chunk_state


def ssd_chunkwise_torch(x, A, B_t, C_t, dt, chunk_size: int = 64, cdtype=torch.complex64):
    """models/ssd_complex.py:58-119 on any torch device, masked before exp; returns float32.

    ``cdtype=torch.complex128`` (with float64/complex128 inputs) evaluates the same algorithm in
    double precision, the ground truth for long sequences where fp32 cumsum differences lose
    phase accuracy.
    """
    Bsz, T, H, D = x.shape
    C = int(chunk_size)
    pad = (C - (T % C)) % C
    if pad:
        x = F.pad(x, (0, 0, 0, 0, 0, pad))
        B_t = F.pad(B_t, (0, 0, 0, 0, 0, pad))
        C_t = F.pad(C_t, (0, 0, 0, 0, 0, pad))
        dt = F.pad(dt, (0, 0, 0, pad))
    Tp = T + pad
    nc = Tp // C
    A_log = F.softplus(dt) * A

    def view_chunks(t):
        return t.reshape(Bsz, nc, C, *t.shape[2:])

    Xc = view_chunks(x).to(cdtype)
    Bc, Cc, Ac = view_chunks(B_t), view_chunks(C_t), view_chunks(A_log)
    cs = torch.cumsum(Ac, dim=2)
    decay_states = torch.exp(cs[:, :, -1:, :] - cs)
    y_diag, chunk_state = _chunk_local_pass(Bc, Cc, Xc, Ac, decay_states)

    cd = cs[:, :, -1, :].permute(0, 2, 1).contiguous()
    cd_cum = torch.cumsum(cd, dim=-1)
    cd_shift = torch.cat([torch.zeros_like(cd_cum[..., :1]), cd_cum[..., :-1]], dim=-1)
    cd_seg = cd_shift.unsqueeze(-1) - cd_cum.unsqueeze(-2)
    strict = torch.tril(torch.ones(nc, nc, device=x.device, dtype=torch.bool), diagonal=-1)
    neg_inf = torch.full((), float("-inf"), dtype=cd_seg.dtype, device=cd_seg.device)
    decay_chunk = torch.exp(torch.where(strict, cd_seg, neg_inf))
    carried = torch.einsum("bhzc,bchpn->bzhpn", decay_chunk, chunk_state)
    y_off = torch.einsum("bclhn,bchpn,bclh->bclhp", Cc, carried, torch.exp(cs))
    return (y_diag + y_off).real.reshape(Bsz, Tp, H, D)[:, :T, :, :]

"""Generate the golden fixtures in this folder from the reference implementation itself.

Run from the repository root in a container where the reference checkout is present, giving its
root directory (or set M3SSD_REFERENCE to it):

    python tests/golden/make_golden.py --reference <reference checkout>

``lm_tiny.npz``: a two-layer reference ``Mamba3Transformer`` (models/transformer.py) on CPU, its
parameters, logits, loss and parameter gradients for one batch (see ``make_lm_fixture``).

For every in_proj case (``PROJ_CASES`` in ``oracle/cases.py``) it runs the reference block's own
unpacking of its in_proj output and the operator call inside it (models/mamba_block.py:73-104), and
records the unpacked operands, y, and the gradients of proj and A (see ``run_reference_block``).

For every case in ``oracle/cases.py`` it runs the reference's own ``ssd_complex_chunkwise``
(models/ssd_complex.py:58-119, ``ssd_dispatch="pytorch"``) on CPU, backpropagates
``sum(dy * y)`` through it with torch.autograd, and stores outputs and gradients. Small cases store
the full tensors together with their inputs; the B2 L256 H4 block-shape cases store the input checksums
and a fixed random sample of 4096 entries per tensor (full tensors would be megabytes).
Entries where the reference is not finite (its exp-then-mask overflow) are stored as NaN and are
skipped by the tests.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.cases import (CASES, PROJ_CASES, PROJ_SAMPLED, SAMPLED_CASES,  # noqa: E402
                          make_case, make_proj_case)

N_SAMPLE = 4096


def checksum(a):
    a = np.asarray(a)
    if np.iscomplexobj(a):
        return np.array([np.abs(a.real).astype(np.float64).sum(), np.abs(a.imag).astype(np.float64).sum()])
    return np.array([np.abs(a).astype(np.float64).sum(), 0.0])


def run_reference(ssd_complex_chunkwise, inp, dy, chunk):
    xs = [torch.from_numpy(np.ascontiguousarray(inp[k])).clone().requires_grad_(True)
          for k in ("x", "A", "B_t", "C_t", "dt")]
    y = ssd_complex_chunkwise(*xs, chunk_size=chunk, ssd_dispatch="pytorch")
    (y * torch.from_numpy(dy)).sum().backward()
    out = {"y": y.detach().numpy()}
    for k, t in zip(("dx", "dA", "dB", "dC", "ddt"), xs):
        out[k] = t.grad.detach().numpy()
    return out


def run_reference_block(proj_np, A_np, dy, chunk, dims):
    """The reference block's own SSD input path on a given projection.

    A Mamba3Block (models/mamba_block.py) whose in_proj returns `proj` runs its forward; the
    operator call inside it (models/mamba_block.py:100-104) is wrapped to record its arguments and
    result. The gradient of sum(dy * y) is then taken with respect to proj and A through the
    block's slicing and torch.complex (:73-84) and the reference operator.
    """
    import torch.nn as nn
    import models.mamba_block as mb  # the reference itself

    H, D, N = dims
    cfg = dict(d_model=16, n_heads=H, head_dim=D, state_dim=N, chunk_size=chunk, ffn_dim=32)
    block = mb.Mamba3Block(cfg)
    proj = torch.from_numpy(proj_np.copy()).requires_grad_(True)

    class FixedProj(nn.Module):
        def forward(self, h):
            return proj

    block.in_proj = FixedProj()
    with torch.no_grad():
        block.A.copy_(torch.from_numpy(A_np))
    seen = {}
    original = mb.ssd_complex_chunkwise

    def recording(x_ssm, A, B_t, C_t, dt, **kw):
        y = original(x_ssm, A, B_t, C_t, dt, **kw)
        seen.update(x=x_ssm, B_t=B_t, C_t=C_t, dt=dt, y=y)
        return y

    mb.ssd_complex_chunkwise = recording
    try:
        block._forward_impl(torch.zeros(proj.shape[0], proj.shape[1], 16))
    finally:
        mb.ssd_complex_chunkwise = original
    y = seen["y"]
    dproj, dA = torch.autograd.grad((y * torch.from_numpy(dy)).sum(), [proj, block.A])
    out = {"y": y.detach().numpy(), "dproj": dproj.numpy(), "dA": dA.numpy()}
    unpacked = {k: seen[k].detach().numpy() for k in ("x", "B_t", "C_t", "dt")}
    return out, unpacked


LM_TINY = dict(vocab_size=50, d_model=16, n_layers=2, n_heads=2, head_dim=64, state_dim=64,
               chunk_size=64, ffn_dim=32, max_seq_len=128)


def make_lm_fixture():
    """A tiny reference Mamba3Transformer (models/transformer.py) on CPU in fp32: its parameters
    (A set to seeded complex decays), one batch of tokens and targets, the logits, the
    cross-entropy loss and the gradient of every parameter. Pins the model around the operator
    (m3ssd.lm) to the reference's layers, names and initialisation-independent wiring."""
    from models.transformer import Mamba3Transformer  # the reference itself

    torch.manual_seed(11)
    model = Mamba3Transformer(dict(LM_TINY))
    rng = np.random.Generator(np.random.PCG64(77))
    H = LM_TINY["n_heads"]
    with torch.no_grad():
        for layer in model.layers:
            # slow decays: the reference's exp-then-mask stays finite over a 64-chunk
            a = -np.exp(rng.uniform(np.log(0.01), 0.0, H)) + 1j * rng.uniform(-np.pi, np.pi, H)
            layer.A.copy_(torch.from_numpy(a.astype(np.complex64)))
    T = 128
    tokens = torch.from_numpy(rng.integers(0, LM_TINY["vocab_size"], (2, T)).astype(np.int64))
    targets = torch.from_numpy(rng.integers(0, LM_TINY["vocab_size"], (2, T)).astype(np.int64))
    logits = model(tokens)
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)),
                                             targets.reshape(-1))
    loss.backward()
    rec = {"tokens": tokens.numpy(), "targets": targets.numpy(),
           "logits": logits.detach().numpy(), "loss": np.float64(loss.item())}
    for name, prm in model.state_dict().items():
        rec["param::" + name] = prm.numpy()
    for name, prm in model.named_parameters():
        rec["grad::" + name] = prm.grad.numpy()
    path = os.path.join(HERE, "lm_tiny.npz")
    np.savez_compressed(path, **rec)
    print(f"lm_tiny loss={loss.item():.5f} -> {os.path.getsize(path) / 1024:.1f} KiB")


def make_proj_fixtures(only):
    for name in PROJ_CASES:
        if only and name not in only:
            continue
        proj, A, dy, chunk, dims = make_proj_case(name)
        ref, unpacked = run_reference_block(proj, A, dy, chunk, dims)
        rec = {"chunk": np.int64(chunk), "dims": np.array(dims, np.int64),
               "sum_proj": checksum(proj), "sum_dy": checksum(dy), "sum_A": checksum(A)}
        if name in PROJ_SAMPLED:
            rng = np.random.Generator(np.random.PCG64(4321))
            for k, v in ref.items():
                v = np.asarray(v)
                idx = (np.sort(rng.choice(v.size, N_SAMPLE, replace=False)).astype(np.int64)
                       if v.size > N_SAMPLE else np.arange(v.size, dtype=np.int64))
                rec["idx_" + k] = idx
                rec[k] = v.reshape(-1)[idx]
                rec["nonfinite_" + k] = np.float64(np.mean(~np.isfinite(v)))
        else:
            rec["in_proj"] = proj
            rec["in_A"] = A
            rec["in_dy"] = dy
            for k, v in unpacked.items():
                rec["unpacked_" + k] = v
            for k, v in ref.items():
                rec[k] = v
                rec["nonfinite_" + k] = np.float64(np.mean(~np.isfinite(v)))
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **rec)
        print(f"{name:16s} chunk={chunk:3d} nonfinite(y)={rec['nonfinite_y']:.3f} "
              f"-> {os.path.getsize(path) / 1024:.1f} KiB")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("M3SSD_REFERENCE"),
                    required="M3SSD_REFERENCE" not in os.environ,
                    help="root of the reference checkout (default: $M3SSD_REFERENCE)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from models.ssd_complex import ssd_complex_chunkwise  # the reference itself

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    if not args.only or "lm_tiny" in args.only:
        make_lm_fixture()
    make_proj_fixtures(args.only)
    for name in CASES:
        if args.only and name not in args.only:
            continue
        inp, dy, chunk = make_case(name)
        ref = run_reference(ssd_complex_chunkwise, inp, dy, chunk)
        rec = {"chunk": np.int64(chunk)}
        for k in ("x", "A", "B_t", "C_t", "dt"):
            rec["sum_" + k] = checksum(inp[k])
        rec["sum_dy"] = checksum(dy)
        if name in SAMPLED_CASES:
            rng = np.random.Generator(np.random.PCG64(1234))
            for k, v in ref.items():
                v = np.asarray(v)
                if v.size > N_SAMPLE:
                    idx = np.sort(rng.choice(v.size, N_SAMPLE, replace=False)).astype(np.int64)
                else:
                    idx = np.arange(v.size, dtype=np.int64)
                rec["idx_" + k] = idx
                rec[k] = v.reshape(-1)[idx]
                rec["nonfinite_" + k] = np.float64(np.mean(~np.isfinite(v)))
        else:
            for k in ("x", "A", "B_t", "C_t", "dt"):
                rec["in_" + k] = inp[k]
            rec["in_dy"] = dy
            for k, v in ref.items():
                rec[k] = v
                rec["nonfinite_" + k] = np.float64(np.mean(~np.isfinite(v)))
        path = os.path.join(HERE, name + ".npz")
        np.savez_compressed(path, **rec)
        print(f"{name:16s} chunk={chunk:3d} nonfinite(y)={rec['nonfinite_y']:.3f} "
              f"-> {os.path.getsize(path) / 1024:.1f} KiB")


if __name__ == "__main__":
    main()

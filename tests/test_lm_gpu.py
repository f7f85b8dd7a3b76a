"""The model around the operator (m3ssd.lm) with the CUDA operator inside, on the GPU.

* fp32: the two-layer reference model of tests/golden/lm_tiny.npz (made by the reference itself on
  CPU) with its parameters loaded: logits, loss and every parameter gradient within the tensor-core
  path's stated tolerances.
* bf16 autocast (the reference trainer's mode): the fused SSD input path (ssd_from_proj, y stored
  as bf16) against the block's own unpacking with the plain operator and autocast's cast in front
  of MIMO: same logits, same gradients.
* train_step: loss goes down on a repeated batch.
"""
import numpy as np
import pytest
import torch

import m3ssd
from m3ssd import lm
from test_lm_cpu import LM_TINY, _fixture, _rel
from tolerances import TOL

pytestmark = pytest.mark.gpu


def _model(dev, ssd_fn=None):
    _, params, _ = _fixture()
    model = lm.Mamba3Transformer(dict(LM_TINY), ssd_fn=ssd_fn).to(dev)
    model.load_state_dict({k: v.to(dev) for k, v in params.items()}, strict=True)
    return model


def _unfused(x, A, B_t, C_t, dt, chunk):
    return m3ssd.ssd_complex_chunkwise(x, A, B_t, C_t, dt, chunk_size=chunk)


def test_lm_with_cuda_operator_matches_reference_model(cuda_device):
    tol = TOL["tensor"]
    g, _, grads = _fixture()
    model = _model(cuda_device)
    tokens = torch.from_numpy(g["tokens"]).to(cuda_device)
    targets = torch.from_numpy(g["targets"]).to(cuda_device)
    logits = model(tokens)
    assert _rel(logits.detach().cpu().numpy(), g["logits"]) < tol["y_normwise"]
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)),
                                             targets.reshape(-1))
    assert abs(loss.item() - float(g["loss"])) < 1e-4 * abs(float(g["loss"]))
    loss.backward()
    for k, p in model.named_parameters():
        assert _rel(p.grad.cpu().numpy(), grads[k]) < tol["g_normwise"], k
    # the training form: cross-entropy on the padded logits (pad columns at -inf)
    with torch.no_grad():
        fused_loss = model(tokens, targets)
    assert abs(fused_loss.item() - loss.item()) < 1e-6 * abs(loss.item())


def test_bf16_autocast_fused_equals_block_composition(cuda_device):
    g, _, _ = _fixture()
    tokens = torch.from_numpy(g["tokens"]).to(cuda_device)
    targets = torch.from_numpy(g["targets"]).to(cuda_device)
    out = []
    for fn in (None, _unfused):
        model = _model(cuda_device, ssd_fn=fn)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(tokens)
            loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)).float(),
                                                     targets.reshape(-1))
        loss.backward()
        out.append((logits.detach(), {k: p.grad.detach() for k, p in model.named_parameters()}))
    (l0, g0), (l1, g1) = out
    assert l0.dtype == torch.bfloat16
    assert torch.equal(l0, l1)
    for k in g0:
        rel = ((g0[k] - g1[k]).abs().max() / g1[k].abs().max().clamp_min(1e-30)).item()
        assert rel < 1e-6, (k, rel)


def test_train_step_reduces_loss_on_a_repeated_batch(cuda_device):
    g, _, _ = _fixture()
    model = _model(cuda_device)
    tokens = torch.from_numpy(g["tokens"]).to(cuda_device)
    targets = torch.from_numpy(g["targets"]).to(cuda_device)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-3)
    losses = [lm.train_step(model, opt, tokens, targets).item() for _ in range(8)]
    assert all(np.isfinite(losses))
    assert losses[-1] < losses[0] - 0.1, losses

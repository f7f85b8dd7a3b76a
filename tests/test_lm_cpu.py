"""The model around the operator (m3ssd.lm) against the reference's own model, on CPU.

tests/golden/lm_tiny.npz holds a two-layer reference Mamba3Transformer (models/transformer.py):
its parameters, one batch, the logits, the loss and every parameter's gradient (fp32, no
autocast). Here the same parameters load into m3ssd.lm.Mamba3Transformer with the operator
replaced by the CPU restatement of the reference's SSD (oracle/ssd_torch_cpu.py, identical to the
reference where it is finite), so what is compared is everything around the operator: layer
order, residuals, norms, MIMO, the FFN, the tied head and the parameter names. The GPU test
(tests/test_lm_gpu.py) repeats this with the CUDA operator inside.
"""
import os

import numpy as np
import pytest
import torch

from m3ssd import lm
from oracle.ssd_torch_cpu import ssd_chunkwise_torch

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "lm_tiny.npz")
LM_TINY = dict(vocab_size=50, d_model=16, n_layers=2, n_heads=2, head_dim=64, state_dim=64,
               chunk_size=64, ffn_dim=32, max_seq_len=128)


def _ssd_cpu(x, A, B_t, C_t, dt, chunk):
    return ssd_chunkwise_torch(x, A, B_t, C_t, dt, chunk_size=chunk)


def _fixture():
    g = dict(np.load(GOLDEN))
    params = {k[len("param::"):]: torch.from_numpy(v) for k, v in g.items()
              if k.startswith("param::")}
    grads = {k[len("grad::"):]: v for k, v in g.items() if k.startswith("grad::")}
    return g, params, grads


def _rel(a, b):
    a, b = np.asarray(a), np.asarray(b)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def test_state_dict_matches_the_reference_model():
    _, params, _ = _fixture()
    model = lm.Mamba3Transformer(dict(LM_TINY))
    sd = model.state_dict()
    assert sorted(sd) == sorted(params)
    for k, v in params.items():
        assert tuple(sd[k].shape) == tuple(v.shape), k
        assert sd[k].dtype == v.dtype, k
    # initialisation: MIMO identity, A = -1, tied head
    assert torch.equal(model.layers[0].mimo.mix.weight, torch.eye(128))
    assert torch.equal(model.layers[1].A, torch.full((2,), -1.0, dtype=torch.complex64))
    assert model.lm_head.weight is model.embed.weight


def test_logits_loss_and_grads_match_the_reference_model():
    g, params, grads = _fixture()
    model = lm.Mamba3Transformer(dict(LM_TINY), ssd_fn=_ssd_cpu)
    model.load_state_dict(params, strict=True)
    tokens = torch.from_numpy(g["tokens"])
    targets = torch.from_numpy(g["targets"])
    logits = model(tokens)
    assert _rel(logits.detach().numpy(), g["logits"]) < 1e-5
    loss = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.size(-1)),
                                             targets.reshape(-1))
    assert abs(loss.item() - float(g["loss"])) < 1e-5 * abs(float(g["loss"]))
    loss.backward()
    named = dict(model.named_parameters())
    assert sorted(named) == sorted(grads)
    for k, ref in grads.items():
        assert _rel(named[k].grad.numpy(), ref) < 1e-4, k


def test_train_step_updates_every_parameter_once():
    g, params, _ = _fixture()
    model = lm.Mamba3Transformer(dict(LM_TINY), ssd_fn=_ssd_cpu)
    model.load_state_dict(params, strict=True)
    before = {k: v.detach().clone() for k, v in model.named_parameters()}
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    loss = lm.train_step(model, opt, torch.from_numpy(g["tokens"]),
                         torch.from_numpy(g["targets"]), amp_dtype=None)
    assert abs(loss.item() - float(g["loss"])) < 1e-5 * abs(float(g["loss"]))
    for k, v in model.named_parameters():
        assert not torch.equal(v, before[k]), k
        assert v.grad is None, k  # zeroed (set to None) after the step


def test_model_without_ssd_fn_has_no_cpu_path():
    model = lm.Mamba3Transformer(dict(LM_TINY))
    with pytest.raises(RuntimeError, match="no CPU"):
        model(torch.zeros(1, 64, dtype=torch.long))

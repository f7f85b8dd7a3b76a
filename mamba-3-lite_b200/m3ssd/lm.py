"""The reference's language model with this operator in its blocks: the whole-model step.

The caller of the operator in atandra2000/Mamba-3-Lite is ``Mamba3Block`` (models/mamba_block.py:
15-121) inside ``Mamba3Transformer`` (models/transformer.py:30-78), trained by ``train_step``
(training/pretrain.py:136-171). The reference's modules cannot be imported where this package
runs, so this module states the same network around ``ssd_from_proj``:

    block:  x + out_proj(MIMO(SSD(in_proj(RMSNorm(x)))))  then  x + W_down(silu(g) * u),
            (g, u) = W_gate_up(RMSNorm(x))                         (models/mamba_block.py:52-96)
    MIMO:   one dense (H*D x H*D) mix of the head channels, identity-initialised (models/mimo.py)
    model:  embedding -> blocks -> RMSNorm -> tied lm_head; Linear / Embedding weights ~ N(0, std)
            except the MIMO identity (models/transformer.py:45-78)

Module, attribute and parameter names, shapes, dtypes and initialisation are the reference's, so a
reference checkpoint's state_dict loads into ``Mamba3Transformer`` here unchanged and the other
way round. The differences:

* the block's SSD input path (slices, ``.float()``, ``torch.complex``, the operator call,
  models/mamba_block.py:73-104) is one fused call, ``ssd_from_proj``, whose results are identical
  to that composition with this package's operator; under bf16 autocast y leaves the kernels as
  bf16, the dtype the MIMO Linear would cast it to (bit-identical);
* ``ssd_dispatch`` is accepted and ignored (every value runs the CUDA kernels);
* ``ssd_fn`` (tests only) replaces the operator by another function of
  ``(x, A, B_t, C_t, dt, chunk_size)`` on the unpacked operands, e.g. a CPU restatement.

``train_step`` is the reference's micro-step without gradient accumulation, NaN guard or LR
schedule: autocast forward, cross-entropy, backward, gradient-norm clip, optimizer step, zero grad.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ssd_proj import ssd_from_proj, unpack_proj


@dataclass
class ModelConfig:
    """The reference's model hyperparameters (models/transformer.py:12-27), same defaults."""
    vocab_size: int = 50257
    d_model: int = 1024
    n_layers: int = 28
    n_heads: int = 16
    head_dim: int = 64
    state_dim: int = 64
    chunk_size: int = 64
    ssd_dispatch: str = "cuda"
    ffn_dim: int = 2048
    max_seq_len: int = 2048
    weight_tying: bool = True
    rms_norm_eps: float = 1e-5
    init_std: float = 0.02
    grad_checkpoint: bool = False


class MIMO(nn.Module):
    """Dense mix of all head channels, (B, T, H, D) in and out, identity at initialisation."""

    def __init__(self, n_heads: int, head_dim: int):
        super().__init__()
        self.n_heads = n_heads
        self.head_dim = head_dim
        self.mix = nn.Linear(n_heads * head_dim, n_heads * head_dim, bias=False)
        nn.init.eye_(self.mix.weight)
        self.mix._identity_init = True  # kept by the model-wide initialiser

    def forward(self, y: torch.Tensor) -> torch.Tensor:
        Bsz, T, H, D = y.shape
        return self.mix(y.reshape(Bsz, T, H * D)).reshape(Bsz, T, H, D)


def _autocast_bf16() -> bool:
    return (torch.is_autocast_enabled("cuda")
            and torch.get_autocast_dtype("cuda") == torch.bfloat16)


class Mamba3Block(nn.Module):
    """One layer: complex SSD mixing with MIMO, then a SwiGLU FFN, both pre-norm residual."""

    def __init__(self, cfg: dict, layer_idx: int = 0, ssd_fn=None):
        super().__init__()
        self.layer_idx = layer_idx
        self.d_model = cfg["d_model"]
        self.n_heads = cfg["n_heads"]
        self.head_dim = cfg["head_dim"]
        self.state_dim = cfg["state_dim"]
        self.chunk_size = cfg.get("chunk_size", 64)
        self.rms_norm_eps = cfg.get("rms_norm_eps", 1e-5)
        self.grad_checkpoint = cfg.get("grad_checkpoint", False)
        self.ssd_fn = ssd_fn
        H, D, N = self.n_heads, self.head_dim, self.state_dim
        self.in_proj = nn.Linear(self.d_model, H * (D + 4 * N + 1), bias=False)
        self.mimo = MIMO(H, D)
        self.out_proj = nn.Linear(H * D, self.d_model, bias=False)
        self.A = nn.Parameter(torch.full((H,), -1.0, dtype=torch.complex64))
        self.norm1 = nn.RMSNorm(self.d_model, eps=self.rms_norm_eps)
        self.norm2 = nn.RMSNorm(self.d_model, eps=self.rms_norm_eps)
        self.ffn_gate_up = nn.Linear(self.d_model, 2 * cfg["ffn_dim"], bias=False)
        self.ffn_down = nn.Linear(cfg["ffn_dim"], self.d_model, bias=False)

    def _ssd(self, proj: torch.Tensor) -> torch.Tensor:
        H, D, N = self.n_heads, self.head_dim, self.state_dim
        if self.ssd_fn is not None:
            x, B_t, C_t, dt = unpack_proj(proj, H, D, N)
            return self.ssd_fn(x, self.A, B_t, C_t, dt, self.chunk_size)
        y_dtype = torch.bfloat16 if _autocast_bf16() else torch.float32
        return ssd_from_proj(proj, self.A, H, D, N, chunk_size=self.chunk_size, y_dtype=y_dtype)

    def _forward_impl(self, x: torch.Tensor) -> torch.Tensor:
        Bsz, T, _ = x.shape
        y = self.mimo(self._ssd(self.in_proj(self.norm1(x))))
        x = x + self.out_proj(y.reshape(Bsz, T, self.n_heads * self.head_dim))
        gate, up = self.ffn_gate_up(self.norm2(x)).chunk(2, dim=-1)
        return x + self.ffn_down(F.silu(gate) * up)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """(B, T, d_model) -> (B, T, d_model)."""
        if self.grad_checkpoint and self.training:
            return torch.utils.checkpoint.checkpoint(self._forward_impl, x, use_reentrant=False)
        return self._forward_impl(x)


class Mamba3Transformer(nn.Module):
    """Token ids (B, T) -> logits (B, T, vocab)."""

    def __init__(self, cfg: ModelConfig | dict, ssd_fn=None):
        super().__init__()
        if isinstance(cfg, dict):
            cfg = ModelConfig(**cfg)
        self.cfg = cfg
        self.embed = nn.Embedding(cfg.vocab_size, cfg.d_model)
        self.layers = nn.ModuleList([Mamba3Block(cfg.__dict__, layer_idx=i, ssd_fn=ssd_fn)
                                     for i in range(cfg.n_layers)])
        self.norm_f = nn.RMSNorm(cfg.d_model, eps=cfg.rms_norm_eps)
        self.lm_head = nn.Linear(cfg.d_model, cfg.vocab_size, bias=False)
        if cfg.weight_tying:
            self.lm_head.weight = self.embed.weight
        self.apply(self._init_weights)

    def _init_weights(self, module):
        if getattr(module, "_identity_init", False):
            return
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=self.cfg.init_std)

    def _padded_logits(self, h: torch.Tensor) -> torch.Tensor:
        """lm_head(h) with the head's rows padded to a multiple of 64 on the GPU: with the
        reference's 50257-entry vocabulary the logits' row stride is not 16-byte aligned and
        cuBLAS falls back to an old unaligned tensor-op kernel (~7x slower on the head's three
        GEMMs). The first `vocab_size` columns are the logits."""
        pad = (-self.cfg.vocab_size) % 64
        if pad == 0 or h.device.type != "cuda":
            return self.lm_head(h)
        return F.linear(h, F.pad(self.lm_head.weight, (0, 0, 0, pad)))

    def forward(self, tokens: torch.Tensor, targets: torch.Tensor | None = None) -> torch.Tensor:
        """Logits (B, T, vocab) as the reference's model returns them; with ``targets`` the mean
        cross-entropy instead (ignore_index -100), computed on the padded logits with the pad
        columns at -inf (the same loss, without copying the logits out of their padded rows)."""
        x = self.embed(tokens)
        for layer in self.layers:
            x = layer(x)
        logits = self._padded_logits(self.norm_f(x))
        V = self.cfg.vocab_size
        if targets is None:
            return logits[..., :V]
        if logits.size(-1) > V:
            logits[..., V:] = float("-inf")  # exp(-inf) = 0: the pad columns add nothing
        return F.cross_entropy(logits.reshape(-1, logits.size(-1)), targets.reshape(-1),
                               ignore_index=-100)


def train_step(model: nn.Module, optimizer: torch.optim.Optimizer, tokens: torch.Tensor,
               targets: torch.Tensor, max_grad_norm: float = 1.0,
               amp_dtype: torch.dtype | None = torch.bfloat16) -> torch.Tensor:
    """One optimizer step on one batch; returns the cross-entropy loss (a device scalar, not
    synchronised). ``amp_dtype=None`` runs without autocast."""
    device_type = tokens.device.type
    ctx = (torch.autocast(device_type, dtype=amp_dtype) if amp_dtype is not None
           else torch.autocast(device_type, enabled=False))
    with ctx:
        loss = model(tokens, targets)  # the reference's cross-entropy over model(tokens)
    loss.backward()
    nn.utils.clip_grad_norm_(model.parameters(), max_grad_norm)
    optimizer.step()
    optimizer.zero_grad(set_to_none=True)
    return loss.detach()

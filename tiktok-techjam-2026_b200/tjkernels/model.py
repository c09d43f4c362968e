"""A stand-alone encoder module with the harness's parameter layout.

The reference hook lives on the harness's ``BaselineTransformer``
(``torch_transformer_benchmark.py:155-179``); the engine only needs a module
with ``config`` (d_model, num_heads, ffn_dim, num_layers, causal) and the
submodules ``layers[i].norm1 / attention.{q,k,v,out}_proj / norm2 / ffn_in /
ffn_out`` and ``final_norm``.  ``Encoder`` provides exactly that layout (same
names and construction order, so a seeded construction gives the same default
initialisation and a strict ``load_state_dict`` from the harness model
works), with ``forward`` routed to the sm_100a engine.  It is for callers
without the harness: the benchmark and the multi-GPU shards.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.nn as nn

from .engine import forward as _engine_forward


@dataclass(frozen=True)
class EncoderConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool = True


class _Attention(nn.Module):
    def __init__(self, d_model: int) -> None:
        super().__init__()
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)


class _Block(nn.Module):
    def __init__(self, d_model: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = _Attention(d_model)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)


class Encoder(nn.Module):
    """Pre-LN causal encoder stack; ``forward`` runs the tjkernels engine."""

    def __init__(self, config: EncoderConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [_Block(config.d_model, config.ffn_dim) for _ in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor,
                valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        return _engine_forward(self, x, valid_token_mask)


def torch_forward(module: nn.Module, x: torch.Tensor,
                  valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The harness's forward in plain torch fp32 on ``module``'s parameters,
    for accuracy checks (the autotuner's gate), never the engine's path.

    Pre-LN blocks ``x += attn(LN1 x)``, ``x += W2 gelu_erf(W1 LN2 x)``; keys
    at or above a query (causal) or at padded positions get -inf before an
    fp32 softmax; padded rows are zeroed after attention, after each block and
    at the end (``torch_transformer_benchmark.py:66-179``).
    """
    import torch.nn.functional as F

    cfg = module.config
    b, s, d = x.shape
    heads = cfg.num_heads
    hd = d // heads
    mask = valid_token_mask
    keep = None if mask is None else mask.to(torch.float32)[:, :, None]
    h = x.float()
    causal = torch.ones(s, s, dtype=torch.bool, device=x.device).triu(1) if cfg.causal else None

    def lin(layer, t):
        return F.linear(t, layer.weight.float(), layer.bias.float())

    def ln(norm, t):
        return F.layer_norm(t, (d,), norm.weight.float(), norm.bias.float(), norm.eps)

    for blk in module.layers:
        a = ln(blk.norm1, h)
        att = blk.attention
        q, k, v = (lin(p, a).view(b, s, heads, hd).transpose(1, 2)
                   for p in (att.q_proj, att.k_proj, att.v_proj))
        scores = (q @ k.transpose(-1, -2)) * hd ** -0.5
        if causal is not None:
            scores = scores.masked_fill(causal, float("-inf"))
        if mask is not None:
            scores = scores.masked_fill(~mask.bool()[:, None, None, :], float("-inf"))
        ctx = (torch.softmax(scores, dim=-1) @ v).transpose(1, 2).reshape(b, s, d)
        attn = lin(att.out_proj, ctx)
        if keep is not None:
            attn = attn * keep
        h = h + attn
        h = h + lin(blk.ffn_out, F.gelu(lin(blk.ffn_in, ln(blk.norm2, h)), approximate="none"))
        if keep is not None:
            h = h * keep
    out = ln(module.final_norm, h)
    if keep is not None:
        out = out * keep
    return out.to(x.dtype)

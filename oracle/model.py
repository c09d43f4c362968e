"""CPU oracle for the fused causal Transformer-encoder forward.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (the ``tjkernels``
package, the C-ABI library) may import this module; it is the checker that
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
compare against.

It restates, in plain fp32 PyTorch on the CPU, the reference harness's model
and helpers (file:line refer to ``torch_transformer_benchmark.py`` in the
reference project):

* ``ModelConfig``         -- ``TransformerConfig`` (:37-62), same field names.
* ``ReferenceModel``      -- ``BaselineTransformer`` (:155-179) built from
  ``BaselineTransformerBlock`` (:131-152) and ``BaselineSelfAttention``
  (:65-128).  Submodule names and construction order are the same, so the
  same ``torch.manual_seed`` yields bit-identical default-initialised weights
  and a strict ``load_state_dict`` between the two succeeds.
* ``generate_case``       -- ``generate_random_case`` (:238-276): same
  generator calls in the same order, so a seed gives the same ``x``/mask.
* ``within_budget`` / ``budget_usage`` -- the accuracy rule of
  ``compare_outputs`` (:293-360, the OR test at :318-320) and the
  budget-usage figure of ``bench/autotune.py:61-68``.

Parity pin: ``tests/golden/make_golden.py`` ran the reference's own
``BaselineTransformer`` and ``generate_random_case`` (imported from the
reference checkout) and stored inputs, outputs and per-parameter checksums in
``tests/golden/*.npz``; ``tests/test_oracle_golden.py`` checks this module
against them.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F


@dataclass(frozen=True)
class ModelConfig:
    """Shape of one benchmark case (``TransformerConfig``, harness :37-62)."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads

    @property
    def tokens(self) -> int:
        return self.batch_size * self.seq_len


class _Attention(nn.Module):
    """Multi-head self-attention with separate q/k/v/out projections
    (harness :65-128).  ``q_proj``..``out_proj`` are created in this order so
    the RNG stream matches the reference's default initialisation."""

    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.q_proj = nn.Linear(d_model, d_model)
        self.k_proj = nn.Linear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor],
                causal: bool) -> torch.Tensor:
        b, s, _ = x.shape
        heads, hd = self.num_heads, self.head_dim

        def split(t: torch.Tensor) -> torch.Tensor:
            return t.view(b, s, heads, hd).transpose(1, 2)

        q, k, v = split(self.q_proj(x)), split(self.k_proj(x)), split(self.v_proj(x))
        scores = (q @ k.transpose(-2, -1)) * (hd ** -0.5)
        if causal:
            upper = torch.ones((s, s), dtype=torch.bool, device=x.device).triu(1)
            scores = scores.masked_fill(upper, float("-inf"))
        if mask is not None:
            scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(x.dtype)
        ctx = (probs @ v).transpose(1, 2).reshape(b, s, self.d_model)
        out = self.out_proj(ctx)
        if mask is not None:
            out = out.masked_fill(~mask[..., None], 0)
        return out


class _Block(nn.Module):
    """Pre-LN block: x += attn(LN1 x); x += W2 gelu_erf(W1 LN2 x)
    (harness :131-152)."""

    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = _Attention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)

    def forward(self, x: torch.Tensor, mask: Optional[torch.Tensor],
                causal: bool) -> torch.Tensor:
        x = x + self.attention(self.norm1(x), mask, causal)
        x = x + self.ffn_out(F.gelu(self.ffn_in(self.norm2(x)), approximate="none"))
        if mask is not None:
            x = x.masked_fill(~mask[..., None], 0)
        return x


class ReferenceModel(nn.Module):
    """The reference encoder stack (``BaselineTransformer``, harness
    :155-179): ``layers`` then ``final_norm``, padded rows zeroed."""

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList(
            [_Block(config.d_model, config.num_heads, config.ffn_dim)
             for _ in range(config.num_layers)]
        )
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor,
                valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        for layer in self.layers:
            x = layer(x, valid_token_mask, self.config.causal)
        x = self.final_norm(x)
        if valid_token_mask is not None:
            x = x.masked_fill(~valid_token_mask[..., None], 0)
        return x


def build_model(config: ModelConfig, seed: int = 0) -> ReferenceModel:
    """Seeded default initialisation on the CPU in fp32, exactly as the
    harness does (``torch.manual_seed`` then construct, :687,694)."""
    torch.manual_seed(seed)
    return ReferenceModel(config).eval()


def generate_case(config: ModelConfig, seed: int, padding_ratio: float,
                  input_scale: float = 1.0,
                  device: str = "cpu") -> Tuple[torch.Tensor, torch.Tensor]:
    """Seeded input and prefix mask (``generate_random_case``, :238-276).

    The minimum valid length is ``max(1, round(S * (1 - padding_ratio)))`` and
    lengths are drawn uniformly in ``[min_valid, S]``; padded rows of ``x``
    are zero.  Generate on the CPU and move: CPU and CUDA generators give
    different streams.
    """
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    b, s, d = config.batch_size, config.seq_len, config.d_model
    x = torch.randn(b, s, d, generator=gen, device=device, dtype=torch.float32)
    x = x * input_scale
    if padding_ratio <= 0:
        return x, torch.ones(b, s, dtype=torch.bool, device=device)
    min_valid = max(1, int(round(s * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=s + 1, size=(b,),
                            generator=gen, device=device)
    mask = torch.arange(s, device=device)[None, :] < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


@torch.no_grad()
def oracle_forward(model: ReferenceModel, x: torch.Tensor,
                   mask: Optional[torch.Tensor]) -> torch.Tensor:
    """fp32 forward with full-precision matmuls (TF32 off).

    Calls ``ReferenceModel.forward`` explicitly, so a subclass that routes
    its own ``forward`` elsewhere (the harness hook) is still checked against
    the reference math."""
    prev = torch.get_float32_matmul_precision()
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.set_float32_matmul_precision("highest")
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return ReferenceModel.forward(model, x, mask)
    finally:
        torch.set_float32_matmul_precision(prev)
        torch.backends.cuda.matmul.allow_tf32 = prev_tf32


def within_budget(ref: torch.Tensor, got: torch.Tensor,
                  atol: float = 1e-2, rtol: float = 1e-2) -> torch.Tensor:
    """Element-wise ``|got-ref| <= atol OR |got-ref| <= rtol*|ref|`` on finite
    values (harness :313-321)."""
    ref = ref.detach().float()
    got = got.detach().float()
    err = (got - ref).abs()
    finite = torch.isfinite(ref) & torch.isfinite(got)
    return finite & ((err <= atol) | (err <= rtol * ref.abs()))


def budget_usage(ref: torch.Tensor, got: torch.Tensor,
                 atol: float = 1e-2, rtol: float = 1e-2) -> float:
    """Worst fraction of its own error budget any element uses
    (``bench/autotune.py:61-68``); <= 1.0 means every element passes."""
    ref = ref.detach().float()
    err = (got.detach().float() - ref).abs()
    budget = (ref.abs() * rtol).clamp_min(atol)
    usage = err / budget
    if not bool(torch.isfinite(usage).all()):
        return math.inf
    return float(usage.max()) if usage.numel() else 0.0


# The five configurations the benchmark is quoted on: (config, padding ratio).
# Padding ratio p gives lengths uniform in [max(1, round(S(1-p))), S].
BENCH_CONFIGS = {
    0: (ModelConfig(2, 128, 512, 8, 2048, 4, True), 0.5),
    1: (ModelConfig(1, 64, 768, 12, 3072, 4, True), 0.0),
    2: (ModelConfig(8, 1024, 1024, 16, 4096, 4, True), 1.0 - 1.0 / 1024),
    3: (ModelConfig(4, 4096, 1024, 16, 4096, 4, True), 0.5),
    4: (ModelConfig(64, 2048, 4096, 32, 16384, 12, True), 0.5),
}


def forward_flops(config: ModelConfig) -> float:
    """Algorithmic forward FLOPs on the full padded shape: per layer
    QKV 6Td^2 + out-proj 2Td^2 + FFN 4TdF + causal attention
    4*B*H*hd*S(S+1)/2 (half of that without the causal triangle)."""
    t, d, f = config.tokens, config.d_model, config.ffn_dim
    b, s, h, hd = config.batch_size, config.seq_len, config.num_heads, config.head_dim
    attn = 4.0 * b * h * hd * (s * (s + 1) / 2 if config.causal else s * s)
    return config.num_layers * (8.0 * t * d * d + 4.0 * t * d * f + attn)

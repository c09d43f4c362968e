"""Multi-GPU layouts of the forward (one process per GPU).

Batch sharding (the default): every layer of the encoder works within one
sequence (row-wise GEMMs and LayerNorms, causal self-attention inside a
sequence), so sequences are independent: a batch splits across ranks with no
collective in the forward.  Weights are replicated.  ``shard_range`` gives
each rank a contiguous slice of the batch; ``balanced_shards`` instead
balances the valid-token work when padded tiles are skipped.

Tensor parallelism (optional, for the largest model): each rank holds H/W
heads and F/W FFN columns.  QKV and FFN-in are column-parallel, the
out-projection and FFN-out row-parallel; their partial outputs are summed
with an all-reduce (the bias added once, by rank 0), so every rank keeps the
full residual stream and runs the LayerNorms replicated.  ``tp_shard`` cuts
one block's weights; ``tp_torch_forward`` is the same computation in plain
torch fp32 (the check for the sharding math on any backend);
``enable_tensor_parallel`` switches a module's engine to this layout.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence, Tuple

import torch


def shard_range(batch: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous [start, end) of sequences for ``rank``; sizes differ by <= 1."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def balanced_shards(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Assign sequences to ranks so each rank's sum of causal work
    (len*(len+1)/2 attention plus len for the GEMMs) is balanced: greedy
    longest-first onto the least-loaded rank."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: -int(lengths[i]))
    loads = [0.0] * world
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        n = int(lengths[i])
        r = min(range(world), key=lambda k: (loads[k], k))
        shards[r].append(i)
        loads[r] += n * (n + 1) / 2 + n
    return [sorted(s) for s in shards]


def balanced_equal_shards(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Like ``balanced_shards`` but every rank gets the same number of
    sequences (``len(lengths)`` must be a multiple of ``world``): sort by
    causal work, longest first, and deal in snake order (0..w-1, w-1..0, ...),
    so each rank's batch has the same shape and close to the same work."""
    if world <= 0 or len(lengths) % world != 0:
        raise ValueError("the number of sequences must be a positive multiple of world")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    shards: List[List[int]] = [[] for _ in range(world)]
    for k, i in enumerate(order):
        rnd, pos = divmod(k, world)
        shards[pos if rnd % 2 == 0 else world - 1 - pos].append(i)
    return [sorted(s) for s in shards]


def tp_shard(block: torch.nn.Module, rank: int, world: int) -> Dict[str, torch.Tensor]:
    """Rank ``rank``'s slice of one block (nn.Linear ``[out, in]`` layouts):
    wqkv ``[3d/W, d]`` (its heads' rows of q, k and v), wo ``[d, d/W]``,
    w1 ``[F/W, d]``, w2 ``[d, F/W]``; biases of the column-parallel layers
    sliced, of the row-parallel ones kept whole (rank 0 adds them)."""
    att = block.attention
    d = att.q_proj.weight.shape[1]
    f = block.ffn_in.weight.shape[0]
    if d % world or f % world:
        raise ValueError(f"d_model {d} and ffn_dim {f} must divide by the tensor-parallel size")
    ds, fs = d // world, f // world
    rows = slice(rank * ds, (rank + 1) * ds)
    cols = slice(rank * fs, (rank + 1) * fs)
    return {
        "wqkv": torch.cat([att.q_proj.weight[rows], att.k_proj.weight[rows],
                           att.v_proj.weight[rows]], dim=0),
        "bqkv": torch.cat([att.q_proj.bias[rows], att.k_proj.bias[rows],
                           att.v_proj.bias[rows]], dim=0),
        "wo": att.out_proj.weight[:, rows],
        "bo": att.out_proj.bias,
        "w1": block.ffn_in.weight[cols],
        "b1": block.ffn_in.bias[cols],
        "w2": block.ffn_out.weight[:, cols],
        "b2": block.ffn_out.bias,
    }


def tp_torch_forward(module: torch.nn.Module, x: torch.Tensor,
                     valid_token_mask: Optional[torch.Tensor], rank: int, world: int,
                     group=None) -> torch.Tensor:
    """The tensor-parallel forward in plain torch fp32 with ``all_reduce``
    over ``group`` (any backend, gloo included): the reference for the
    sharded computation that ``enable_tensor_parallel`` runs on the GPU."""
    import torch.distributed as dist
    import torch.nn.functional as F

    cfg = module.config
    b, s, d = x.shape
    heads = cfg.num_heads // world
    hd = d // cfg.num_heads
    mask = valid_token_mask
    keep = None if mask is None else mask.to(torch.float32)[:, :, None]
    h = x.float()
    causal = torch.ones(s, s, dtype=torch.bool, device=x.device).triu(1) if cfg.causal else None

    def ln(norm, t):
        return F.layer_norm(t, (d,), norm.weight.float(), norm.bias.float(), norm.eps)

    def reduced(partial, bias):
        dist.all_reduce(partial, group=group)
        return partial + bias.float()

    for blk in module.layers:
        w = {k: v.float() for k, v in tp_shard(blk, rank, world).items()}
        qkv = F.linear(ln(blk.norm1, h), w["wqkv"], w["bqkv"]).view(b, s, 3, heads, hd)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
        scores = (q @ k.transpose(-1, -2)) * hd ** -0.5
        if causal is not None:
            scores = scores.masked_fill(causal, float("-inf"))
        if mask is not None:
            scores = scores.masked_fill(~mask.bool()[:, None, None, :], float("-inf"))
        ctx = (torch.softmax(scores, dim=-1) @ v).transpose(1, 2).reshape(b, s, heads * hd)
        attn = reduced(F.linear(ctx, w["wo"]), w["bo"])
        if keep is not None:
            attn = attn * keep
        h = h + attn
        hid = F.gelu(F.linear(ln(blk.norm2, h), w["w1"], w["b1"]), approximate="none")
        h = h + reduced(F.linear(hid, w["w2"]), w["b2"])
        if keep is not None:
            h = h * keep
    out = ln(module.final_norm, h)
    if keep is not None:
        out = out * keep
    return out.to(x.dtype)


def enable_tensor_parallel(module: torch.nn.Module, group=None) -> None:
    """Run ``module``'s engine tensor-parallel over ``group`` (default: the
    world): this rank keeps its slice of the weights, every rank must call
    the forward with the same inputs, and each gets the full output."""
    import torch.distributed as dist
    from . import engine

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cfg = module.config
    if cfg.num_heads % world or cfg.ffn_dim % world:
        raise ValueError("num_heads and ffn_dim must divide by the tensor-parallel size")
    object.__setattr__(module, "_tj_tp", (group, rank, world))
    engine.reset_engines(module)


def disable_tensor_parallel(module: torch.nn.Module) -> None:
    from . import engine

    if hasattr(module, "_tj_tp"):
        object.__delattr__(module, "_tj_tp")
    engine.reset_engines(module)

"""Shape -> execution-plan dispatch.

Same surface as the reference's ``tjkernels/plans.py``: a frozen ``Plan`` of
knobs (:29-67), ``shape_key`` (:70-77), ``default_plan`` heuristics
(:80-134), a JSON table of tuned plans keyed by shape (:147-157),
``set_override`` (:141-144), ``select_plan`` with ``TJ_*`` environment
overrides (:160-190) and ``save_plans`` (:193-198).

The knobs differ because there is one backend: the kernel-choice knobs of the
reference (attn/ffn/norm = triton|torch|sdpa) are gone, and the remaining ones
choose the tensor-core input type, the precision of the residual deltas and
whether the whole forward is replayed as a CUDA graph.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass, replace
from pathlib import Path
from typing import Dict, Optional

import torch

_PLAN_FILE = Path(__file__).with_name("plans.json")

_DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}
_DTYPE_NAMES = {v: k for k, v in _DTYPES.items()}

# A whole-forward graph costs one copy-in and one clone-out of the activations;
# above this input size that copy is no longer free (reference: plans.py:107-110).
GRAPH_MAX_INPUT_BYTES = 64 * 1024 * 1024


@dataclass(frozen=True)
class Plan:
    """Execution knobs for one (shape, dtype) combination."""

    # Tensor-core input type of every GEMM and of attention (fp32 accumulate).
    compute_dtype: torch.dtype = torch.float16
    # Precision the residual stream is kept in (always fp32 here).
    residual_dtype: torch.dtype = torch.float32
    # Precision of the attention-output and FFN-output deltas that the next
    # add+LayerNorm folds into the fp32 residual: float32, or a 16-bit type,
    # which means the compute dtype.  16-bit deltas cut the LayerNorm and
    # GEMM-output traffic by 4 bytes per element (measured +2-4% tokens/s at
    # configs 2-3) and moved the config-4 budget usage from 0.16 to 0.19.
    delta_dtype: torch.dtype = torch.float16
    # Whole-forward CUDA graph replay.
    cuda_graph: bool = True
    # Skip the GEMM / LayerNorm work of 128-row tiles that hold only padding
    # (prefix masks); padded rows still come out exactly zero.
    skip_padding: bool = True
    # Run the FFN as one kernel whose hidden tile never reaches HBM
    # (tjb_ffn_fused, d_model <= 1024) instead of two GEMM launches through a
    # hidden scratch.  Off by default: measured 2.2x slower on B200 at
    # d_model 1024 (its shared-memory hidden chunk leaves room for only a
    # 3-stage operand ring).
    ffn_single_kernel: bool = False
    # Hand attention work items out from a device counter (heaviest causal
    # rows first) instead of a fixed stride over the CTAs, so that ragged
    # prefix lengths do not leave SMs idle.
    attn_dynamic: bool = True
    # Give the GEMMs a workspace for stream-K (tjb_gemm_bias_tiles_ws): when a
    # long-K GEMM's last wave of tiles would leave at least three quarters of
    # the SMs idle, every CTA takes an equal run of k-blocks and split tiles
    # meet in the workspace.  The kernel decides per launch from the live
    # tile count; shapes outside that window run unchanged.
    gemm_stream_k: bool = True
    # Run the out-projection and FFN-out GEMMs with the residual add and the
    # next LayerNorm in their epilogue (tjb_gemm_add_layernorm; d_model 256,
    # 512, 768 or 1024), so their outputs never reach HBM and those
    # LayerNorms need no pass of their own.  Off by default; on, for the
    # out-projection only, in the tuned plan of the B8 S1024 shape (0.7 %;
    # fusing its FFN-out too is 4 % slower, since that GEMM needs stream-K
    # for its K = 4096 tail wave).  The B4 S4096 plan keeps its LayerNorms
    # standalone: with CTA-pair GEMMs and the persistent LayerNorm kernel the
    # fused form no longer wins there.  Slower where the GEMM has too few
    # 128 x 256 tiles (B1 S64: one row block, three CTAs).
    fuse_layernorm: bool = False
    # With fuse_layernorm: also fuse the FFN-out GEMM (False keeps it on the
    # plain GEMM, with stream-K, and a standalone add+LayerNorm after it).
    fuse_layernorm_ffn: bool = True
    # Run the whole forward as one persistent cooperative kernel
    # (tjb_forward_small: at most 256 tokens, sequences of at most 128,
    # head_dim 64, fp16) instead of a launch per op: phases separated by grid
    # barriers, weight-streaming GEMMs with the weights on the MMA's M side
    # and split-K for the narrow ones.  On in the tuned plan of B1 S64 d768
    # (3 % faster than the per-op graph); slower at B2 S128 d512.
    whole_forward: bool = False
    label: str = "default"

    def to_json(self) -> Dict[str, object]:
        return {
            "compute_dtype": _DTYPE_NAMES[self.compute_dtype],
            "residual_dtype": _DTYPE_NAMES[self.residual_dtype],
            "delta_dtype": _DTYPE_NAMES[self.delta_dtype],
            "cuda_graph": self.cuda_graph,
            "skip_padding": self.skip_padding,
            "ffn_single_kernel": self.ffn_single_kernel,
            "attn_dynamic": self.attn_dynamic,
            "gemm_stream_k": self.gemm_stream_k,
            "fuse_layernorm": self.fuse_layernorm,
            "fuse_layernorm_ffn": self.fuse_layernorm_ffn,
            "whole_forward": self.whole_forward,
            "label": self.label,
        }

    @staticmethod
    def from_json(blob: Dict[str, object]) -> "Plan":
        blob = dict(blob)
        for key, default in (("compute_dtype", "float16"), ("residual_dtype", "float32"),
                             ("delta_dtype", "float16")):
            blob[key] = _DTYPES[str(blob.get(key, default))]
        # "gemm_split_tail" named an earlier, slower split of the last wave;
        # plans that carry it take the stream-K default.
        blob.pop("gemm_split_tail", None)
        fields = Plan.__dataclass_fields__.keys()
        return Plan(**{k: v for k, v in blob.items() if k in fields})


def shape_key(batch: int, seq: int, d_model: int, heads: int, ffn_dim: int, layers: int,
              causal: bool, dtype: torch.dtype) -> str:
    return (f"b{batch}_s{seq}_d{d_model}_h{heads}_f{ffn_dim}_l{layers}"
            f"_{'causal' if causal else 'full'}_{_DTYPE_NAMES[dtype]}")


def default_plan(batch: int, seq: int, d_model: int, heads: int, ffn_dim: int, layers: int,
                 causal: bool, dtype: torch.dtype, device: torch.device) -> Plan:
    """Heuristic plan used when no tuned plan exists for the shape."""
    if device.type != "cuda":
        raise RuntimeError("tjkernels runs on CUDA (sm_100) devices only; no CPU fallback")
    # fp16 and bf16 run at the same tensor-core rate on sm_100; fp16 keeps 3
    # more mantissa bits, which the per-element budget needs at d_model 4096 /
    # 12 layers (bf16 measured 1.2x over budget there).  LayerNorm bounds
    # every activation, so the fp16 range is never approached.
    compute = dtype if dtype in (torch.float16, torch.bfloat16) else torch.float16
    x_bytes = batch * seq * d_model * torch.empty((), dtype=dtype).element_size()
    return Plan(
        compute_dtype=compute,
        residual_dtype=torch.float32,
        delta_dtype=compute,
        cuda_graph=x_bytes <= GRAPH_MAX_INPUT_BYTES,
        label="heuristic",
    )


_cache: Optional[Dict[str, Plan]] = None
_override: Optional[Plan] = None


def set_override(plan: Optional[Plan]) -> None:
    """Force one plan regardless of shape (tests, tuning)."""
    global _override
    _override = plan


def has_override() -> bool:
    return _override is not None


def _load_tuned() -> Dict[str, Plan]:
    global _cache
    if _cache is None:
        _cache = {}
        if _PLAN_FILE.exists() and os.environ.get("TJ_IGNORE_PLANS") != "1":
            raw = json.loads(_PLAN_FILE.read_text())
            _cache = {k: Plan.from_json(v) for k, v in raw.items()}
    return _cache


def select_plan(batch: int, seq: int, d_model: int, heads: int, ffn_dim: int, layers: int,
                causal: bool, dtype: torch.dtype, device: torch.device) -> Plan:
    if _override is not None:
        return _override
    key = shape_key(batch, seq, d_model, heads, ffn_dim, layers, causal, dtype)
    plan = _load_tuned().get(key)
    if plan is None:
        plan = default_plan(batch, seq, d_model, heads, ffn_dim, layers, causal, dtype, device)
    if os.environ.get("TJ_NO_GRAPH") == "1":
        plan = replace(plan, cuda_graph=False)
    forced = os.environ.get("TJ_COMPUTE_DTYPE")
    if forced in ("float16", "bfloat16"):
        plan = replace(plan, compute_dtype=_DTYPES[forced])
    if os.environ.get("TJ_FFN_SINGLE_KERNEL") == "1":
        plan = replace(plan, ffn_single_kernel=True)
    if os.environ.get("TJ_NO_SKIP") == "1":
        plan = replace(plan, skip_padding=False)
    if os.environ.get("TJ_ATTN_STATIC") == "1":
        plan = replace(plan, attn_dynamic=False)
    if os.environ.get("TJ_NO_STREAM_K") == "1":
        plan = replace(plan, gemm_stream_k=False)
    if os.environ.get("TJ_FUSE_LN") in ("0", "1"):
        plan = replace(plan, fuse_layernorm=os.environ["TJ_FUSE_LN"] == "1")
    if os.environ.get("TJ_FUSE_LN_FFN") in ("0", "1"):
        plan = replace(plan, fuse_layernorm_ffn=os.environ["TJ_FUSE_LN_FFN"] == "1")
    if os.environ.get("TJ_WHOLE_FORWARD") in ("0", "1"):
        plan = replace(plan, whole_forward=os.environ["TJ_WHOLE_FORWARD"] == "1")
    forced = os.environ.get("TJ_DELTA_DTYPE")
    if forced in _DTYPES:
        plan = replace(plan, delta_dtype=_DTYPES[forced])
    return plan


def save_plans(plans: Dict[str, Plan], path: Path = _PLAN_FILE) -> None:
    path.write_text(json.dumps({k: v.to_json() for k, v in plans.items()}, indent=2) + "\n")
    global _cache
    _cache = None

"""Execution engine: packs weights once, then runs the forward on sm_100a.

Same public surface and contract as the reference's ``tjkernels/engine.py``:
``forward(module, x, valid_token_mask)`` (:317-324), ``get_engine`` (:303-309),
``reset_engines`` (:312-314), an ``Engine`` that reads the parameters off the
baseline module instead of owning them (:1-7, :58-79), packs them per plan
(:83-127), and runs the per-layer loop with the deferred residual (:205-269),
optionally replayed as a CUDA graph (:273-300).

Per layer (T = B*S tokens, residual stream fp32 [T, d]):

    res, h  = add_layernorm(res, pending, ln1)      # pending = last FFN delta
    qkv     = gemm(h, Wqkv) + bqkv                   # [T, 3d] -> [B,S,3,H,hd]
    ctx     = attention(qkv)                         # [T, d], causal, in place
    attn    = gemm(ctx, Wo) + bo                     # delta (compute dtype by default)
    res, h2 = add_layernorm(res, attn, ln2)
    pending = ffn(h2)                                # delta
    out     = add_layernorm(res, pending, final_ln)  # padded rows -> exact 0

Padding masks are classified on the device (``tjb_mask_lengths``): no host
synchronisation at all, unlike the reference's memoised ``.item()`` calls
(:131-158).  A prefix mask lets attention skip query tiles past a sequence's
length and stop keys at it; any other mask is applied key by key inside the
attention kernel (the reference routed that case to SDPA with a bias).
Padded rows never influence valid rows (row-wise ops, masked keys), so they
are zeroed once, by the final LayerNorm -- and with a prefix mask the
LayerNorms and GEMMs skip every 128-row tile that holds no row attention can
read (``tjb_row_tiles``; plan knob ``skip_padding``), so a half-padded batch
costs about half the work.
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from .graphs import GraphCache
from . import plans
from .plans import Plan, select_plan
from . import kernels as K


@dataclass
class LayerWeights:
    """Packed weights of one block, in nn.Linear ``[out, in]`` layout."""

    ln1_w: torch.Tensor
    ln1_b: torch.Tensor
    ln1_eps: float
    wqkv: torch.Tensor   # [3d, d]  rows: q | k | v
    bqkv: torch.Tensor   # [3d] fp32
    wo: torch.Tensor     # [d, d]
    bo: torch.Tensor     # [d] fp32
    ln2_w: torch.Tensor
    ln2_b: torch.Tensor
    ln2_eps: float
    w1: torch.Tensor     # [F, d]
    b1: torch.Tensor     # [F] fp32
    w2: torch.Tensor     # [d, F]
    b2: torch.Tensor     # [d] fp32


def padded_head_dim(hd: int) -> int:
    """The head_dim the attention kernel runs a head of ``hd`` at: 64 or 128
    (heads past 128 are left as they are and rejected by the kernel)."""
    if hd <= 64:
        return 64
    if hd <= 128:
        return 128
    return hd


def pad_heads(t: torch.Tensor, width: int, dim: int) -> torch.Tensor:
    """Zero-pad dimension ``dim`` of ``t`` (one head's features) to ``width``."""
    if t.shape[dim] == width:
        return t
    shape = list(t.shape)
    shape[dim] = width - t.shape[dim]
    return torch.cat([t, t.new_zeros(shape)], dim=dim)


class Engine:
    def __init__(self, module: torch.nn.Module) -> None:
        cfg = module.config
        param = next(module.parameters())
        self.device = param.device
        self.dtype = param.dtype
        self.d_model = cfg.d_model
        self.num_heads = cfg.num_heads
        self.head_dim = cfg.d_model // cfg.num_heads
        self.ffn_dim = cfg.ffn_dim
        self.num_layers = cfg.num_layers
        self.causal = cfg.causal
        self.scale = self.head_dim ** -0.5
        # The attention kernel runs head_dim 64 or 128.  A smaller head (the
        # reference's d=128/H=4 correctness shape has 32), or one between 64
        # and 128, is stored zero-padded to the next of the two: the padded
        # Q/K columns add nothing to the scores, the padded V columns make
        # zero context columns, and the out-projection ignores them (zero
        # weight columns); the softmax scale stays 1/sqrt(real head_dim).
        self.head_dim_run = padded_head_dim(self.head_dim)

        self.plan: Optional[Plan] = None
        self._plan_cache: Dict[Tuple[int, int], Plan] = {}
        self._built_for: Optional[Tuple] = None
        self.layers: List[LayerWeights] = []
        self.final_ln: Optional[Tuple[torch.Tensor, torch.Tensor, float]] = None
        self._module = module
        self._graphs = GraphCache()
        # Tensor-parallel layout (parallel.enable_tensor_parallel): this rank
        # keeps num_heads/W heads and ffn_dim/W FFN columns; the partial
        # outputs of the out-projection and FFN-out are all-reduced.
        self._tp = getattr(module, "_tj_tp", None)
        # Work counter of the dynamic attention schedule: zero between calls
        # (each launch returns it to zero), reused by every layer in order.
        self._attn_sched: Optional[torch.Tensor] = None
        # Split-K workspace of the GEMMs, shared by all of them in order.
        self._gemm_ws: Optional[torch.Tensor] = None
        self._ln_ws: Optional[torch.Tensor] = None
        # Workspaces that a larger row count has superseded: captured graphs
        # of the smaller shapes still point at them, so they live until those
        # graphs are released.
        self._ln_ws_retired: List[torch.Tensor] = []
        # Whole-forward kernel (plan.whole_forward): its block pointer table
        # and one workspace per (batch, seq, device).
        self._small: Optional[K.SmallModel] = None
        self._small_ws: Dict[Tuple[int, int, torch.device], torch.Tensor] = {}
        # Pinned host word that every forward ends by copying the device
        # status word into (stream-ordered, no host synchronisation; part of
        # the captured graph too).  The next call reads it: non-zero means a
        # kernel's bounded wait ran out, which can leave the workspaces above
        # mid-update, so they are zeroed again and the call raises.
        self._status_host: Optional[torch.Tensor] = None

    # ---------------------------------------------------------------- weights

    def _build(self, plan: Plan) -> None:
        """Pack weights for ``plan``; once per (compute dtype, model dtype, device)."""
        key = (plan.compute_dtype, self.dtype, self.device)
        if self._built_for == key:
            return
        cdt = plan.compute_dtype
        layers: List[LayerWeights] = []
        if self._tp is not None:
            self._build_tp(plan)
            return
        heads, hd, hdr = self.num_heads, self.head_dim, self.head_dim_run
        with torch.no_grad():
            for block in self._module.layers:
                attn = block.attention
                wqkv = torch.cat([attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight],
                                 dim=0)
                bqkv = torch.cat([attn.q_proj.bias, attn.k_proj.bias, attn.v_proj.bias], dim=0)
                wo = attn.out_proj.weight
                if hdr != hd:
                    wqkv = pad_heads(wqkv.view(3 * heads, hd, -1), hdr, dim=1).reshape(
                        3 * heads * hdr, -1)
                    bqkv = pad_heads(bqkv.view(3 * heads, hd), hdr, dim=1).reshape(-1)
                    wo = pad_heads(wo.view(wo.shape[0], heads, hd), hdr, dim=2).reshape(
                        wo.shape[0], heads * hdr)
                layers.append(LayerWeights(
                    ln1_w=block.norm1.weight.float().contiguous(),
                    ln1_b=block.norm1.bias.float().contiguous(),
                    ln1_eps=block.norm1.eps,
                    wqkv=wqkv.to(cdt).contiguous(),
                    bqkv=bqkv.float().contiguous(),
                    wo=wo.to(cdt).contiguous(),
                    bo=attn.out_proj.bias.float().contiguous(),
                    ln2_w=block.norm2.weight.float().contiguous(),
                    ln2_b=block.norm2.bias.float().contiguous(),
                    ln2_eps=block.norm2.eps,
                    w1=block.ffn_in.weight.to(cdt).contiguous(),
                    b1=block.ffn_in.bias.float().contiguous(),
                    w2=block.ffn_out.weight.to(cdt).contiguous(),
                    b2=block.ffn_out.bias.float().contiguous(),
                ))
            fn = self._module.final_norm
            self.final_ln = (fn.weight.float().contiguous(), fn.bias.float().contiguous(),
                             fn.eps)
        self.layers = layers
        self._attn_sched = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._gemm_ws = K.gemm_workspace(self.device)
        self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._built_for = key
        self._small = None
        self._graphs.clear()
        self._ln_ws_retired.clear()

    def _build_tp(self, plan: Plan) -> None:
        """This rank's slice of every block (tensor-parallel layout); the
        row-parallel biases stay on rank 0 only (zero elsewhere)."""
        from .parallel import tp_shard

        _, rank, world = self._tp
        if self.head_dim_run != self.head_dim:
            raise RuntimeError("tensor parallelism needs head_dim 64 or 128")
        cdt = plan.compute_dtype
        layers: List[LayerWeights] = []
        with torch.no_grad():
            for block in self._module.layers:
                w = tp_shard(block, rank, world)
                keep = 1.0 if rank == 0 else 0.0
                layers.append(LayerWeights(
                    ln1_w=block.norm1.weight.float().contiguous(),
                    ln1_b=block.norm1.bias.float().contiguous(),
                    ln1_eps=block.norm1.eps,
                    wqkv=w["wqkv"].to(cdt).contiguous(),
                    bqkv=w["bqkv"].float().contiguous(),
                    wo=w["wo"].to(cdt).contiguous(),
                    bo=(w["bo"].float() * keep).contiguous(),
                    ln2_w=block.norm2.weight.float().contiguous(),
                    ln2_b=block.norm2.bias.float().contiguous(),
                    ln2_eps=block.norm2.eps,
                    w1=w["w1"].to(cdt).contiguous(),
                    b1=w["b1"].float().contiguous(),
                    w2=w["w2"].to(cdt).contiguous(),
                    b2=(w["b2"].float() * keep).contiguous(),
                ))
            fn = self._module.final_norm
            self.final_ln = (fn.weight.float().contiguous(), fn.bias.float().contiguous(),
                             fn.eps)
        self.layers = layers
        self._attn_sched = torch.zeros(2, dtype=torch.int32, device=self.device)
        self._gemm_ws = K.gemm_workspace(self.device)
        self._status_host = torch.zeros(1, dtype=torch.int32).pin_memory()
        self._built_for = (plan.compute_dtype, self.dtype, self.device)
        self._graphs.clear()
        self._ln_ws_retired.clear()

    # ---------------------------------------------------------------- compute

    def _forward_impl(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        plan = self.plan
        assert plan is not None and self.final_ln is not None
        batch, seq, d = x.shape
        tokens = batch * seq
        heads, hd = self.num_heads, self.head_dim_run
        tp_on = self._tp is not None  # (the group itself may be None: the world)
        tp_group = None
        if tp_on:
            import torch.distributed as dist
            tp_group, _, tp_world = self._tp
            heads //= tp_world

        if (plan.whole_forward and not tp_on and self.head_dim == hd
                and abs(self.scale - hd ** -0.5) < 1e-12
                and K.forward_small_supports(batch, seq, d, heads, self.layers[0].w1.shape[0],
                                             len(self.layers), hd, plan.compute_dtype)):
            return self._forward_whole(x, mask)

        mask_u8 = lengths = flags = tiles = None
        if mask is not None:
            mask_u8 = mask.contiguous().view(torch.uint8) if mask.dtype == torch.bool \
                else (mask != 0).to(torch.uint8)
            if plan.skip_padding:
                lengths, flags, tiles = K.mask_lengths_tiles(mask_u8)
            else:
                lengths, flags = K.mask_lengths(mask_u8)

        res = x.reshape(tokens, d)
        if res.dtype != torch.float32 or not res.is_contiguous():
            res = res.float().contiguous()
        own_res = res.data_ptr() != x.data_ptr()
        # With tensor parallelism the deltas are the per-rank partial sums the
        # all-reduce adds; they travel in the delta dtype too (16-bit by
        # default: half the bytes of fp32 on NVLink).
        delta_dtype = torch.float32 if plan.delta_dtype == torch.float32 else plan.compute_dtype
        ws = self._gemm_ws if plan.gemm_stream_k else None
        if (plan.fuse_layernorm and not tp_on and K.gemm_add_layernorm_supports(d)
                and plan.compute_dtype in (torch.float16, torch.bfloat16)):
            return self._forward_fused_ln(x, res, own_res, tiles, lengths, mask_u8, flags,
                                          heads, hd, ws).view(batch, seq, d)
        pending: Optional[torch.Tensor] = None
        for lw in self.layers:
            res, h = K.fused_add_layernorm(
                res, pending, lw.ln1_w, lw.ln1_b, lw.ln1_eps, out_dtype=plan.compute_dtype,
                residual_out=res if (own_res and pending is not None) else None,
                m_tiles=tiles)
            own_res = own_res or pending is not None
            qkv = K.gemm_bias(h, lw.wqkv, lw.bqkv, m_tiles=tiles, workspace=ws)
            ctx = K.flash_attention(qkv.view(batch, seq, 3, heads, hd), heads,
                                    causal=self.causal, lengths=lengths, key_mask=mask_u8,
                                    mask_flags=flags, scale=self.scale,
                                    sched=self._attn_sched if plan.attn_dynamic else None,
                                    skip_dead_rows=tiles is not None)
            attn_out = K.gemm_bias(ctx, lw.wo, lw.bo, out_dtype=delta_dtype, m_tiles=tiles,
                                   workspace=ws)
            if tp_on:
                dist.all_reduce(attn_out, group=tp_group)
            res, h2 = K.fused_add_layernorm(
                res, attn_out, lw.ln2_w, lw.ln2_b, lw.ln2_eps, out_dtype=plan.compute_dtype,
                residual_out=res if own_res else None, m_tiles=tiles)
            own_res = True
            if (plan.ffn_single_kernel and not tp_on and
                    K.ffn_fused_supports(d, self.ffn_dim)):
                pending = K.ffn_single_kernel(h2, lw.w1, lw.b1, lw.w2, lw.b2,
                                              out_dtype=delta_dtype, m_tiles=tiles)
            else:
                pending = K.fused_ffn(h2, lw.w1, lw.b1, lw.w2, lw.b2, out_dtype=delta_dtype,
                                      m_tiles=tiles, workspace=ws)
            if tp_on:
                dist.all_reduce(pending, group=tp_group)

        fw, fb, feps = self.final_ln
        _, out = K.fused_add_layernorm(res, pending, fw, fb, feps, out_dtype=self.dtype,
                                       write_residual=False, row_mask=mask_u8)
        return out.view(batch, seq, d)

    def _forward_whole(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        """The whole forward as one launch (tjb_forward_small)."""
        batch, seq, d = x.shape
        valid = None
        if mask is not None:
            valid = mask.contiguous().view(torch.uint8) if mask.dtype == torch.bool \
                else (mask != 0).to(torch.uint8)
        xf = x if (x.dtype == torch.float32 and x.is_contiguous()) else x.float().contiguous()
        ffn = self.layers[0].w1.shape[0]
        if self._small is None:
            self._small = K.SmallModel(self.layers, self.final_ln)
        key = (batch, seq, x.device)
        ws = self._small_ws.get(key)
        if ws is None:
            ws = self._small_ws[key] = K.forward_small_workspace(batch, seq, d, ffn, x.device)
        out = K.forward_small(self._small, xf, valid, self.num_heads, ffn, self.causal, ws)
        return out if out.dtype == self.dtype else out.to(self.dtype)

    def _forward_fused_ln(self, x, res, own_res, tiles, lengths, mask_u8, flags, heads, hd,
                          ws) -> torch.Tensor:
        """The same block sequence with LayerNorms inside the GEMM that
        produces their input (tjb_gemm_add_layernorm): out-projection ->
        res += attention out, h2 = LN2(res); with ``plan.fuse_layernorm_ffn``
        also FFN-out -> res += FFN out, h = LN1 of the next block (or the
        final LayerNorm, which writes the output and zeroes padded rows);
        without it the FFN runs as in the plain sequence (stream-K GEMMs) and
        its add+LayerNorm stays a launch of its own."""
        plan = self.plan
        batch, seq, d = x.shape
        cdt = plan.compute_dtype
        delta_dtype = torch.float32 if plan.delta_dtype == torch.float32 else cdt
        layers = self.layers
        lw0 = layers[0]
        res, h = K.fused_add_layernorm(res, None, lw0.ln1_w, lw0.ln1_b, lw0.ln1_eps,
                                       out_dtype=cdt, m_tiles=tiles)
        ln_ws = self._ln_workspace(batch * seq, d, x.device)
        pending: Optional[torch.Tensor] = None
        out = None
        for i, lw in enumerate(layers):
            if pending is not None:
                res, h = K.fused_add_layernorm(res, pending, lw.ln1_w, lw.ln1_b, lw.ln1_eps,
                                               out_dtype=cdt, residual_out=res, m_tiles=tiles)
            qkv = K.gemm_bias(h, lw.wqkv, lw.bqkv, m_tiles=tiles, workspace=ws)
            ctx = K.flash_attention(qkv.view(batch, seq, 3, heads, hd), heads,
                                    causal=self.causal, lengths=lengths, key_mask=mask_u8,
                                    mask_flags=flags, scale=self.scale,
                                    sched=self._attn_sched if plan.attn_dynamic else None,
                                    skip_dead_rows=tiles is not None)
            # The first write goes to a fresh buffer unless the residual is
            # already private (it may be the caller's input).
            res, h2 = K.gemm_add_layernorm(ctx, lw.wo, lw.bo, res, lw.ln2_w, lw.ln2_b,
                                           lw.ln2_eps, out_dtype=cdt,
                                           residual_out=res if own_res else None,
                                           m_tiles=tiles, workspace=ln_ws)
            own_res = True
            if not plan.fuse_layernorm_ffn:
                pending = K.fused_ffn(h2, lw.w1, lw.b1, lw.w2, lw.b2, out_dtype=delta_dtype,
                                      m_tiles=tiles, workspace=ws)
                continue
            hidden = K.gemm_bias(h2, lw.w1, lw.b1, act=K.ACT_GELU, m_tiles=tiles, workspace=ws)
            if i + 1 < len(layers):
                nxt = layers[i + 1]
                res, h = K.gemm_add_layernorm(hidden, lw.w2, lw.b2, res, nxt.ln1_w, nxt.ln1_b,
                                              nxt.ln1_eps, out_dtype=cdt, residual_out=res,
                                              m_tiles=tiles, workspace=ln_ws)
            else:
                fw, fb, feps = self.final_ln
                # Tiles the list skips are all padding: their output rows stay
                # zero; inside listed tiles the row mask zeroes padded rows.
                alloc = torch.zeros if tiles is not None else torch.empty
                _, out = K.gemm_add_layernorm(hidden, lw.w2, lw.b2, res, fw, fb, feps,
                                              out_dtype=self.dtype, write_residual=False,
                                              row_mask=mask_u8, m_tiles=tiles, workspace=ln_ws,
                                              out=alloc((batch * seq, d), dtype=self.dtype,
                                                        device=x.device))
        if pending is not None:
            fw, fb, feps = self.final_ln
            _, out = K.fused_add_layernorm(res, pending, fw, fb, feps, out_dtype=self.dtype,
                                           write_residual=False, row_mask=mask_u8)
        return out

    def _ln_workspace(self, rows: int, d: int, device: torch.device) -> torch.Tensor:
        """The row-statistics workspace of tjb_gemm_add_layernorm, kept for the
        largest row count seen (the kernels of one forward run in order).  A
        workspace that a larger one replaces is kept alive, not freed: graphs
        captured with it would otherwise replay into reused memory."""
        ws = self._ln_ws
        if ws is None or ws.device != device or ws.numel() < K.gemm_add_layernorm_workspace_bytes(
                rows, d):
            if ws is not None:
                self._ln_ws_retired.append(ws)
            self._ln_ws = ws = K.gemm_add_layernorm_workspace(rows, d, device)
        return ws

    def _forward_reported(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        """The forward followed by the stream-ordered status snapshot."""
        out = self._forward_impl(x, mask)
        K.device_status_async(self._status_host, self.device)
        return out

    # ----------------------------------------------------------------- status

    def check_status(self, synchronize: bool = True) -> None:
        """Raise ``KernelError`` (TJB_ERR_DEVICE_TIMEOUT) if a kernel of an
        earlier forward recorded that one of its bounded device-side waits
        ran out.  Every call does this check without synchronising (it sees
        the forwards that have finished by then); ``synchronize=True`` waits
        for all of them first."""
        if self._status_host is None:
            return
        if synchronize:
            torch.cuda.synchronize(self.device)
        if int(self._status_host[0]) != 0:
            self._recover()

    def _recover(self) -> None:
        """After a device-side timeout: clear the device status word, zero
        every workspace a kernel may have left mid-update (row-statistics
        counters, stream-K counters, the attention work counter) and raise."""
        from ._lib import KernelError

        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            status = K.device_status(clear=True) or int(self._status_host[0])
            for ws in (self._gemm_ws, self._ln_ws, self._attn_sched, *self._ln_ws_retired,
                       *self._small_ws.values()):
                if ws is not None:
                    ws.zero_()
            torch.cuda.synchronize(self.device)
        self._status_host.zero_()
        raise KernelError("tjkernels forward", status,
                          "a device-side wait of an earlier forward ran out (its output is "
                          "not valid); workspaces re-zeroed, the next call runs normally")

    # ------------------------------------------------------------------- call

    def __call__(self, x: torch.Tensor, mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if not x.is_cuda:
            raise RuntimeError("tjkernels runs on CUDA (sm_100) tensors only; no CPU fallback")
        self.check_status(synchronize=False)
        batch, seq, _ = x.shape
        plan = None if plans.has_override() else self._plan_cache.get((batch, seq))
        if plan is None:
            plan = select_plan(batch, seq, self.d_model, self.num_heads, self.ffn_dim,
                               self.num_layers, self.causal, self.dtype, self.device)
            if not plans.has_override():
                self._plan_cache[(batch, seq)] = plan
        self.plan = plan
        self._build(plan)
        if plan.cuda_graph and self._tp is None:
            key = (tuple(x.shape), x.dtype, mask is not None, plan)
            return self._graphs.get(key, self._forward_reported, x, mask).run(x, mask)
        return self._forward_reported(x, mask)


def get_engine(module: torch.nn.Module) -> Engine:
    engine = getattr(module, "_tj_engine", None)
    param = next(module.parameters())
    if engine is None or engine.dtype != param.dtype or engine.device != param.device:
        engine = Engine(module)
        object.__setattr__(module, "_tj_engine", engine)
    return engine


def reset_engines(module: torch.nn.Module) -> None:
    if hasattr(module, "_tj_engine"):
        object.__delattr__(module, "_tj_engine")


def forward(module: torch.nn.Module, x: torch.Tensor,
            valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The ``UserOptimizedTransformer.forward`` hook body."""
    if os.environ.get("TJ_DISABLE") == "1":
        return super(type(module), module).forward(x, valid_token_mask)
    return get_engine(module)(x, valid_token_mask)

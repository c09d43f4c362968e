"""Kernel facade: torch tensors in, torch tensors out, sm_100a kernels inside.

Same functions and argument meaning as the reference facade
(``tjkernels/kernels/__init__.py`` in the reference project):
``fused_add_layernorm`` (:48-70), ``layernorm``, ``fused_ffn`` (:80-89) and
``flash_attention`` (``tjkernels/kernels/attention.py:189-226``), plus
``gemm_bias`` (the ``torch.addmm`` calls of ``engine.py:245,247``) and
``mask_lengths`` (the device-side replacement of ``Engine._mask_mode``).

Differences by design: there is no Triton and no torch fallback.  Every call
runs the CUDA library on the tensor's device and current stream; a CPU tensor,
an unsupported shape or dtype raises instead of silently switching backend.
Outputs are allocated here with ``torch.empty`` (the caching allocator, so the
calls capture into CUDA graphs); the library itself never allocates.
"""

from __future__ import annotations

import ctypes

from typing import Optional, Tuple

import torch

from .. import _lib

_CODES = {torch.float32: _lib.TJB_F32, torch.float16: _lib.TJB_F16,
          torch.bfloat16: _lib.TJB_BF16}

ACT_NONE, ACT_GELU = 0, 1


def _code(dtype: torch.dtype) -> int:
    try:
        return _CODES[dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {dtype}") from None


def _need_cuda(*tensors: Optional[torch.Tensor]) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tjkernels runs on CUDA (sm_100) tensors only; no CPU fallback")


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def fused_add_layernorm(
    residual: torch.Tensor,
    delta: Optional[torch.Tensor],
    weight: torch.Tensor,
    bias: torch.Tensor,
    eps: float,
    out_dtype: Optional[torch.dtype] = None,
    write_residual: bool = True,
    row_mask: Optional[torch.Tensor] = None,
    residual_out: Optional[torch.Tensor] = None,
    m_tiles: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """``x = residual + delta``; return ``(x, layernorm(x))``.

    ``residual`` is fp32 ``[rows, d]``; ``delta`` fp32/fp16/bf16 or None.
    With ``write_residual=False`` the sum is not stored and the first result
    is ``residual`` itself.  ``residual_out`` (may alias ``residual``) receives
    the sum instead of a fresh tensor.  Rows with ``row_mask == 0`` (uint8)
    get an exactly-zero normalised output.  With ``m_tiles`` (from
    ``row_tiles``) only the live 128-row tiles are read and written.
    """
    _need_cuda(residual, delta, weight, bias, row_mask)
    if residual.dtype != torch.float32:
        raise TypeError("the residual stream is fp32")
    rows, d = residual.shape
    out_dtype = out_dtype or residual.dtype
    out = torch.empty((rows, d), dtype=out_dtype, device=residual.device)
    res_out = None
    if write_residual and delta is not None:
        res_out = residual_out if residual_out is not None else torch.empty_like(residual)
    if delta is not None and not delta.is_contiguous():
        delta = delta.contiguous()
    status = _lib.lib().tjb_add_layernorm_tiles(
        _ptr(residual), _ptr(delta), _ptr(res_out), _ptr(out), _ptr(weight), _ptr(bias),
        rows, d, float(eps), _code(delta.dtype) if delta is not None else _lib.TJB_F32,
        _code(out_dtype), _ptr(row_mask), _ptr(m_tiles), _stream(residual.device))
    _lib.check(status, "tjb_add_layernorm")
    return (res_out if res_out is not None else residual), out


def layernorm(x, weight, bias, eps, out_dtype=None):
    """Plain LayerNorm over the last dim, emitting ``out_dtype`` directly."""
    return fused_add_layernorm(x, None, weight, bias, eps, out_dtype=out_dtype,
                               write_residual=False)[1]


def gemm_bias(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor],
              act: int = ACT_NONE, out_dtype: Optional[torch.dtype] = None,
              out: Optional[torch.Tensor] = None,
              m_tiles: Optional[torch.Tensor] = None,
              workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``act(a @ w.T + bias)``: a ``[M, K]``, w ``[N, K]`` (nn.Linear layout),
    both fp16 or both bf16; bias fp32 ``[N]``; fp32 accumulation.  With
    ``m_tiles`` only the listed 128-row tiles of the output are computed.
    ``workspace`` (see :func:`gemm_workspace`) lets the kernel use stream-K."""
    _need_cuda(a, w, bias)
    m, k = a.shape
    n, k2 = w.shape
    if k != k2:
        raise ValueError(f"inner dims differ: {k} vs {k2}")
    if a.dtype != w.dtype:
        raise TypeError("a and w must share a dtype")
    out_dtype = out_dtype or a.dtype
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    if workspace is not None:
        status = _lib.lib().tjb_gemm_bias_tiles_ws(
            _ptr(a), _ptr(w), _ptr(bias), _ptr(out), m, n, k, a.stride(0), w.stride(0),
            out.stride(0), _code(a.dtype), _code(out.dtype), act, _ptr(m_tiles),
            _ptr(workspace), workspace.numel() * workspace.element_size(), _stream(a.device))
    else:
        status = _lib.lib().tjb_gemm_bias_tiles(
            _ptr(a), _ptr(w), _ptr(bias), _ptr(out), m, n, k, a.stride(0), w.stride(0),
            out.stride(0), _code(a.dtype), _code(out.dtype), act, _ptr(m_tiles),
            _stream(a.device))
    _lib.check(status, "tjb_gemm_bias")
    return out


def gemm_add_layernorm(a: torch.Tensor, w: torch.Tensor, bias: torch.Tensor,
                       residual: torch.Tensor, weight: torch.Tensor, ln_bias: torch.Tensor,
                       eps: float, out_dtype: Optional[torch.dtype] = None,
                       residual_out: Optional[torch.Tensor] = None, write_residual: bool = True,
                       row_mask: Optional[torch.Tensor] = None,
                       m_tiles: Optional[torch.Tensor] = None,
                       out: Optional[torch.Tensor] = None,
                       workspace: Optional[torch.Tensor] = None
                       ) -> Tuple[Optional[torch.Tensor], torch.Tensor]:
    """One kernel for ``residual_out = residual + a @ w.T + bias`` (fp32) and
    ``out = LayerNorm(residual_out) * weight + ln_bias``: the out-projection
    or FFN-out GEMM with the add+LayerNorm that follows it in a pre-LN block.
    ``residual_out`` may be ``residual`` (in place); with ``write_residual``
    False it is not written.  N (= d_model) must be 256, 512, 768 or 1024.
    ``workspace`` (see :func:`gemm_add_layernorm_workspace`) carries the row
    statistics between the tiles of a row block; one is made when it is None.
    Returns ``(residual_out, out)``."""
    _need_cuda(a, w, bias, residual, weight, ln_bias)
    m, k = a.shape
    n, k2 = w.shape
    if k != k2 or residual.shape != (m, n):
        raise ValueError("shape mismatch")
    if a.dtype != w.dtype or residual.dtype != torch.float32:
        raise TypeError("a and w share a 16-bit dtype; the residual is fp32")
    for t in (a, w, residual):
        if not t.is_contiguous():
            raise ValueError("contiguous tensors only")
    out_dtype = out_dtype or a.dtype
    if out is None:
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    elif out.shape != (m, n) or out.dtype != out_dtype or not out.is_contiguous():
        raise ValueError("out must be a contiguous [M, N] tensor of out_dtype")
    if write_residual and residual_out is None:
        residual_out = torch.empty_like(residual)
    res_out = residual_out if write_residual else None
    if workspace is None:
        workspace = gemm_add_layernorm_workspace(m, n, a.device)
    status = _lib.lib().tjb_gemm_add_layernorm(
        _ptr(a), _ptr(w), _ptr(bias), _ptr(residual), _ptr(res_out), _ptr(weight),
        _ptr(ln_bias), _ptr(out), m, n, k, float(eps), _code(a.dtype), _code(out_dtype),
        _ptr(row_mask), _ptr(m_tiles), _ptr(workspace),
        workspace.numel() * workspace.element_size(), _stream(a.device))
    _lib.check(status, "tjb_gemm_add_layernorm")
    return res_out, out


def gemm_add_layernorm_supports(d_model: int) -> bool:
    return d_model in (256, 512, 768, 1024)


def gemm_add_layernorm_workspace(rows: int, d_model: int, device: torch.device) -> torch.Tensor:
    """A zeroed workspace for :func:`gemm_add_layernorm` on up to ``rows``
    rows (``tjb_gemm_add_layernorm_workspace_bytes``); calls that may overlap
    on the GPU need separate workspaces."""
    return torch.zeros(gemm_add_layernorm_workspace_bytes(rows, d_model), dtype=torch.uint8,
                       device=device)


def gemm_add_layernorm_workspace_bytes(rows: int, d_model: int) -> int:
    return int(_lib.lib().tjb_gemm_add_layernorm_workspace_bytes(rows, d_model))


def gemm_workspace(device: torch.device) -> torch.Tensor:
    """A zeroed stream-K workspace for :func:`gemm_bias` / :func:`fused_ffn`
    (``tjb_gemm_workspace_bytes`` bytes); calls that may overlap on the GPU
    need separate workspaces."""
    nbytes = int(_lib.lib().tjb_gemm_workspace_bytes())
    return torch.zeros(nbytes, dtype=torch.uint8, device=device)


def fused_ffn(h: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
              b2: torch.Tensor, out_dtype: Optional[torch.dtype] = None,
              m_tiles: Optional[torch.Tensor] = None,
              workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``gelu_erf(h @ w1.T + b1) @ w2.T + b2``; w1 ``[F, d]``, w2 ``[d, F]``;
    with ``m_tiles`` only the listed 128-row tiles are computed; ``workspace``
    lets both GEMMs use stream-K."""
    _need_cuda(h, w1, b1, w2, b2)
    t, d = h.shape
    f = w1.shape[0]
    out_dtype = out_dtype or h.dtype
    out = torch.empty((t, d), dtype=out_dtype, device=h.device)
    hidden = torch.empty((t, f), dtype=h.dtype, device=h.device)
    if workspace is not None:
        status = _lib.lib().tjb_ffn_tiles_ws(
            _ptr(h), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(out), _ptr(hidden), t, d, f,
            _code(h.dtype), _code(out_dtype), _ptr(m_tiles), _ptr(workspace),
            workspace.numel() * workspace.element_size(), _stream(h.device))
    else:
        status = _lib.lib().tjb_ffn_tiles(
            _ptr(h), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(out), _ptr(hidden), t, d, f,
            _code(h.dtype), _code(out_dtype), _ptr(m_tiles), _stream(h.device))
    _lib.check(status, "tjb_ffn")
    return out


def ffn_fused_supports(d_model: int, ffn_dim: int) -> bool:
    """Shapes the single-kernel FFN (hidden kept on chip) handles."""
    c = d_model // 256
    return d_model % 256 == 0 and 1 <= c <= 4 and ffn_dim % (128 * c) == 0


def ffn_single_kernel(h: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
                      b2: torch.Tensor, out_dtype: Optional[torch.dtype] = None,
                      m_tiles: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Same result as ``fused_ffn`` from one kernel whose [T, F] hidden tile
    never reaches HBM (``tjb_ffn_fused``); raises for unsupported shapes."""
    _need_cuda(h, w1, b1, w2, b2)
    t, d = h.shape
    f = w1.shape[0]
    out_dtype = out_dtype or h.dtype
    out = torch.empty((t, d), dtype=out_dtype, device=h.device)
    status = _lib.lib().tjb_ffn_fused(
        _ptr(h), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _ptr(out), t, d, f,
        _code(h.dtype), _code(out_dtype), _ptr(m_tiles), _stream(h.device))
    _lib.check(status, "tjb_ffn_fused")
    return out


def flash_supports(head_dim: int, causal: bool = True) -> bool:
    return head_dim in (64, 128)


def flash_attention(qkv: torch.Tensor, heads: int, causal: bool = True,
                    lengths: Optional[torch.Tensor] = None,
                    key_mask: Optional[torch.Tensor] = None,
                    mask_flags: Optional[torch.Tensor] = None,
                    scale: Optional[float] = None,
                    sched: Optional[torch.Tensor] = None,
                    skip_dead_rows: bool = False) -> torch.Tensor:
    """qkv ``[B, S, 3, H, hd]`` (contiguous) -> out ``[B*S, H*hd]``.

    ``sched``: optional int32 ``[2]`` device tensor, zero, that switches to
    the dynamic work queue (``tjb_flash_fwd_sched``); the kernel leaves it
    zero again.  Calls that may overlap on the GPU need separate tensors.
    ``skip_dead_rows`` (with ``sched`` and a prefix mask): query tiles wholly
    past ``lengths[b]`` are not computed and their rows are left unwritten
    instead of zeroed.
    """
    _need_cuda(qkv, lengths, key_mask, mask_flags, sched)
    b, s, three, h, hd = qkv.shape
    if three != 3 or h != heads:
        raise ValueError("qkv must be [B, S, 3, H, hd]")
    if not qkv.is_contiguous():
        raise ValueError("qkv must be contiguous")
    out = torch.empty((b * s, h * hd), dtype=qkv.dtype, device=qkv.device)
    scale = hd ** -0.5 if scale is None else scale
    if sched is not None:
        if sched.dtype != torch.int32 or sched.numel() < 2:
            raise ValueError("sched must be an int32 tensor of two elements")
        status = _lib.lib().tjb_flash_fwd_sched(
            _ptr(qkv), _ptr(out), b, s, h, hd, float(scale), int(causal), _ptr(lengths),
            _ptr(key_mask), _ptr(mask_flags), _code(qkv.dtype), _ptr(sched),
            int(skip_dead_rows), _stream(qkv.device))
        _lib.check(status, "tjb_flash_fwd_sched")
        return out
    status = _lib.lib().tjb_flash_fwd(
        _ptr(qkv), _ptr(out), b, s, h, hd, float(scale), int(causal), _ptr(lengths),
        _ptr(key_mask), _ptr(mask_flags), _code(qkv.dtype), _stream(qkv.device))
    _lib.check(status, "tjb_flash_fwd")
    return out


def mask_lengths(mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Device-side padding-mask classification, no host sync.

    Returns ``(lengths int32 [B], flags int32 [1])``; ``flags`` is 0 for a
    prefix mask and non-zero otherwise.
    """
    _need_cuda(mask)
    if mask.dtype == torch.bool:
        mask = mask.contiguous().view(torch.uint8)
    b, s = mask.shape
    lengths = torch.empty((b,), dtype=torch.int32, device=mask.device)
    flags = torch.empty((1,), dtype=torch.int32, device=mask.device)
    status = _lib.lib().tjb_mask_lengths(_ptr(mask), b, s, _ptr(lengths), _ptr(flags),
                                         _stream(mask.device))
    _lib.check(status, "tjb_mask_lengths")
    return lengths, flags


def mask_lengths_tiles(mask: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``mask_lengths`` and ``row_tiles`` from one launch (tjb_mask_lengths_tiles):
    ``(lengths, flags, tiles)``, all on the device, no host sync."""
    _need_cuda(mask)
    if mask.dtype == torch.bool:
        mask = mask.contiguous().view(torch.uint8)
    b, s = mask.shape
    lengths = torch.empty((b,), dtype=torch.int32, device=mask.device)
    flags = torch.empty((1,), dtype=torch.int32, device=mask.device)
    tiles = torch.empty((1 + (b * s + 127) // 128,), dtype=torch.int32, device=mask.device)
    status = _lib.lib().tjb_mask_lengths_tiles(_ptr(mask), b, s, _ptr(lengths), _ptr(flags),
                                               _ptr(tiles), _stream(mask.device))
    _lib.check(status, "tjb_mask_lengths_tiles")
    return lengths, flags, tiles


def row_tiles(lengths: Optional[torch.Tensor], flags: Optional[torch.Tensor], batch: int,
              seq: int, device: torch.device) -> torch.Tensor:
    """Device-side list of live 128-row tiles of the [B*S] token axis:
    int32 ``[1 + ceil(B*S/128)]``, element 0 the count (see tjb_row_tiles)."""
    _need_cuda(lengths, flags)
    tiles = torch.empty((1 + (batch * seq + 127) // 128,), dtype=torch.int32, device=device)
    status = _lib.lib().tjb_row_tiles(_ptr(lengths), _ptr(flags), batch, seq, _ptr(tiles),
                                      _stream(device))
    _lib.check(status, "tjb_row_tiles")
    return tiles


def device_status(clear: bool = False) -> int:
    """The device status word (0, or TJB_ERR_DEVICE_TIMEOUT); synchronises."""
    return int(_lib.lib().tjb_device_status(int(clear)))


def device_status_async(dst: torch.Tensor, device: torch.device) -> None:
    """Enqueue, on the current stream of ``device``, a copy of the device
    status word into ``dst`` (a pinned host int32 tensor) that lands once the
    kernels queued before it have finished; no synchronisation, so it may be
    captured at the end of a CUDA graph."""
    if dst.is_cuda or dst.dtype != torch.int32 or not dst.is_pinned():
        raise TypeError("device_status_async writes into a pinned host int32 tensor")
    status = _lib.lib().tjb_device_status_async(_ptr(dst), _stream(device))
    _lib.check(status, "tjb_device_status_async")


# Contract of tjb_forward_small (include/tjb200.h).
SMALL_MAX_TOKENS, SMALL_MAX_SEQ, SMALL_MAX_LAYERS = 256, 128, 12


def forward_small_supports(batch: int, seq: int, d_model: int, heads: int, ffn_dim: int,
                           layers: int, head_dim: int, dtype: torch.dtype) -> bool:
    """Whether tjb_forward_small takes this shape (host check, no device work)."""
    return (dtype == torch.float16 and head_dim == 64 and heads * 64 == d_model
            and batch * seq <= SMALL_MAX_TOKENS and seq <= SMALL_MAX_SEQ
            and 0 < layers <= SMALL_MAX_LAYERS and d_model % 128 == 0 and ffn_dim % 128 == 0
            and d_model <= 1280)


def forward_small_workspace(batch: int, seq: int, d_model: int, ffn_dim: int,
                            device: torch.device) -> torch.Tensor:
    """A zeroed workspace for :func:`forward_small` (its first words hold the
    grid barrier; keep one per stream of calls)."""
    n = int(_lib.lib().tjb_forward_small_workspace_bytes(batch, seq, d_model, ffn_dim))
    return torch.zeros(n, dtype=torch.uint8, device=device)


class SmallModel:
    """The per-block device pointers tjb_forward_small reads (a ctypes array
    of tjb_small_layer), built once from fp16 weights; keeps the tensors it
    points to alive."""

    def __init__(self, layers, final_ln) -> None:
        self._keep = []
        arr = (_lib.SmallLayer * len(layers))()
        for i, lw in enumerate(layers):
            for t in (lw.wqkv, lw.wo, lw.w1, lw.w2):
                if t.dtype != torch.float16 or not t.is_contiguous():
                    raise TypeError("tjb_forward_small takes contiguous fp16 weights")
            fields = dict(wqkv=lw.wqkv, wo=lw.wo, w1=lw.w1, w2=lw.w2, bqkv=lw.bqkv, bo=lw.bo,
                          b1=lw.b1, b2=lw.b2, ln1_w=lw.ln1_w, ln1_b=lw.ln1_b, ln2_w=lw.ln2_w,
                          ln2_b=lw.ln2_b)
            for name, t in fields.items():
                self._keep.append(t)
                setattr(arr[i], name, t.data_ptr())
            arr[i].ln1_eps = float(lw.ln1_eps)
            arr[i].ln2_eps = float(lw.ln2_eps)
        self.layers = arr
        self.count = len(layers)
        # Bytes of parameters one forward streams, and GEMM weights (for FLOP counts).
        self.param_bytes = sum(t.numel() * t.element_size() for t in self._keep)
        self.gemm_params = sum(lw.wqkv.numel() + lw.wo.numel() + lw.w1.numel() + lw.w2.numel()
                               for lw in layers)
        self.lnf_w, self.lnf_b, self.lnf_eps = final_ln
        self._keep += [self.lnf_w, self.lnf_b]
        self.param_bytes += 2 * self.lnf_w.numel() * 4


def forward_small(model: SmallModel, x: torch.Tensor, valid: Optional[torch.Tensor], heads: int,
                  ffn_dim: int, causal: bool, workspace: torch.Tensor,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The whole encoder forward in one launch (tjb_forward_small): ``x`` fp32
    ``[B, S, d]``; ``valid`` uint8 ``[B, S]`` (0 = padded token) or None.
    Returns fp32 ``[B, S, d]`` with padded rows zero."""
    _need_cuda(x, valid, workspace)
    b, s, d = x.shape
    if x.dtype != torch.float32 or not x.is_contiguous():
        raise TypeError("x must be contiguous fp32")
    if valid is not None:
        if valid.dtype == torch.bool:
            valid = valid.contiguous().view(torch.uint8)
        if valid.shape != (b, s) or not valid.is_contiguous():
            raise ValueError("valid must be a contiguous [B, S] mask")
    if out is None:
        out = torch.empty_like(x)
    status = _lib.lib().tjb_forward_small(
        ctypes.addressof(model.layers), model.count, _ptr(model.lnf_w), _ptr(model.lnf_b),
        float(model.lnf_eps), _ptr(x), _ptr(out), _ptr(valid), b, s, d, heads, ffn_dim,
        int(causal), _lib.TJB_F16, _ptr(workspace), workspace.numel(), _stream(x.device))
    _lib.check(status, "tjb_forward_small")
    return out


__all__ = [
    "ACT_NONE", "ACT_GELU", "fused_add_layernorm", "layernorm", "gemm_bias", "gemm_workspace",
    "gemm_add_layernorm_workspace", "gemm_add_layernorm_workspace_bytes",
    "gemm_add_layernorm", "gemm_add_layernorm_supports",
    "fused_ffn",
    "ffn_single_kernel", "ffn_fused_supports",
    "flash_attention", "flash_supports", "mask_lengths", "mask_lengths_tiles", "row_tiles",
    "device_status",
    "device_status_async",
    "forward_small", "forward_small_supports", "forward_small_workspace", "SmallModel",
]

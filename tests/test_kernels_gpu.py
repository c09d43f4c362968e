"""Kernel-level parity of the sm_100a library against fp32/fp64 torch
references (modelled on the reference's bench/test_flash.py:36-48, which
checks flash attention against an fp64 reference).  Calls go through the C
ABI via the tjkernels.kernels facade."""

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(autouse=True, scope="module")
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    yield


def K():
    import tjkernels.kernels as kernels
    return kernels


# ------------------------------------------------------------------ LayerNorm

@pytest.mark.parametrize("rows,d", [(1, 128), (37, 96), (256, 512), (1000, 768),
                                    (513, 1024), (64, 4096), (8, 8192),
                                    # above 1024 rows with d <= 1024: the persistent
                                    # warp-per-row kernel (several rows per warp)
                                    (1025, 1024), (5500, 1024), (2049, 96), (40000, 512)])
@pytest.mark.parametrize("delta_dtype", [None, torch.float32, torch.bfloat16, torch.float16])
def test_add_layernorm(rows, d, delta_dtype):
    g = torch.Generator(device=DEV).manual_seed(rows * 7 + d)
    res = torch.randn(rows, d, device=DEV, generator=g) * 3 + 0.5
    delta = None if delta_dtype is None else \
        torch.randn(rows, d, device=DEV, generator=g).to(delta_dtype)
    w = torch.randn(d, device=DEV, generator=g)
    b = torch.randn(d, device=DEV, generator=g)
    x = res + (0 if delta is None else delta.float())
    ref = F.layer_norm(x, (d,), w, b, 1e-5)
    new_res, out = K().fused_add_layernorm(res, delta, w, b, 1e-5, out_dtype=torch.float32)
    assert (out - ref).abs().max().item() < 1e-4
    if delta is not None:
        assert torch.equal(new_res, x)
    _, out16 = K().fused_add_layernorm(res, delta, w, b, 1e-5, out_dtype=torch.bfloat16)
    assert ((out16.float() - ref).abs() <= 1e-2 * ref.abs() + 1e-2).all()


@pytest.mark.parametrize("rows", [300, 7000])
@pytest.mark.parametrize("delta_dtype", [torch.float32, torch.float16])
def test_add_layernorm_row_mask_and_inplace(rows, delta_dtype):
    d = 1024
    res = torch.randn(rows, d, device=DEV)
    delta = torch.randn(rows, d, device=DEV).to(delta_dtype)
    w, b = torch.randn(d, device=DEV), torch.randn(d, device=DEV)
    mask = (torch.rand(rows, device=DEV) > 0.4).to(torch.uint8)
    expect_res = res + delta.float()
    ref = F.layer_norm(expect_res, (d,), w, b, 1e-5)
    got_res, out = K().fused_add_layernorm(res, delta, w, b, 1e-5, out_dtype=torch.float32,
                                           row_mask=mask, residual_out=res)
    assert got_res.data_ptr() == res.data_ptr()
    assert torch.equal(res, expect_res)
    keep = mask.bool()
    assert (out[~keep] == 0).all()
    assert (out[keep] - ref[keep]).abs().max().item() < 1e-4


# ----------------------------------------------------------------------- GEMM

GEMM_SHAPES = [(1, 64, 64), (64, 2304, 768), (100, 136, 96), (128, 256, 128), (256, 1536, 512),
               (300, 1024, 1024), (1000, 3072, 1024), (2048, 1024, 4096), (4096, 4096, 1024)]


@pytest.mark.parametrize("m,n,k", GEMM_SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemm_bias(m, n, k, dtype):
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    a = torch.randn(m, k, device=DEV, generator=g).to(dtype)
    w = (torch.randn(n, k, device=DEV, generator=g) / math.sqrt(k)).to(dtype)
    bias = torch.randn(n, device=DEV, generator=g)
    ref = a.double() @ w.double().T + bias.double()
    out32 = K().gemm_bias(a, w, bias, out_dtype=torch.float32)
    scale = ref.abs().max().item() + 1e-6
    assert (out32.double() - ref).abs().max().item() <= 1e-5 * scale + 1e-5
    out16 = K().gemm_bias(a, w, bias)
    assert out16.dtype == dtype
    tol = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    assert ((out16.double() - ref).abs() <= tol * ref.abs() + 1e-3 * scale).all()


# Shapes that take the CTA-pair kernel (256 x 256 tiles over two CTAs): an
# odd number of 128-row tiles (the last pair's second CTA has no rows), M
# not a multiple of 128, N not a multiple of 256 (the peer's B half partly or
# wholly past N), several rounds of the persistent grid.
PAIR_SHAPES = [(1000, 3072, 1024), (4096, 4096, 1024), (5504, 3072, 1024), (1151, 2304, 768),
               (3000, 1160, 512), (640, 1408, 1024), (16384, 1024, 256)]


@pytest.mark.parametrize("m,n,k", PAIR_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_gemm_cta_pair(m, n, k, dtype, monkeypatch):
    """The CTA-pair GEMM against fp64 (fp32 and 16-bit output, with GELU), and
    against the single-CTA kernel of the same shape (TJB_GEMM_PAIR=0), which
    does the same products in the same order."""
    g = torch.Generator(device=DEV).manual_seed(m + 3 * n + k)
    a = torch.randn(m, k, device=DEV, generator=g).to(dtype)
    w = (torch.randn(n, k, device=DEV, generator=g) / math.sqrt(k)).to(dtype)
    bias = torch.randn(n, device=DEV, generator=g)
    ref = a.double() @ w.double().T + bias.double()
    scale = ref.abs().max().item() + 1e-6
    monkeypatch.setenv("TJB_GEMM_PAIR", "1")
    for _ in range(2):
        out32 = K().gemm_bias(a, w, bias, out_dtype=torch.float32)
        assert (out32.double() - ref).abs().max().item() <= 1e-5 * scale + 1e-5
    out16 = K().gemm_bias(a, w, bias, act=K().ACT_GELU)
    ref_g = F.gelu(ref, approximate="none")
    tol = 2 ** -7 if dtype == torch.bfloat16 else 2 ** -10
    assert ((out16.double() - ref_g).abs() <= tol * ref_g.abs() + 1e-3 * scale).all()
    monkeypatch.setenv("TJB_GEMM_PAIR", "0")
    single = K().gemm_bias(a, w, bias, out_dtype=torch.float32)
    assert (out32 - single).abs().max().item() <= 1e-6 * scale


@pytest.mark.parametrize("listed", [[0, 2, 3, 7], [1, 4, 6], [5]])
def test_gemm_cta_pair_live_tiles(listed, monkeypatch):
    """With a live-tile list each CTA of a pair takes one listed tile (an odd
    count leaves the last pair's second CTA without rows); unlisted tiles are
    not written."""
    monkeypatch.setenv("TJB_GEMM_PAIR", "1")
    m, n, k = 1000, 2048, 512
    g = torch.Generator(device=DEV).manual_seed(len(listed))
    a = torch.randn(m, k, device=DEV, generator=g).half()
    w = (torch.randn(n, k, device=DEV, generator=g) / 16).half()
    bias = torch.randn(n, device=DEV, generator=g)
    tiles = torch.tensor([len(listed)] + listed + [0] * (8 - len(listed)), dtype=torch.int32,
                         device=DEV)
    out = torch.full((m, n), 7.0, dtype=torch.float32, device=DEV)
    K().gemm_bias(a, w, bias, out_dtype=torch.float32, out=out, m_tiles=tiles)
    ref = a.double() @ w.double().T + bias.double()
    for t in range(8):
        rows = slice(t * 128, min(t * 128 + 128, m))
        if t in listed:
            assert (out[rows].double() - ref[rows]).abs().max().item() < 1e-3
        else:
            assert (out[rows] == 7.0).all()


# Stream-K on CTA pairs for (5120, 1024, 4096), (5376, 1024, 3072), (4480,
# 1032, 4096) (a partial last column tile), (5504, 1024, 4096) (an odd
# number of row tiles: the last pair's second CTA has no rows of its own)
# and (2816, 2048, 4096); its single-CTA small-M form for (64, 768, 3072),
# (128, 1024, 4096) and (100, 200, 2048); the other shapes (among them
# (9600, 1024, 4096): more than two waves) take the whole-tile path with a
# workspace passed.
SPLIT_SHAPES = [(5120, 1024, 1024), (5120, 1024, 4096), (5376, 1024, 3072), (9600, 1024, 4096),
                (4480, 1032, 4096), (5504, 1024, 4096), (2816, 2048, 4096), (64, 768, 3072),
                (128, 1024, 4096), (100, 200, 2048), (4608, 3072, 1024), (300, 136, 512),
                (2000, 1032, 2048), (129, 64, 64)]


@pytest.mark.parametrize("m,n,k", SPLIT_SHAPES)
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16])
def test_gemm_stream_k(m, n, k, out_dtype):
    """Stream-K (equal k-block runs per CTA, split tiles' partials meeting in
    the workspace) matches fp64 and the whole-tile kernel, with GELU and a
    live-tile list too, and leaves the workspace's counters at zero for the
    next call."""
    g = torch.Generator(device=DEV).manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, device=DEV, generator=g).half()
    w = (torch.randn(n, k, device=DEV, generator=g) / math.sqrt(k)).half()
    bias = torch.randn(n, device=DEV, generator=g)
    ws = K().gemm_workspace(DEV)
    flags_at = ws.numel() - 2 * 160 * 4  # two int32 counters per workspace slot
    for act in (K().ACT_NONE, K().ACT_GELU):
        ref = a.double() @ w.double().T + bias.double()
        if act == K().ACT_GELU:
            ref = F.gelu(ref, approximate="none")
        for _ in range(2):
            got = K().gemm_bias(a, w, bias, act=act, out_dtype=out_dtype, workspace=ws)
            whole = K().gemm_bias(a, w, bias, act=act, out_dtype=out_dtype)
            scale = ref.abs().max().item() + 1e-6
            tol = 1e-5 if out_dtype == torch.float32 else 2 ** -10
            assert ((got.double() - ref).abs() <= tol * ref.abs() + 1e-4 * scale).all()
            assert (got.double() - whole.double()).abs().max().item() <= 2e-3 * scale
            assert int(ws[flags_at:].view(torch.int32).abs().sum()) == 0
    # Live-tile list: every other 128-row tile.
    n_tiles = (m + 127) // 128
    live = list(range(0, n_tiles, 2))
    tiles = torch.tensor([len(live)] + live + [0] * (n_tiles - len(live)), dtype=torch.int32,
                         device=DEV)
    out = torch.zeros(m, n, dtype=out_dtype, device=DEV)
    K().gemm_bias(a, w, bias, out_dtype=out_dtype, out=out, m_tiles=tiles, workspace=ws)
    ref = a.double() @ w.double().T + bias.double()
    rows = torch.zeros(m, dtype=torch.bool, device=DEV)
    for t in live:
        rows[t * 128:(t + 1) * 128] = True
    scale = ref.abs().max().item() + 1e-6
    assert ((out.double()[rows] - ref[rows]).abs() <= 2 ** -10 * ref[rows].abs() + 1e-4 * scale).all()
    assert bool((out[~rows] == 0).all())
    assert int(ws[flags_at:].view(torch.int32).abs().sum()) == 0


@pytest.mark.parametrize("m,n,k", [(200, 512, 256), (1024, 4096, 1024)])
def test_gemm_gelu(m, n, k):
    a = torch.randn(m, k, device=DEV).bfloat16()
    w = (torch.randn(n, k, device=DEV) / math.sqrt(k)).bfloat16()
    bias = torch.randn(n, device=DEV)
    ref = F.gelu(a.double() @ w.double().T + bias.double(), approximate="none")
    out = K().gemm_bias(a, w, bias, act=K().ACT_GELU, out_dtype=torch.float32)
    assert (out.double() - ref).abs().max().item() < 1e-4


def test_gemm_no_bias_and_errors():
    a = torch.randn(128, 64, device=DEV).bfloat16()
    w = torch.randn(64, 64, device=DEV).bfloat16()
    out = K().gemm_bias(a, w, None, out_dtype=torch.float32)
    assert (out.double() - a.double() @ w.double().T).abs().max().item() < 1e-3
    from tjkernels._lib import KernelError
    with pytest.raises(KernelError):  # N not a multiple of 8
        K().gemm_bias(a, torch.randn(60, 64, device=DEV).bfloat16(), None)


# ------------------------------------------------------- GEMM + add + LayerNorm

@pytest.mark.parametrize("m,n,k", [(300, 1024, 1024), (129, 256, 512), (1000, 768, 3072),
                                   (64, 512, 256), (2000, 1024, 4096), (8192, 1024, 1024),
                                   (9000, 768, 512)])
@pytest.mark.parametrize("out_dtype", [torch.float16, torch.float32])
def test_gemm_add_layernorm(m, n, k, out_dtype):
    """res + a @ w.T + bias and its LayerNorm in one kernel (row statistics
    exchanged through a workspace) against fp64; in place, with a live-tile
    list and with a row mask; the workspace's counters are zero afterwards."""
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    a = torch.randn(m, k, device=DEV, generator=g).half()
    w = (torch.randn(n, k, device=DEV, generator=g) / math.sqrt(k)).half()
    bias = torch.randn(n, device=DEV, generator=g) * 0.1
    res = torch.randn(m, n, device=DEV, generator=g) * 2 + 0.5
    gamma = 1 + 0.1 * torch.randn(n, device=DEV, generator=g)
    beta = 0.1 * torch.randn(n, device=DEV, generator=g)
    ref_res = res.double() + a.double() @ w.double().T + bias.double()
    ref = F.layer_norm(ref_res, (n,), gamma.double(), beta.double(), eps=1e-5)
    ws = K().gemm_add_layernorm_workspace(m, n, DEV)
    res_out, out = K().gemm_add_layernorm(a, w, bias, res, gamma, beta, 1e-5,
                                          out_dtype=out_dtype, workspace=ws)
    assert (res_out.double() - ref_res).abs().max().item() < 1e-3
    tol = 4e-3 if out_dtype == torch.float16 else 1e-4
    assert (out.double() - ref).abs().max().item() < tol
    # In place, every other 128-row tile live, odd rows masked to zero.
    n_tiles = (m + 127) // 128
    live = list(range(0, n_tiles, 2))
    tiles = torch.tensor([len(live)] + live + [0] * (n_tiles - len(live)), dtype=torch.int32,
                         device=DEV)
    row_mask = (torch.arange(m, device=DEV) % 2 == 0).to(torch.uint8)
    res2 = res.clone()
    _, out2 = K().gemm_add_layernorm(a, w, bias, res2, gamma, beta, 1e-5, out_dtype=out_dtype,
                                     residual_out=res2, row_mask=row_mask, m_tiles=tiles,
                                     workspace=ws)
    counters = ws[:2 * n_tiles * 4].view(torch.int32)
    assert int(counters.abs().sum().item()) == 0
    rows = torch.zeros(m, dtype=torch.bool, device=DEV)
    for t in live:
        rows[t * 128:(t + 1) * 128] = True
    assert (res2.double()[rows] - ref_res[rows]).abs().max().item() < 1e-3
    assert torch.equal(res2[~rows], res[~rows])  # dead tiles untouched
    keep = rows & row_mask.bool()
    assert (out2.double()[keep] - ref[keep]).abs().max().item() < tol
    assert bool((out2[rows & ~row_mask.bool()] == 0).all())


@pytest.mark.parametrize("m,n,k", [(300, 1024, 1024), (9000, 768, 512)])
def test_gemm_add_layernorm_bf16(m, n, k):
    """The bf16-operand form of the fused GEMM + add + LayerNorm against
    fp64 (bf16 output)."""
    g = torch.Generator(device=DEV).manual_seed(7 * m + n)
    a = torch.randn(m, k, device=DEV, generator=g).bfloat16()
    w = (torch.randn(n, k, device=DEV, generator=g) / math.sqrt(k)).bfloat16()
    bias = torch.randn(n, device=DEV, generator=g) * 0.1
    res = torch.randn(m, n, device=DEV, generator=g)
    gamma = 1 + 0.1 * torch.randn(n, device=DEV, generator=g)
    beta = 0.1 * torch.randn(n, device=DEV, generator=g)
    ref_res = res.double() + a.double() @ w.double().T + bias.double()
    ref = F.layer_norm(ref_res, (n,), gamma.double(), beta.double(), eps=1e-5)
    res_out, out = K().gemm_add_layernorm(a, w, bias, res, gamma, beta, 1e-5)
    assert out.dtype == torch.bfloat16
    assert (res_out.double() - ref_res).abs().max().item() < 1e-3
    assert (out.double() - ref).abs().max().item() < 3e-2  # bf16 output rounding


def test_gemm_add_layernorm_rejects_unsupported_width():
    from tjkernels._lib import KernelError
    a = torch.randn(16, 64, device=DEV).half()
    w = torch.randn(2048, 64, device=DEV).half()
    z = torch.zeros(2048, device=DEV)
    with pytest.raises(KernelError):
        K().gemm_add_layernorm(a, w, z, torch.zeros(16, 2048, device=DEV), z + 1, z, 1e-5)


# ------------------------------------------------------------------ attention

def attn_reference(qkv, causal, lengths=None, key_mask=None):
    """fp64 attention over [B,S,3,H,hd] -> [B*S, H*hd] (bench/test_flash.py:36-48)."""
    b, s, _, h, hd = qkv.shape
    q = qkv[:, :, 0].transpose(1, 2).double()
    k = qkv[:, :, 1].transpose(1, 2).double()
    v = qkv[:, :, 2].transpose(1, 2).double()
    scores = (q @ k.transpose(-2, -1)) * hd ** -0.5
    if causal:
        scores = scores.masked_fill(
            torch.ones(s, s, dtype=torch.bool, device=qkv.device).triu(1), float("-inf"))
    if lengths is not None:
        keep = torch.arange(s, device=qkv.device)[None, :] < lengths[:, None]
        scores = scores.masked_fill(~keep[:, None, None, :], float("-inf"))
    if key_mask is not None:
        scores = scores.masked_fill(~key_mask.bool()[:, None, None, :], float("-inf"))
    probs = torch.softmax(scores, dim=-1)
    probs = torch.nan_to_num(probs, nan=0.0)
    return (probs @ v).transpose(1, 2).reshape(b * s, h * hd)


ATTN_CASES = [(1, 1, 1, 64), (2, 37, 2, 64), (2, 128, 4, 64), (1, 200, 2, 128),
              (2, 256, 2, 64), (1, 1000, 2, 64), (1, 513, 1, 128), (2, 2048, 2, 64),
              (1, 1, 1, 128), (3, 300, 4, 128), (2, 2048, 2, 128)]


@pytest.mark.parametrize("b,s,h,hd", ATTN_CASES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_flash_dense(b, s, h, hd, causal, dtype):
    g = torch.Generator(device=DEV).manual_seed(b * 1000 + s + h + hd)
    qkv = torch.randn(b, s, 3, h, hd, device=DEV, generator=g).to(dtype)
    out = K().flash_attention(qkv, h, causal=causal)
    ref = attn_reference(qkv, causal)
    err = (out.double() - ref).abs().max().item()
    assert err < (2e-2 if dtype == torch.bfloat16 else 4e-3), err


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("hd", [64, 128])
def test_flash_growing_scores_rescale(causal, hd):
    """Key norms growing along the sequence push a row's running max up by far
    more than the lazy-rescale threshold several times after the first key
    tile, so the output accumulator is rescaled in tensor memory mid-row."""
    b, s, h = 2, 1000, 2
    g = torch.Generator(device=DEV).manual_seed(31 + hd)
    qkv = torch.randn(b, s, 3, h, hd, device=DEV, generator=g)
    qkv[:, :, 1] *= (1.0 + torch.arange(s, device=DEV) / 64.0).clamp(max=8.0)[None, :, None, None]
    qkv = qkv.half()
    out = K().flash_attention(qkv, h, causal=causal)
    ref = attn_reference(qkv, causal)
    err = (out.double() - ref).abs().max().item()
    assert err < 4e-3, err


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("hd", [64, 128])
def test_flash_prefix_lengths(causal, hd):
    b, s, h = 4, 700, 2
    qkv = torch.randn(b, s, 3, h, hd, device=DEV).bfloat16()
    lengths = torch.tensor([700, 1, 129, 384], dtype=torch.int32, device=DEV)
    mask = torch.arange(s, device=DEV)[None, :] < lengths[:, None]
    lens, flags = K().mask_lengths(mask)
    assert torch.equal(lens, lengths) and int(flags.item()) == 0
    out = K().flash_attention(qkv, h, causal=causal, lengths=lens,
                              key_mask=mask.to(torch.uint8), mask_flags=flags)
    ref = attn_reference(qkv, causal, lengths=lengths)
    valid = mask.reshape(-1)
    assert (out.double()[valid] - ref[valid]).abs().max().item() < 2e-2
    # Query tiles wholly past the length are skipped and written as zeros.
    rows = out.view(b, s, -1)
    assert (rows[1, 128:] == 0).all()
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("hd", [64, 128])
def test_flash_general_key_mask(hd):
    b, s, h = 2, 300, 2
    qkv = torch.randn(b, s, 3, h, hd, device=DEV).bfloat16()
    key_mask = (torch.rand(b, s, device=DEV) > 0.3)
    key_mask[:, 0] = True
    lens, flags = K().mask_lengths(key_mask)
    assert int(flags.item()) != 0
    out = K().flash_attention(qkv, h, causal=True, lengths=lens,
                              key_mask=key_mask.to(torch.uint8), mask_flags=flags)
    ref = attn_reference(qkv, True, key_mask=key_mask)
    assert (out.double() - ref).abs().max().item() < 2e-2
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("mask_kind", ["none", "prefix", "general"])
def test_flash_dynamic_schedule_matches_static(hd, mask_kind):
    """Items handed out from the device counter give the same bits as the
    fixed stride (each item is computed the same way whichever CTA takes it),
    and every launch leaves the counter at zero for the next one."""
    b, s, h = 5, 900, 4
    g = torch.Generator(device=DEV).manual_seed(hd + len(mask_kind))
    qkv = torch.randn(b, s, 3, h, hd, device=DEV, generator=g).half()
    kw = {}
    if mask_kind != "none":
        if mask_kind == "prefix":
            lengths = torch.tensor([900, 1, 300, 0, 641], dtype=torch.int32, device=DEV)
            mask = torch.arange(s, device=DEV)[None, :] < lengths[:, None]
        else:
            mask = torch.rand(b, s, device=DEV, generator=g) > 0.4
            mask[:, 0] = True
        lens, flags = K().mask_lengths(mask)
        kw = dict(lengths=lens, key_mask=mask.to(torch.uint8), mask_flags=flags)
    ref = K().flash_attention(qkv, h, causal=True, **kw)
    sched = torch.zeros(2, dtype=torch.int32, device=DEV)
    for _ in range(3):
        out = K().flash_attention(qkv, h, causal=True, sched=sched, **kw)
        assert torch.equal(out, ref)
        assert sched.tolist() == [0, 0]


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("mask_kind", ["prefix", "general"])
def test_flash_skip_dead_rows(hd, mask_kind):
    """skip_dead_rows leaves the rows of query tiles wholly past a prefix
    length as they were and gives the same bits everywhere else; with a mask
    that is not a prefix nothing is skipped and every row matches."""
    b, s, h = 5, 900, 4
    g = torch.Generator(device=DEV).manual_seed(7 * hd + len(mask_kind))
    qkv = torch.randn(b, s, 3, h, hd, device=DEV, generator=g).half()
    if mask_kind == "prefix":
        lengths = torch.tensor([900, 1, 300, 0, 641], dtype=torch.int32, device=DEV)
        mask = torch.arange(s, device=DEV)[None, :] < lengths[:, None]
    else:
        mask = torch.rand(b, s, device=DEV, generator=g) > 0.4
        mask[:, 0] = True
    lens, flags = K().mask_lengths(mask)
    kw = dict(lengths=lens, key_mask=mask.to(torch.uint8), mask_flags=flags)
    ref = K().flash_attention(qkv, h, causal=True, **kw)
    sched = torch.zeros(2, dtype=torch.int32, device=DEV)
    # Fill the caching allocator's next block with a marker so that unwritten
    # rows are visible: flash_attention's output reuses the freed block.
    marker = torch.full((b * s, h * hd), 7.0, dtype=torch.float16, device=DEV)
    del marker
    out = K().flash_attention(qkv, h, causal=True, sched=sched, skip_dead_rows=True, **kw)
    assert sched.tolist() == [0, 0]
    live = torch.ones(b, s, dtype=torch.bool, device=DEV)
    if mask_kind == "prefix":
        tile0 = (torch.arange(s, device=DEV) // 128 * 128)[None, :]
        live = tile0 < lens.long()[:, None]
    live = live.reshape(-1)
    assert torch.equal(out[live], ref[live])
    if mask_kind == "prefix":
        # Dead rows are unspecified: left as they were (7.0) where the whole
        # work item was skipped, zero where a live tile shares the item.
        dead = out[~live]
        unwritten = (dead == 7.0).all(dim=1)
        assert bool((unwritten | (dead == 0).all(dim=1)).all())
        assert int(unwritten.sum()) > 0, "no dead work item was skipped"


def test_flash_unsupported_head_dim():
    from tjkernels._lib import KernelError
    qkv = torch.randn(1, 64, 3, 4, 32, device=DEV).bfloat16()
    with pytest.raises(KernelError):
        K().flash_attention(qkv, 4)


# ------------------------------------------------------------------------ FFN

@pytest.mark.parametrize("t,d,f", [(1, 128, 512), (256, 512, 2048), (1000, 1024, 4096)])
def test_ffn(t, d, f):
    h = torch.randn(t, d, device=DEV).bfloat16()
    w1 = (torch.randn(f, d, device=DEV) / math.sqrt(d)).bfloat16()
    w2 = (torch.randn(d, f, device=DEV) / math.sqrt(f)).bfloat16()
    b1, b2 = torch.randn(f, device=DEV), torch.randn(d, device=DEV)
    hidden = F.gelu(h.double() @ w1.double().T + b1.double(), approximate="none")
    ref = hidden.bfloat16().double() @ w2.double().T + b2.double()
    out = K().fused_ffn(h, w1, b1, w2, b2, out_dtype=torch.float32)
    assert (out.double() - ref).abs().max().item() < 2e-2


# ------------------------------------------------------------- mask / status

def test_mask_lengths_cases():
    m = torch.zeros(3, 50, dtype=torch.bool, device=DEV)
    m[0, :50] = True
    m[1, :7] = True
    lens, flags = K().mask_lengths(m)
    assert lens.tolist() == [50, 7, 0] and int(flags.item()) == 0
    m[2, 10] = True  # 0 -> 1 step: not a prefix
    lens, flags = K().mask_lengths(m)
    assert lens.tolist() == [50, 7, 1] and int(flags.item()) != 0


def test_bounded_wait_times_out_and_reports():
    from tjkernels import _lib
    assert K().device_status(clear=True) == 0
    never = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.check(_lib.lib().tjb_selftest_wait(never.data_ptr(), 50_000_000,
                                            torch.cuda.current_stream().cuda_stream), "wait")
    assert K().device_status(clear=True) == 7  # TJB_ERR_DEVICE_TIMEOUT
    assert K().device_status() == 0
    ready = torch.ones(1, dtype=torch.int32, device=DEV)
    _lib.check(_lib.lib().tjb_selftest_wait(ready.data_ptr(), 50_000_000,
                                            torch.cuda.current_stream().cuda_stream), "wait")
    assert K().device_status() == 0
    # The context is still usable afterwards.
    x = torch.randn(128, 64, device=DEV).bfloat16()
    assert torch.isfinite(K().gemm_bias(x, x[:64], None)).all()


# ------------------------------------------------------- padding-aware tiles

def row_tiles_reference(lengths, b, s):
    """Live 128-row tiles: those holding a row (b, s) with s < round_up(len, 128)."""
    t = b * s
    live = []
    for tile in range((t + 127) // 128):
        r0, r1 = tile * 128, min(tile * 128 + 128, t)
        if any((r % s) < (min(lengths[r // s], s) + 127) // 128 * 128 for r in range(r0, r1)):
            live.append(tile)
    return live


@pytest.mark.parametrize("b,s,lens", [(4, 1024, [1024, 1, 300, 0]), (3, 200, [200, 17, 129]),
                                      (5, 37, [1, 37, 20, 0, 5]), (2, 4096, [2048, 4000])])
def test_row_tiles(b, s, lens):
    lengths = torch.tensor(lens, dtype=torch.int32, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    tiles = K().row_tiles(lengths, flags, b, s, torch.device(DEV)).cpu().tolist()
    expect = row_tiles_reference(lens, b, s)
    assert tiles[0] == len(expect) and tiles[1:1 + tiles[0]] == expect
    flags.fill_(9)  # non-prefix mask: every tile is live
    tiles = K().row_tiles(lengths, flags, b, s, torch.device(DEV)).cpu().tolist()
    n = (b * s + 127) // 128
    assert tiles[0] == n and tiles[1:1 + n] == list(range(n))


def _mask_cases():
    g = torch.Generator().manual_seed(5)
    cases = []
    for b, s in ((8, 1024), (3, 200), (5, 37), (2, 4096), (40, 512), (1, 1), (70, 64), (4, 16)):
        lens = torch.randint(0, s + 1, (b,), generator=g)
        lens[0] = s
        if b > 1:
            lens[1] = 0
        prefix = torch.arange(s)[None, :] < lens[:, None]
        holed = prefix.clone()
        holed[b - 1, s // 2] = not holed[b - 1, s // 2]  # a 0 -> 1 rise, where S allows
        if s > 2:
            holed[b - 1, 0] = False
            holed[b - 1, s - 1] = True
        for m in (prefix, holed):
            mi = m.to(torch.int)
            rises = bool(((mi[:, 1:] == 1) & (mi[:, :-1] == 0)).any())
            cases.append((m, not rises))
    return cases


@pytest.mark.parametrize("case", range(16))
def test_mask_lengths_tiles_matches_separate_calls(case):
    """The one-launch classification + tile listing equals tjb_mask_lengths
    followed by tjb_row_tiles, for prefix masks and masks with a rise, S a
    multiple of 16 (16-byte loads) or not, more rows than warps, empty rows;
    and on a mask that does not start on a 16-byte boundary."""
    mask, is_prefix = _mask_cases()[case]
    for offset in (0, 3):
        buf = torch.zeros(mask.numel() + offset, dtype=torch.uint8)
        buf[offset:] = mask.flatten().to(torch.uint8)
        m = buf.to(DEV)[offset:].view(mask.shape)
        b, s = mask.shape
        lens, flags = K().mask_lengths(m)
        tiles = K().row_tiles(lens, flags, b, s, torch.device(DEV))
        lens2, flags2, tiles2 = K().mask_lengths_tiles(m)
        assert torch.equal(lens, lens2)
        assert torch.equal(lens2.cpu(), mask.sum(-1).to(torch.int32))
        assert (int(flags2) == 0) == is_prefix and (int(flags) == 0) == is_prefix
        n = int(tiles[0])
        assert int(tiles2[0]) == n and torch.equal(tiles[1:1 + n], tiles2[1:1 + n])


def test_gemm_and_layernorm_visit_only_listed_tiles():
    m, n, k = 1000, 512, 256
    a = torch.randn(m, k, device=DEV).half()
    w = (torch.randn(n, k, device=DEV) / 16).half()
    bias = torch.randn(n, device=DEV)
    listed = [0, 2, 7]  # tile 7 is the ragged last tile (rows 896..999)
    tiles = torch.tensor([len(listed)] + listed + [0] * 5, dtype=torch.int32, device=DEV)
    out = torch.full((m, n), 7.0, dtype=torch.float32, device=DEV)
    K().gemm_bias(a, w, bias, out_dtype=torch.float32, out=out, m_tiles=tiles)
    ref = a.double() @ w.double().T + bias.double()
    for t in range(8):
        rows = slice(t * 128, min(t * 128 + 128, m))
        if t in listed:
            assert (out[rows].double() - ref[rows]).abs().max().item() < 1e-3
        else:
            assert (out[rows] == 7.0).all()
    res = torch.randn(m, 1024, device=DEV)
    delta = torch.randn(m, 1024, device=DEV)
    w1, b1 = torch.randn(1024, device=DEV), torch.randn(1024, device=DEV)
    res0 = res.clone()
    new_res, h = K().fused_add_layernorm(res, delta, w1, b1, 1e-5, out_dtype=torch.float32,
                                         residual_out=res, m_tiles=tiles)
    ref_h = F.layer_norm(res0 + delta, (1024,), w1, b1, 1e-5)
    for t in range(8):
        rows = slice(t * 128, min(t * 128 + 128, m))
        if t in listed:
            assert (h[rows] - ref_h[rows]).abs().max().item() < 1e-4
            assert torch.equal(new_res[rows], (res0 + delta)[rows])
        else:
            assert torch.equal(new_res[rows], res0[rows])


def test_add_layernorm_live_tiles_many_rows():
    """The persistent LayerNorm over a tile list of more than 1024 rows: listed
    tiles (the ragged last one included) are normalised, the others are left
    untouched."""
    m, d = 9000, 1024  # 71 tiles, the last one 40 rows
    listed = [0, 3, 4, 5, 17, 30, 31, 32, 50, 69, 70]
    n_tiles = (m + 127) // 128
    tiles = torch.tensor([len(listed)] + listed + [0] * (n_tiles - len(listed)),
                         dtype=torch.int32, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(5)
    res = torch.randn(m, d, device=DEV, generator=g)
    delta = torch.randn(m, d, device=DEV, generator=g).half()
    w, b = torch.randn(d, device=DEV, generator=g), torch.randn(d, device=DEV, generator=g)
    res0 = res.clone()
    new_res, h = K().fused_add_layernorm(res, delta, w, b, 1e-5, out_dtype=torch.float16,
                                         residual_out=res, m_tiles=tiles)
    x = res0 + delta.float()
    ref = F.layer_norm(x, (d,), w, b, 1e-5)
    for t in range(n_tiles):
        rows = slice(t * 128, min(t * 128 + 128, m))
        if t in listed:
            assert ((h[rows].float() - ref[rows]).abs() <= 1e-2 * ref[rows].abs() + 1e-2).all()
            assert torch.equal(new_res[rows], x[rows])
        else:
            assert torch.equal(new_res[rows], res0[rows])


@pytest.mark.parametrize("t,d,f", [(1, 256, 1024), (200, 512, 2048), (1000, 768, 3072),
                                   (4096, 1024, 4096), (300, 1024, 4096)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_ffn_single_kernel_matches_two_gemm_path(t, d, f, dtype):
    g = torch.Generator(device=DEV).manual_seed(t + d + f)
    h = torch.randn(t, d, device=DEV, generator=g).to(dtype)
    w1 = (torch.randn(f, d, device=DEV, generator=g) / math.sqrt(d)).to(dtype)
    w2 = (torch.randn(d, f, device=DEV, generator=g) / math.sqrt(f)).to(dtype)
    b1 = torch.randn(f, device=DEV, generator=g)
    b2 = torch.randn(d, device=DEV, generator=g)
    assert K().ffn_fused_supports(d, f)
    two = K().fused_ffn(h, w1, b1, w2, b2, out_dtype=torch.float32)
    one = K().ffn_single_kernel(h, w1, b1, w2, b2, out_dtype=torch.float32)
    # Same products, same k order, hidden rounded to the same 16-bit type.
    assert (one - two).abs().max().item() < 1e-3
    hidden = F.gelu(h.double() @ w1.double().T + b1.double(), approximate="none")
    ref = hidden.to(dtype).double() @ w2.double().T + b2.double()
    assert (one.double() - ref).abs().max().item() < 2e-2


def test_ffn_single_kernel_live_tiles():
    t, d, f = 1000, 1024, 4096
    h = torch.randn(t, d, device=DEV).half()
    w1 = (torch.randn(f, d, device=DEV) / 32).half()
    w2 = (torch.randn(d, f, device=DEV) / 64).half()
    b1, b2 = torch.randn(f, device=DEV), torch.randn(d, device=DEV)
    listed = [1, 3, 7]
    tiles = torch.tensor([3] + listed + [0] * 5, dtype=torch.int32, device=DEV)
    full = K().ffn_single_kernel(h, w1, b1, w2, b2, out_dtype=torch.float32)
    out = K().ffn_single_kernel(h, w1, b1, w2, b2, out_dtype=torch.float32, m_tiles=tiles)
    for tile in listed:
        rows = slice(tile * 128, min(tile * 128 + 128, t))
        assert torch.equal(out[rows], full[rows])


def test_ffn_single_kernel_rejects_unsupported():
    from tjkernels._lib import KernelError
    h = torch.randn(8, 4096, device=DEV).half()
    w = torch.randn(16384, 4096, device=DEV).half()
    with pytest.raises(KernelError):
        K().ffn_single_kernel(h, w, torch.zeros(16384, device=DEV), w.T.contiguous(),
                              torch.zeros(4096, device=DEV))

"""Host-side checks that need no GPU: the C-ABI library loads and exports
every symbol the header declares; argument validation answers without a
device; plan dispatch; and the engine refuses to fall back to the CPU."""

import json
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tjb200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^(?:int|size_t|const char\*)\s+(tjb_\w+)\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from tjkernels import _lib
    names = declared_symbols()
    assert len(names) >= 9
    handle = _lib.load()
    for name in names:
        assert hasattr(handle, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    assert handle.tjb_version() >= 100


def test_status_strings():
    from tjkernels import _lib
    lib = _lib.lib()
    assert lib.tjb_status_string(0) == b"ok"
    assert b"timed out" in lib.tjb_status_string(7)
    assert lib.tjb_status_string(12345) == b"unknown status"


def test_argument_validation_without_device():
    """Null pointers and bad shapes are rejected before any device work."""
    from tjkernels import _lib
    lib = _lib.lib()
    assert lib.tjb_add_layernorm(None, None, None, None, None, None, 4, 8, 1e-5, 0, 0,
                                 None, None) == 1
    assert lib.tjb_gemm_bias(None, None, None, None, 1, 8, 8, 8, 8, 8, 2, 2, 0, None) == 1
    assert lib.tjb_flash_fwd(None, None, 1, 1, 1, 64, 1.0, 1, None, None, None, 2, None) == 1
    # Non-null but shape-invalid arguments: K not a multiple of 8.
    fake = 1 << 20
    assert lib.tjb_gemm_bias(fake, fake, None, fake, 1, 8, 7, 8, 8, 8, 2, 2, 0, None) == 2
    # Unsupported head dim.
    assert lib.tjb_flash_fwd(fake, fake, 1, 1, 1, 48, 1.0, 1, None, None, None, 2, None) == 2
    # Unsupported dtype (fp32 tensor-core input).
    assert lib.tjb_gemm_bias(fake, fake, None, fake, 1, 8, 8, 8, 8, 8, 0, 0, 0, None) == 4


def test_gemm_add_layernorm_contract_without_device():
    """The fused GEMM + LayerNorm sizes its workspace on the host and rejects
    a missing or short workspace, unsupported widths and misaligned pointers
    before any device work."""
    from tjkernels import _lib
    lib = _lib.lib()
    for m, n in ((1, 256), (300, 1024), (16384, 768), (8192, 1024)):
        blocks = -(-m // 128)
        counters = -(-(2 * blocks * 4) // 256) * 256
        assert lib.tjb_gemm_add_layernorm_workspace_bytes(m, n) == counters + (n // 256) * 2 * m * 8
    assert lib.tjb_gemm_add_layernorm_workspace_bytes(0, 1024) == 256
    fake = 1 << 20
    f16, f32 = _lib.TJB_F16, _lib.TJB_F32

    def call(n=1024, k=1024, ws=fake, ws_bytes=None, a=fake):
        if ws_bytes is None:
            ws_bytes = lib.tjb_gemm_add_layernorm_workspace_bytes(300, n)
        return lib.tjb_gemm_add_layernorm(a, fake, fake, fake, fake, fake, fake, fake, 300, n,
                                          k, 1e-5, f16, f32, None, None, ws, ws_bytes, None)

    assert call(ws=None) == 1                                  # no workspace
    assert call(ws_bytes=1024) == 1                            # workspace too small
    assert call(n=2048) == 2                                   # wider than four 256-column tiles
    assert call(n=1000) == 2                                   # not a multiple of 256
    assert call(k=1020) == 2                                   # K not a multiple of 8
    assert call(a=fake + 4) == 3                               # misaligned operand


def test_forward_small_contract_without_device():
    """The whole-forward entry point rejects bad arguments, unsupported
    dtypes and shapes outside its contract before it touches a device, and
    sizes its workspace on the host."""
    import ctypes
    from tjkernels import _lib
    lib = _lib.lib()
    assert lib.tjb_forward_small_workspace_bytes(0, 64, 768, 3072) == 0
    small = lib.tjb_forward_small_workspace_bytes(1, 64, 768, 3072)
    assert small > 0 and lib.tjb_forward_small_workspace_bytes(4, 64, 768, 3072) > small
    fake = 1 << 20
    layers = (_lib.SmallLayer * 4)()
    for ly in layers:
        for name, _ in _lib.SmallLayer._fields_[:12]:
            setattr(ly, name, fake)
    f16, bf16 = _lib.TJB_F16, _lib.TJB_BF16

    def call(b=1, s=64, d=768, h=12, f=3072, n_layers=4, dtype=f16, ws=fake, lys=layers):
        return lib.tjb_forward_small(ctypes.addressof(lys) if lys is not None else None,
                                     n_layers, fake, fake, 1e-5, fake, fake, None, b, s, d, h, f,
                                     1, dtype, ws, 1 << 30, None)

    assert call(lys=None) == 1                     # no layer table
    assert call(ws=None) == 1                      # no workspace
    assert call(n_layers=0) == 1
    assert call(dtype=bf16) == 4                   # fp16 only
    assert call(d=768, h=6) == 2                   # head_dim 128
    assert call(b=3, s=100, d=512, h=8, f=2048) == 2   # 300 tokens
    assert call(b=1, s=200, d=512, h=8, f=2048) == 2   # sequence longer than 128
    assert call(f=3000) == 2                       # F not a multiple of 128
    assert call(n_layers=13) == 2                  # more than 12 blocks
    assert call() == 8                             # valid call, no device here


def test_ffn_noalloc_limit_without_device():
    """The allocation-free FFN refuses T * F beyond its fixed array before it
    touches a device or a pointer (so the pointers here are never used)."""
    from tjkernels import _lib
    lib = _lib.lib()
    fake = 1 << 20
    too_many_rows = (8 << 20) // 64 + 1
    assert lib.tjb_ffn_noalloc(fake, fake, fake, fake, fake, fake, too_many_rows, 64, 64,
                               _lib.TJB_F16, _lib.TJB_F32, None) == 2
    assert lib.tjb_ffn_noalloc(None, fake, fake, fake, fake, fake, 8, 64, 64,
                               _lib.TJB_F16, _lib.TJB_F32, None) == 1


def test_device_status_async_validation_without_device():
    from tjkernels import _lib
    lib = _lib.lib()
    assert lib.tjb_device_status_async(None, None) == 1
    assert lib.tjb_device_status_async((1 << 20) + 2, None) == 1  # not 4-byte aligned


def test_kernel_error_carries_status():
    from tjkernels import _lib
    with pytest.raises(_lib.KernelError) as info:
        _lib.check(3, "probe")
    assert info.value.status == 3 and "aligned" in str(info.value)


def test_plan_roundtrip_and_env(tmp_path, monkeypatch):
    from tjkernels import plans
    p = plans.Plan(compute_dtype=torch.float16, delta_dtype=torch.bfloat16, cuda_graph=False,
                   label="x")
    assert plans.Plan.from_json(json.loads(json.dumps(p.to_json()))) == p
    key = plans.shape_key(2, 128, 512, 8, 2048, 4, True, torch.float32)
    assert key == "b2_s128_d512_h8_f2048_l4_causal_float32"
    path = tmp_path / "plans.json"
    plans.save_plans({key: p}, path)
    assert json.loads(path.read_text())[key]["compute_dtype"] == "float16"
    dev = torch.device("cuda")
    monkeypatch.setenv("TJ_IGNORE_PLANS", "1")
    plans._cache = None
    base = plans.select_plan(2, 128, 512, 8, 2048, 4, True, torch.float32, dev)
    assert base.compute_dtype == torch.float16 and base.cuda_graph
    big = plans.select_plan(64, 2048, 4096, 32, 16384, 12, True, torch.float32, dev)
    assert not big.cuda_graph  # 2 GB input: graph copy-in/clone-out not free
    monkeypatch.setenv("TJ_NO_GRAPH", "1")
    monkeypatch.setenv("TJ_COMPUTE_DTYPE", "bfloat16")
    forced = plans.select_plan(2, 128, 512, 8, 2048, 4, True, torch.float32, dev)
    assert not forced.cuda_graph and forced.compute_dtype == torch.bfloat16
    monkeypatch.setenv("TJ_NO_STREAM_K", "1")
    assert not plans.select_plan(2, 128, 512, 8, 2048, 4, True, torch.float32, dev).gemm_stream_k
    monkeypatch.setenv("TJ_FUSE_LN", "1")
    assert plans.select_plan(2, 128, 512, 8, 2048, 4, True, torch.float32, dev).fuse_layernorm
    plans.set_override(p)
    try:
        assert plans.select_plan(1, 1, 1, 1, 1, 1, True, torch.float32, dev) is p
    finally:
        plans.set_override(None)
        plans._cache = None


def test_fused_layernorm_plan_selection(monkeypatch):
    """The tuned B8 S1024 plan fuses only the out-projection's LayerNorm into
    its GEMM; the B4 S4096 one keeps the LayerNorms standalone (faster there
    since the persistent LayerNorm kernel); TJ_FUSE_LN=0/1 overrides."""
    from tjkernels import plans
    dev = torch.device("cuda")
    monkeypatch.delenv("TJ_IGNORE_PLANS", raising=False)
    monkeypatch.delenv("TJ_FUSE_LN", raising=False)
    plans._cache = None
    try:
        long_seq = (4, 4096, 1024, 16, 4096, 4, True, torch.float32, dev)
        p3 = plans.select_plan(*long_seq)
        assert not p3.fuse_layernorm
        p2 = plans.select_plan(8, 1024, 1024, 16, 4096, 4, True, torch.float32, dev)
        assert p2.fuse_layernorm and not p2.fuse_layernorm_ffn
        monkeypatch.setenv("TJ_FUSE_LN", "1")
        assert plans.select_plan(*long_seq).fuse_layernorm
        monkeypatch.setenv("TJ_FUSE_LN", "0")
        assert not plans.select_plan(8, 1024, 1024, 16, 4096, 4, True, torch.float32,
                                     dev).fuse_layernorm
    finally:
        plans._cache = None


def test_layernorm_workspace_outlives_the_graphs_that_use_it(monkeypatch):
    """When a larger batch grows the fused LayerNorm's workspace, the old one
    stays alive (graphs captured for the smaller shape still point at it)
    until the engine releases its graphs."""
    from tjkernels import engine as E
    from tjkernels import kernels as K
    monkeypatch.setattr(K, "gemm_add_layernorm_workspace",
                        lambda rows, d, device: torch.zeros(
                            K.gemm_add_layernorm_workspace_bytes(rows, d), dtype=torch.uint8))
    eng = E.Engine.__new__(E.Engine)
    eng._ln_ws = None
    eng._ln_ws_retired = []
    cpu = torch.device("cpu")
    small = eng._ln_workspace(1024, 1024, cpu)
    assert eng._ln_workspace(512, 1024, cpu) is small  # fits: reused
    big = eng._ln_workspace(8192, 1024, cpu)
    assert big is not small and big.numel() > small.numel()
    assert any(t is small for t in eng._ln_ws_retired)
    assert eng._ln_workspace(8192, 1024, cpu) is big


def test_plan_json_from_earlier_builds():
    """A plan stored before stream-K (with the retired split-tail key) loads
    with the stream-K default instead of failing."""
    from tjkernels import plans
    old = {"compute_dtype": "float16", "residual_dtype": "float32", "delta_dtype": "float16",
           "cuda_graph": True, "skip_padding": True, "ffn_single_kernel": False,
           "attn_dynamic": True, "gemm_split_tail": False, "label": "tuned"}
    p = plans.Plan.from_json(old)
    assert p.gemm_stream_k and p.label == "tuned" and p.delta_dtype == torch.float16
    assert "gemm_split_tail" not in p.to_json() and p.to_json()["gemm_stream_k"] is True


def test_no_cpu_fallback():
    from tjkernels import plans
    with pytest.raises(RuntimeError):
        plans.default_plan(1, 8, 128, 2, 128, 1, True, torch.float32, torch.device("cpu"))
    import tjkernels.kernels as K
    with pytest.raises(RuntimeError):
        K.gemm_bias(torch.zeros(8, 8, dtype=torch.bfloat16),
                    torch.zeros(8, 8, dtype=torch.bfloat16), None)


def test_tj_disable_runs_baseline(monkeypatch):
    """TJ_DISABLE=1 routes the hook to the baseline forward (engine.py:322)."""
    import tjkernels
    from oracle.model import ModelConfig, ReferenceModel, generate_case

    class Optimized(ReferenceModel):
        def forward(self, x, valid_token_mask=None):
            return tjkernels.forward(self, x, valid_token_mask)

    cfg = ModelConfig(1, 16, 128, 2, 128, 1, True)
    torch.manual_seed(0)
    model = Optimized(cfg).eval()
    x, m = generate_case(cfg, 0, 0.3)
    monkeypatch.setenv("TJ_DISABLE", "1")
    with torch.no_grad():
        out = model(x, m)
        ref = ReferenceModel.forward(model, x, m)
    assert torch.equal(out, ref)


def test_oracle_ignores_subclass_forward():
    """oracle_forward must run the reference math even on a hooked subclass."""
    from oracle.model import ModelConfig, ReferenceModel, generate_case, oracle_forward

    class Hooked(ReferenceModel):
        def forward(self, x, valid_token_mask=None):
            return torch.zeros_like(x)

    cfg = ModelConfig(1, 8, 128, 2, 128, 1, True)
    torch.manual_seed(0)
    model = Hooked(cfg).eval()
    x, m = generate_case(cfg, 0, 0.0)
    assert oracle_forward(model, x, m).abs().sum() > 0

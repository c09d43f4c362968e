"""The whole-forward kernel (tjb_forward_small, plan knob ``whole_forward``)
against the fp32 oracle: the small bench configs (0 and 1), other shapes in
its contract (ragged token counts, non-causal, one layer), a key mask with
holes, eager against graph replay, and repeated launches on one workspace
(the grid barrier's generation word carries over between calls)."""

import pytest
import torch

from oracle.model import (BENCH_CONFIGS, ModelConfig, ReferenceModel, budget_usage,
                          generate_case, oracle_forward)

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


class Optimized(ReferenceModel):
    def forward(self, x, valid_token_mask=None):
        import tjkernels
        return tjkernels.forward(self, x, valid_token_mask)


def make_optimized(cfg: ModelConfig, seed: int) -> Optimized:
    torch.manual_seed(seed)
    ref = ReferenceModel(cfg)
    opt = Optimized(cfg)
    opt.load_state_dict(ref.state_dict(), strict=True)
    return opt.to(DEV).eval()


@pytest.fixture(autouse=True)
def _plans():
    import tjkernels.plans as plans
    plans.set_override(None)
    yield
    plans.set_override(None)


def run_whole(model, x, mask, graph: bool):
    import tjkernels.plans as plans
    from tjkernels.engine import get_engine
    plans.set_override(plans.Plan(cuda_graph=graph, whole_forward=True, label="whole"))
    with torch.inference_mode():
        got = model(x, mask)
    assert get_engine(model)._small is not None, "the whole-forward kernel did not run"
    return got


def check(ref, got, mask):
    valid = mask.bool()
    usage = budget_usage(ref[valid], got[valid])
    assert usage <= 1.0, f"budget usage {usage:.3f}"
    assert bool((got[~valid] == 0).all()), "padded rows are not exactly zero"
    return usage


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("cfg_id", [0, 1])
def test_whole_forward_bench_configs(cfg_id, graph):
    cfg, pad = BENCH_CONFIGS[cfg_id]
    model = make_optimized(cfg, 0)
    x, mask = generate_case(cfg, 0, pad)
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        ref = oracle_forward(model, x, mask)
    first = run_whole(model, x, mask, graph).clone()
    usage = check(ref, first, mask)
    # Later launches reuse the workspace (barrier generation carried over)
    # and reproduce the first output bit for bit.
    for _ in range(3):
        with torch.inference_mode():
            again = model(x, mask)
        assert torch.equal(again, first)
    print(f"config {cfg_id} graph={graph}: budget usage {usage:.3f}")


@pytest.mark.parametrize("b,s,d,h,f,layers,causal,pad", [
    (4, 64, 256, 4, 512, 2, True, 0.5),
    (1, 128, 512, 8, 1024, 3, True, 0.0),
    (2, 96, 384, 6, 1536, 2, False, 0.3),
    (3, 50, 128, 2, 256, 1, True, 0.4),
    (16, 16, 768, 12, 3072, 2, True, 0.5),
])
def test_whole_forward_shapes(b, s, d, h, f, layers, causal, pad):
    cfg = ModelConfig(b, s, d, h, f, layers, causal)
    model = make_optimized(cfg, 5)
    x, mask = generate_case(cfg, 6, pad)
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        ref = oracle_forward(model, x, mask)
    got = run_whole(model, x, mask, graph=False)
    usage = check(ref, got, mask)
    print(f"B{b} S{s} d{d} causal={causal}: budget usage {usage:.3f}")


def test_whole_forward_mask_with_holes():
    """A key mask that is not a prefix: masked keys are left out and masked
    rows come out zero, as in the reference."""
    cfg = ModelConfig(2, 128, 512, 8, 2048, 2, True)
    model = make_optimized(cfg, 7)
    g = torch.Generator().manual_seed(8)
    x = torch.randn(2, 128, 512, generator=g)
    mask = torch.rand(2, 128, generator=g) > 0.3
    mask[:, 0] = True
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        ref = oracle_forward(model, x, mask)
    got = run_whole(model, x, mask, graph=False)
    check(ref, got, mask)


def test_whole_forward_matches_the_per_op_path():
    """Both paths of the engine on config 1 agree within the budget of each
    other (the per-op path is checked against the oracle elsewhere)."""
    import tjkernels.plans as plans
    cfg, pad = BENCH_CONFIGS[1]
    x, mask = generate_case(cfg, 1, pad)
    x, mask = x.to(DEV), mask.to(DEV)
    per_op = make_optimized(cfg, 2)
    plans.set_override(plans.Plan(cuda_graph=False, label="per-op"))
    with torch.inference_mode():
        a = per_op(x, mask)
    whole = make_optimized(cfg, 2)
    b = run_whole(whole, x, mask, graph=False)
    assert budget_usage(a[mask.bool()], b[mask.bool()]) <= 1.0


def test_whole_forward_contract():
    import tjkernels.kernels as K
    from tjkernels._lib import KernelError
    f16 = torch.float16
    assert K.forward_small_supports(1, 64, 768, 12, 3072, 4, 64, f16)
    assert not K.forward_small_supports(1, 64, 768, 6, 3072, 4, 128, f16)   # head_dim 128
    assert not K.forward_small_supports(3, 100, 512, 8, 2048, 4, 64, f16)   # 300 tokens
    assert not K.forward_small_supports(1, 200, 512, 8, 2048, 4, 64, f16)   # sequence > 128
    assert not K.forward_small_supports(1, 64, 768, 12, 3072, 4, 64, torch.bfloat16)
    assert not K.forward_small_supports(1, 64, 768, 12, 3000, 4, 64, f16)   # F % 128
    cfg = ModelConfig(1, 64, 256, 4, 512, 1, True)
    model = make_optimized(cfg, 9)
    x = torch.randn(1, 64, 256, device=DEV)
    run_whole(model, x, None, graph=False)
    from tjkernels.engine import get_engine
    eng = get_engine(model)
    short = torch.zeros(1024, dtype=torch.uint8, device=DEV)
    with pytest.raises(KernelError):
        K.forward_small(eng._small, x, None, 4, 512, True, short)

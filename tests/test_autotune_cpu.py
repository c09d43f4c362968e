"""The plan autotuner's host logic and its accuracy reference, on the CPU:
the candidate set, the budget measure, the input distribution, and
``tjkernels.model.torch_forward`` (the tuner's gate) against the pinned
oracle forward on the same parameters."""

import torch

from oracle.model import ModelConfig, ReferenceModel, generate_case, oracle_forward


def test_candidates_cover_the_knobs():
    from tjkernels import autotune, plans
    base = plans.Plan()
    c512 = autotune.candidates(512, 2048, base)      # single-kernel FFN, fused LN possible
    c4096 = autotune.candidates(4096, 16384, base)   # neither
    assert len(c512) == 6 * len(c4096) == 96
    assert {p.compute_dtype for p in c512} == {torch.float16, torch.bfloat16}
    assert all(p.delta_dtype in (torch.float32, p.compute_dtype) for p in c512)
    assert not any(p.ffn_single_kernel for p in c4096)
    modes = {(p.fuse_layernorm, p.fuse_layernorm_ffn) for p in c512}
    assert modes == {(False, True), (True, False), (True, True)}
    assert not any(p.fuse_layernorm for p in c4096)
    assert len({tuple(sorted(p.to_json().items())) for p in c512}) == len(c512)


def test_budget_usage_and_inputs():
    from tjkernels import autotune
    ref = torch.tensor([0.0, 1.0, -200.0])
    assert autotune.budget_usage(ref, ref) == 0.0
    assert abs(autotune.budget_usage(ref, ref + torch.tensor([0.005, 0.0, 1.0])) - 0.5) < 1e-9
    x, m = autotune.make_inputs(3, 64, 16, 0.5, 7, torch.device("cpu"))
    lengths = m.sum(-1)
    assert bool(((lengths >= 32) & (lengths <= 64)).all())
    assert bool((x[~m] == 0).all())
    x0, m0 = autotune.make_inputs(2, 8, 4, 0.0, 1, torch.device("cpu"))
    assert bool(m0.all())


def test_torch_forward_matches_oracle():
    from tjkernels.model import Encoder, EncoderConfig, torch_forward
    cfg = ModelConfig(2, 48, 128, 4, 256, 2, True)
    torch.manual_seed(0)
    enc = Encoder(EncoderConfig(2, 48, 128, 4, 256, 2, True))
    ref_model = ReferenceModel(cfg)
    ref_model.load_state_dict(enc.state_dict(), strict=True)
    x, mask = generate_case(cfg, 3, 0.5)
    with torch.no_grad():
        got = torch_forward(enc, x, mask)
    want = oracle_forward(ref_model, x, mask)
    assert (got - want).abs().max().item() < 1e-4
    assert bool((got[~mask] == 0).all())

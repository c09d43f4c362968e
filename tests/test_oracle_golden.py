"""Pin the CPU oracle to the reference's own outputs (CPU only).

The fixtures in ``tests/golden`` were produced by running the reference
harness's ``BaselineTransformer`` and ``generate_random_case``
(``torch_transformer_benchmark.py:155-179, 238-276``) -- see
``tests/golden/make_golden.py``.  Here the oracle restatement must reproduce
the inputs, the seeded weights and the outputs.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle.model import ModelConfig, build_model, generate_case, oracle_forward, budget_usage

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = sorted(p.stem for p in GOLDEN.glob("*.npz"))


def load(name):
    blob = np.load(GOLDEN / f"{name}.npz")
    b, s, d, h, f, layers, causal = (int(v) for v in blob["shape"])
    cfg = ModelConfig(b, s, d, h, f, layers, bool(causal))
    return cfg, blob


def test_fixture_set_present():
    assert "cfg0" in CASES and len(CASES) >= 10


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_reference(name):
    cfg, blob = load(name)
    torch.set_float32_matmul_precision("highest")
    model = build_model(cfg, seed=int(blob["model_seed"]))
    # Same seeded weights as the reference module (names and per-tensor sums).
    sd = model.state_dict()
    names = [str(n) for n in blob["param_names"]]
    assert sorted(sd.keys()) == names
    sums = np.array([float(sd[k].double().sum()) for k in names])
    np.testing.assert_allclose(sums, blob["param_sums"], rtol=0, atol=1e-9)
    # Same seeded inputs.
    x, mask = generate_case(cfg, int(blob["seed"]), float(blob["padding"]))
    assert np.array_equal(mask.numpy(), blob["mask"])
    assert float(x.double().sum()) == pytest.approx(float(blob["x_sum"]), abs=1e-9)
    assert float((x.double() ** 2).sum()) == pytest.approx(float(blob["x_sq"]), rel=1e-12)
    if "x" in blob:
        assert np.array_equal(x.numpy(), blob["x"])
    # Same outputs (identical fp32 CPU math; a 1e-5 band absorbs BLAS threading).
    out = oracle_forward(model, x, mask)
    ref = torch.from_numpy(blob["out"])
    assert (out - ref).abs().max().item() <= 1e-5
    assert budget_usage(ref, out) < 1e-2
    # Padded rows are exactly zero.
    assert bool((out[~mask] == 0).all())


def test_budget_rule_planted_error():
    """A planted error just over the budget is caught; one under it is not."""
    ref = torch.tensor([0.0, 0.5, 2.0, -3.0])
    ok = ref + torch.tensor([0.0099, -0.0099, 0.0199, -0.0299])
    bad = ref + torch.tensor([0.0, 0.0, 0.0, 0.0301])
    assert budget_usage(ref, ok) < 1.0
    assert budget_usage(ref, bad) > 1.0

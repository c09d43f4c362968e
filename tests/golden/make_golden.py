"""Generate the golden fixtures that pin the oracle to the reference.

Runs the reference's own ``BaselineTransformer`` and ``generate_random_case``
(``torch_transformer_benchmark.py:155-179`` and ``:238-276``) on the CPU in
fp32 with matmul precision "highest", and stores, per case:

* the input ``x`` (only for the named benchmark config 0; the small cases
  store a checksum of ``x`` instead, to keep the fixtures small),
* the prefix mask,
* the reference output,
* per-parameter sums of the seeded default-initialised weights.

This script needs the reference checkout (pass its path as the first
argument); the fixtures it writes travel with the repository so the tests do
not.  Usage::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py <reference_dir>
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name -> (batch, seq, d_model, heads, ffn, layers, causal, padding, seed, model_seed, store_x)
# The small cases follow the reference's own correctness matrix
# (bench/test_correctness.py:132-156) at batch 2 with head_dim 64 where the
# reference used 32 ("hd32" keeps one head_dim-32 case); "cfg0" is benchmark
# config 0.
CASES = {
    "cfg0": (2, 128, 512, 8, 2048, 4, True, 0.5, 0, 0, True),
    "base": (2, 64, 128, 2, 128, 2, True, 0.0, 1, 1, False),
    "pad03": (2, 64, 128, 2, 128, 2, True, 0.3, 2, 1, False),
    "pad06": (2, 64, 128, 2, 128, 2, True, 0.6, 3, 1, False),
    "noncausal": (2, 64, 128, 2, 128, 2, False, 0.0, 4, 1, False),
    "noncausal_pad": (2, 64, 128, 2, 128, 2, False, 0.4, 5, 1, False),
    "hd32": (2, 64, 128, 4, 128, 2, True, 0.3, 11, 1, False),
    "ragged37": (2, 37, 128, 2, 128, 2, True, 0.0, 6, 1, False),
    "seq1": (2, 1, 128, 2, 128, 2, True, 0.0, 7, 1, False),
    "hd64_s200": (2, 200, 256, 4, 512, 2, True, 0.3, 8, 1, False),
    "hd128": (2, 160, 256, 2, 512, 1, True, 0.5, 9, 1, False),
    "ffn512_l1": (1, 96, 128, 2, 512, 1, True, 0.0, 10, 1, False),
}


def main(reference_dir: str) -> None:
    sys.path.insert(0, reference_dir)
    import torch_transformer_benchmark as ref  # noqa: E402  (the reference harness)

    torch.set_float32_matmul_precision("highest")
    for name, (b, s, d, h, f, layers, causal, pad, seed, mseed, store_x) in CASES.items():
        cfg = ref.TransformerConfig(batch_size=b, seq_len=s, d_model=d, num_heads=h,
                                    ffn_dim=f, num_layers=layers, causal=causal)
        torch.manual_seed(mseed)
        model = ref.BaselineTransformer(cfg).eval()
        x, mask = ref.generate_random_case(cfg, torch.device("cpu"), torch.float32,
                                           seed=seed, padding_ratio=pad, input_scale=1.0)
        with torch.no_grad():
            out = model(x, mask)
        names = sorted(model.state_dict().keys())
        sums = np.array([float(model.state_dict()[k].double().sum()) for k in names])
        blob = dict(
            shape=np.array([b, s, d, h, f, layers, int(causal)], dtype=np.int64),
            padding=np.array(pad, dtype=np.float64),
            seed=np.array(seed, dtype=np.int64),
            model_seed=np.array(mseed, dtype=np.int64),
            mask=mask.numpy(),
            out=out.numpy().astype(np.float32),
            x_sum=np.array(float(x.double().sum())),
            x_sq=np.array(float((x.double() ** 2).sum())),
            param_names=np.array(names),
            param_sums=sums,
        )
        if store_x:
            blob["x"] = x.numpy().astype(np.float32)
        np.savez_compressed(HERE / f"{name}.npz", **blob)
        print(f"{name}: out{tuple(out.shape)} lengths={mask.sum(-1).tolist()}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "../reference")

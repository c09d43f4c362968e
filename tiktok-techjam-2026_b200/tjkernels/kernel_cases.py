"""Run one library kernel on seeded inputs of a given shape (profiling driver).

    python -m tjkernels.kernel_cases gemm M N K [--act gelu] [--out f16|f32] [--stream-k] [--launches 3]
    python -m tjkernels.kernel_cases attn B S H HD [--lengths prefix] [--launches 3]
    python -m tjkernels.kernel_cases ln ROWS D [--launches 3]
    python -m tjkernels.kernel_cases ffn T D F [--launches 3]
    python -m tjkernels.kernel_cases gemm_ln M N K [--launches 3]

Each call launches the kernel ``--launches`` times (fp16 inputs) and prints
the median CUDA-event time of all but the first launch.  It is the
command the ncu summaries of a single kernel are taken with (``ncu -k
regex:<kernel> -s <n> -c 1 python -m tjkernels.kernel_cases ...``), so a
capture sees exactly the kernel, shape and launch count named on its line.
"""

from __future__ import annotations

import argparse
import sys

import torch

from . import kernels as K


def _timed(fn, launches: int) -> float:
    """Median CUDA-event time of launches 2..n (the first is a warm-up)."""
    fn()
    times = []
    for _ in range(max(1, launches - 1)):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    return sorted(times)[len(times) // 2]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("kernel", choices=["gemm", "attn", "ln", "ffn", "gemm_ln"])
    ap.add_argument("dims", type=int, nargs="+")
    ap.add_argument("--act", choices=["none", "gelu"], default="none")
    ap.add_argument("--out", choices=["f16", "f32"], default="f16")
    ap.add_argument("--lengths", choices=["full", "prefix"], default="full")
    ap.add_argument("--stream-k", action="store_true",
                    help="gemm: pass a stream-K workspace")
    ap.add_argument("--launches", type=int, default=3)
    args = ap.parse_args(argv)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)

    def randn(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).half()

    if args.kernel == "gemm":
        m, n, k = args.dims
        a, w = randn(m, k), randn(n, k, scale=k ** -0.5)
        bias = torch.randn(n, device=dev, generator=g)
        out_dtype = torch.float16 if args.out == "f16" else torch.float32
        act = K.ACT_GELU if args.act == "gelu" else K.ACT_NONE
        ws = K.gemm_workspace(dev) if args.stream_k else None
        ms = _timed(lambda: K.gemm_bias(a, w, bias, act=act, out_dtype=out_dtype, workspace=ws),
                    args.launches)
        flops = 2.0 * m * n * k
    elif args.kernel == "attn":
        b, s, h, hd = args.dims
        qkv = randn(b, s, 3, h, hd)
        kw = {}
        if args.lengths == "prefix":
            lengths = torch.randint(s // 2, s + 1, (b,), device=dev, generator=g)
            mask = torch.arange(s, device=dev)[None, :] < lengths[:, None]
            lens, flags = K.mask_lengths(mask)
            kw = dict(lengths=lens, key_mask=mask.to(torch.uint8), mask_flags=flags,
                      sched=torch.zeros(2, dtype=torch.int32, device=dev))
            n_list = lengths.tolist()
        else:
            n_list = [s] * b
        ms = _timed(lambda: K.flash_attention(qkv, h, causal=True, **kw), args.launches)
        flops = sum(4.0 * h * hd * n * (n + 1) / 2 for n in n_list)
    elif args.kernel == "ln":
        rows, d = args.dims
        res = torch.randn(rows, d, device=dev, generator=g)
        delta = randn(rows, d)
        w = torch.ones(d, device=dev)
        bvec = torch.zeros(d, device=dev)
        ms = _timed(lambda: K.fused_add_layernorm(res, delta, w, bvec, 1e-5,
                                                  out_dtype=torch.float16, residual_out=res),
                    args.launches)
        flops = 0.0
    elif args.kernel == "gemm_ln":
        # GEMM + residual add + LayerNorm in one kernel, residual in place.
        m, n, k = args.dims
        a, w = randn(m, k), randn(n, k, scale=k ** -0.5)
        bias = torch.randn(n, device=dev, generator=g)
        res = torch.randn(m, n, device=dev, generator=g)
        gamma = torch.ones(n, device=dev)
        beta = torch.zeros(n, device=dev)
        out = torch.empty(m, n, dtype=torch.float16, device=dev)
        ws = K.gemm_add_layernorm_workspace(m, n, dev)
        ms = _timed(lambda: K.gemm_add_layernorm(a, w, bias, res, gamma, beta, 1e-5,
                                                 residual_out=res, out=out, workspace=ws),
                    args.launches)
        flops = 2.0 * m * n * k
    else:
        t, d, f = args.dims
        h = randn(t, d)
        w1, w2 = randn(f, d, scale=d ** -0.5), randn(d, f, scale=f ** -0.5)
        b1 = torch.zeros(f, device=dev)
        b2 = torch.zeros(d, device=dev)
        ms = _timed(lambda: K.fused_ffn(h, w1, b1, w2, b2, out_dtype=torch.float16),
                    args.launches)
        flops = 4.0 * t * d * f
    rate = f"  {flops / ms / 1e9:.0f} TFLOP/s" if flops else ""
    print(f"{args.kernel} {args.dims}: {ms * 1e3:.1f} us{rate}")
    return 0


if __name__ == "__main__":
    sys.exit(main())

#!/usr/bin/env python3
"""Forward tokens/s of the sm_100a tjkernels engine (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl tjb|reference]

Workload (``--config``, default 2): the BASELINE configs of the fused causal
encoder forward.  Each GPU runs a full config-sized batch (weak scaling: the
per-GPU work is fixed and N GPUs process N times the sequences, with no
collective in the forward; sequences are independent): every rank gets the
same seeded set of prefix lengths (its own data), so the per-GPU work is the
same at every N.  Inputs are synthetic tensors with the harness's shapes and
padding distribution (``generate_random_case``), weights the harness's
default initialisation.

One step = one ``model(x, mask)`` call through the harness hook (the engine,
CUDA-graph replay included), exactly what the reference harness times.
L2 is flushed (a 256 MiB write) between timed steps, outside the timed
events.  ``value`` = all ranks' tokens / max-over-ranks time.

Also reported on the same JSON line (scatter_gather only at N > 1: the same
steps with the inputs on GPU 0, each step scattering the shards over NVLink
and gathering the outputs back):
  e2e       the same call fed from pinned host memory: host->device copy of x
            and the mask, forward, device->host copy of the output, all timed.
  roofline  the dominant kernel (the tcgen05 GEMM) timed live with CUDA
            events in an instrumented eager pass over the same input, the
            plan's kernel families unfused (``kernels``); ``kernels_plan``
            times the plan's own kernels (the fused GEMM + LayerNorm among
            them) the same way, and gives the launch count.
  gpu_launches  library kernels launched in the timed steps (the plan's
            launches per forward times the steps).
  cpu_baseline  the reference PyTorch CPU forward (the fp32 oracle
            restatement) on a bounded sample, rank 0 at N=1.
  clocks    SM clock median and throttle reasons sampled during the timed
            region (NVML).
``--impl reference`` times the reference's CPU forward alone (rank 0 only).
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "tiktok-techjam-2026_b200"))

# cfg -> (batch, seq, d_model, heads, ffn, layers, padding_ratio); BASELINE.json configs.
CONFIGS = {
    0: (2, 128, 512, 8, 2048, 4, 0.5),
    1: (1, 64, 768, 12, 3072, 4, 0.0),
    2: (8, 1024, 1024, 16, 4096, 4, 1.0 - 1.0 / 1024),
    3: (4, 4096, 1024, 16, 4096, 4, 0.5),
    4: (8, 2048, 4096, 32, 16384, 12, 0.5),  # per-GPU shard of the B=64 job
}
CONFIG_NOTE = {
    0: "config0 B2 S128 d512 H8 F2048 L4, prefix padding U[64,128]",
    1: "config1 B1 S64 d768 H12 F3072 L4, no padding",
    2: "config2 B8 S1024 d1024 H16 F4096 L4, prefix padding U[1,1024]",
    3: "config3 B4 S4096 d1024 H16 F4096 L4, prefix padding U[2048,4096]",
    4: "config4 shard B8 (of 64) S2048 d4096 H32 F16384 L12, padding U[1024,2048]",
}
METRIC = "forward tokens/sec"
FLUSH_BYTES = 256 << 20


def synthetic_case(b, s, d, seed, padding, rank=0, world=1):
    """This rank's batch: b sequences with prefix lengths uniform in
    [max(1, round(S(1-p))), S] (the harness's generate_random_case), drawn
    once from ``seed`` and the same on every rank, so that each GPU does the
    same work at any N (weak scaling measures the system, not the draw);
    x ~ N(0,1) per sequence, seeded by its global index rank*b + i, zero on
    padded rows."""
    gen = torch.Generator(device="cpu")
    gen.manual_seed(seed)
    if padding <= 0:
        lengths = torch.full((b,), s, dtype=torch.long)
    else:
        min_valid = max(1, int(round(s * (1.0 - padding))))
        lengths = torch.randint(low=min_valid, high=s + 1, size=(b,), generator=gen)
    xs = []
    for i in range(b):
        g = torch.Generator(device="cpu")
        g.manual_seed(seed + 1 + rank * b + i)
        xs.append(torch.randn(s, d, generator=g, dtype=torch.float32))
    x = torch.stack(xs)
    mask = torch.arange(s)[None, :] < lengths[:, None]
    return x.masked_fill(~mask[..., None], 0), mask


def layer_flops(b, s, d, h, f, lengths):
    """Algorithmic FLOPs of one layer: GEMMs on the full padded shape,
    causal attention on the valid lower triangle."""
    t = b * s
    hd = d // h
    qkv, out, ffn = 6.0 * t * d * d, 2.0 * t * d * d, 4.0 * t * d * f
    attn = sum(4.0 * h * hd * n * (n + 1) / 2 for n in lengths)
    return qkv, out, ffn, attn


def load_peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {"hbm_gbs": p["hbm_gbs"], "tflops": p["bf16_tflops"],
                "tflops_sustained": p["bf16_tflops_sustained"], "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0,
            "source": "fallback"}


class ClockSampler:
    """Samples SM clock and throttle reasons every 20 ms through NVML."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
               "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index: int) -> None:
        self.samples = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception as exc:  # reading clocks is best effort
            self._nv = None
            self.error = str(exc)

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            self._stop.wait(0.02)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [],
                    "samples": 0}
        mhz = statistics.median(s[0] for s in self.samples)
        seen = set()
        for _, mask in self.samples:
            for name, bit in self.REASONS.items():
                if mask & bit:
                    seen.add(name)
        return {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": sorted(seen),
                "samples": len(self.samples)}


class KernelTimer:
    """Wraps the kernel facade so each library call is bracketed by CUDA
    events on the stream it launches on (eager mode only)."""

    def __init__(self, K, cfg):
        self.K = K
        self.cfg = cfg
        self.records = []  # (name, start_event, end_event, flops, bytes, launches)
        self._orig = {}

    def _wrap(self, name, fn, cost):
        def wrapped(*args, **kwargs):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kwargs)
            e.record()
            flops, nbytes, launches = cost(args, kwargs, out)
            self.records.append((name, s, e, flops, nbytes, launches))
            return out
        return wrapped

    def __enter__(self):
        K = self.K

        # FLOPs are counted on the rows that carry tokens: all rows without a
        # tile list, the valid tokens (sum of lengths) when dead tiles are
        # skipped -- the work the caller asked for, never the rows skipped.
        def rows_of(a, kwargs):
            return self.cfg["valid_tokens"] if kwargs.get("m_tiles") is not None else a.shape[0]

        def gemm_cost(args, kwargs, out):
            a, w = args[0], args[1]
            return 2.0 * rows_of(a, kwargs) * a.shape[1] * w.shape[0], 0.0, 1

        def ffn_cost(args, kwargs, out):
            h, w1 = args[0], args[1]
            return 4.0 * rows_of(h, kwargs) * h.shape[1] * w1.shape[0], 0.0, 2

        def ln_cost(args, kwargs, out):
            res, delta = args[0], args[1]
            n = rows_of(res, kwargs) * res.shape[1]
            nbytes = n * 4 + (0 if delta is None else n * delta.element_size())
            if delta is not None and kwargs.get("write_residual", True):
                nbytes += n * 4
            nbytes += n * out[1].element_size()
            return 0.0, float(nbytes), 1

        def attn_cost(args, kwargs, out):
            qkv = args[0]
            b, s, _, h, hd = qkv.shape
            lengths = self.cfg["lengths"]
            return sum(4.0 * h * hd * n * (n + 1) / 2 for n in lengths), 0.0, 1

        def mask_cost(args, kwargs, out):
            return 0.0, 0.0, 1

        for name, cost in (("gemm_bias", gemm_cost), ("fused_ffn", ffn_cost),
                           ("gemm_add_layernorm", gemm_cost),
                           ("fused_add_layernorm", ln_cost), ("flash_attention", attn_cost),
                           ("mask_lengths", mask_cost), ("row_tiles", mask_cost)):
            self._orig[name] = getattr(K, name)
            setattr(K, name, self._wrap(name, self._orig[name], cost))
        return self

    def __exit__(self, *exc):
        for name, fn in self._orig.items():
            setattr(self.K, name, fn)

    def summary(self, steps):
        torch.cuda.synchronize()
        agg = {}
        for name, s, e, flops, nbytes, launches in self.records:
            a = agg.setdefault(name, {"ms": 0.0, "flops": 0.0, "bytes": 0.0, "calls": 0,
                                      "launches": 0})
            a["ms"] += s.elapsed_time(e)
            a["flops"] += flops
            a["bytes"] += nbytes
            a["calls"] += 1
            a["launches"] += launches
        out = {}
        for name, a in agg.items():
            sec = a["ms"] / 1e3
            out[name] = {
                "ms_per_step": a["ms"] / steps,
                "calls_per_step": a["calls"] / steps,
                "launches_per_step": a["launches"] / steps,
                "tflops": a["flops"] / sec / 1e12 if a["flops"] else None,
                "gbs": a["bytes"] / sec / 1e9 if a["bytes"] else None,
                "flops_per_call": a["flops"] / a["calls"],
                "ms_per_call": a["ms"] / a["calls"],
            }
        return out


def cpu_forward_rate(cfg_id, sample_batch, sample_layers, calls, seed=100000):
    """Reference CPU forward (fp32 oracle restatement of BaselineTransformer)
    on a bounded sample; returns (tokens/s for the full-depth forward, info)."""
    from oracle.model import ModelConfig, build_model, generate_case

    b, s, d, h, f, layers, pad = CONFIGS[cfg_id]
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = ModelConfig(sample_batch, s, d, h, f, sample_layers, True)
    model = build_model(cfg, 0)
    x, mask = generate_case(cfg, seed, pad)
    torch.set_float32_matmul_precision("highest")
    times = []
    with torch.inference_mode():
        model(x, mask)  # warm-up
        for _ in range(calls):
            t0 = time.perf_counter_ns()
            model(x, mask)
            times.append((time.perf_counter_ns() - t0) / 1e9)
    sec = statistics.median(times) * layers / sample_layers
    tokens = sample_batch * s
    info = {
        "cores": torch.get_num_threads(),
        "sample": f"{sample_batch} sequence(s) x S={s}, {sample_layers} of {layers} layers "
                  f"(time scaled to {layers}), median of {calls} call(s) after 1 warm-up",
    }
    return tokens / sec, info


def cpu_sample_plan(cfg_id):
    """(batch, layers, calls) so one sample costs a few seconds on the host."""
    return {0: (2, 4, 5), 1: (1, 4, 5), 2: (1, 4, 3), 3: (1, 1, 2), 4: (1, 1, 1)}[cfg_id]


def run_reference(args, rank, world):
    if rank != 0:
        return
    b, s, d, h, f, layers, pad = CONFIGS[args.config]
    sb, sl, _ = cpu_sample_plan(args.config)
    rates, info = [], None
    for i in range(args.warmup + args.steps):
        rate, info = cpu_forward_rate(args.config, sb, sl, 1, seed=100000 + i)
        if i >= args.warmup:
            rates.append(rate)
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": b * s / value * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args.config, world),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": info["cores"],
                         "kind": "port", "sample": info["sample"]},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def workload_config(cfg_id, world, tp=False):
    b, s, d, h, f, layers, pad = CONFIGS[cfg_id]
    if tp:
        return {"workload": CONFIG_NOTE[cfg_id] + f" over {world} GPUs", "global_batch": b,
                "seq_len": s, "d_model": d, "heads": h, "ffn_dim": f, "layers": layers,
                "parallelism": f"tp{world}: heads and FFN columns split, NCCL all-reduce "
                               "of the partial sums (in the plan's delta dtype) after the "
                               "out-projection and FFN-out",
                "l2": "flushed between timed steps (256 MiB write, untimed)"}
    return {"workload": CONFIG_NOTE[cfg_id] + " per GPU", "global_batch": b * world,
            "seq_len": s, "d_model": d, "heads": h, "ffn_dim": f, "layers": layers,
            "parallelism": f"dp{world} batch-sharded, no collective in the forward",
            "l2": "flushed between timed steps (256 MiB write, untimed)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="tjb", choices=["tjb", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp", action="store_true",
                    help="tensor-parallel over the N GPUs (strong scaling) instead of "
                         "batch sharding")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch.distributed as dist
    import tjkernels
    import tjkernels.kernels as K
    from tjkernels import plans
    from tjkernels.model import Encoder, EncoderConfig

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))

    b, s, d, h, f, layers, pad = CONFIGS[args.config]
    cfg = EncoderConfig(b, s, d, h, f, layers, True)
    torch.manual_seed(0)
    model = Encoder(cfg).to(dev).eval()
    tp = args.tp and world > 1
    if tp:
        from tjkernels.parallel import enable_tensor_parallel
        enable_tensor_parallel(model)
    x_cpu, mask_cpu = synthetic_case(b, s, d, 100000, pad, 0 if tp else rank, 1 if tp else world)
    x, mask = x_cpu.to(dev), mask_cpu.to(dev)
    lengths = mask_cpu.sum(-1).tolist()
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    with torch.inference_mode():
        for _ in range(args.warmup):
            model(x, mask)
        torch.cuda.synchronize(dev)
        plan = tjkernels.get_engine(model).plan

        # ----------------------------------------------------- timed region
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(local) as clocks:
            for i in range(args.steps):
                starts[i].record(stream)
                model(x, mask)
                ends[i].record(stream)
                flush.zero_()
            torch.cuda.synchronize(dev)
        barrier()
        step_ms = sum(a.elapsed_time(e) for a, e in zip(starts, ends)) / args.steps

        # ------------------------------------------------------- end to end
        # Every step copies its input from pinned host memory and reads its
        # output back, through the public call model(x, mask).  The copies run
        # on their own streams with two buffer sets, so step i+1's upload and
        # step i-1's download overlap step i's forward (what a serving loop
        # does); the L2 flush between forwards stays inside the timed region.
        x_host = x_cpu.pin_memory()
        m_host = mask_cpu.pin_memory()
        depth = 2
        out_host = [torch.empty((b, s, d), dtype=torch.float32).pin_memory() for _ in range(depth)]
        x_dev = [torch.empty_like(x) for _ in range(depth)]
        m_dev = [torch.empty_like(mask) for _ in range(depth)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(depth)]
        ev_comp = [torch.cuda.Event() for _ in range(depth)]

        def e2e_steps(n):
            for i in range(n):
                k = i % depth
                with torch.cuda.stream(s_in):
                    if i >= depth:
                        s_in.wait_event(ev_comp[k])  # forward i-2 is done with x_dev[k]
                    x_dev[k].copy_(x_host, non_blocking=True)
                    m_dev[k].copy_(m_host, non_blocking=True)
                    ev_in[k].record(s_in)
                stream.wait_event(ev_in[k])
                out = model(x_dev[k], m_dev[k])
                ev_comp[k].record(stream)
                flush.zero_()
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_comp[k])
                    out_host[k].copy_(out, non_blocking=True)
                    out.record_stream(s_out)

        e2e_steps(2 * depth)
        torch.cuda.synchronize(dev)
        e_start = torch.cuda.Event(enable_timing=True)
        e_end = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        e_start.record(s_in)
        s_out.wait_event(e_start)
        stream.wait_event(e_start)
        e2e_steps(args.steps)
        e_end.record(s_out)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = e_start.elapsed_time(e_end) / args.steps

        # ------------------------- scatter/gather from GPU 0 (N > 1 only)
        # The same steps with the inputs starting on GPU 0: each step
        # scatters the ranks' shards over NVLink (NCCL), runs the forward on
        # every GPU and gathers the outputs back to GPU 0.
        sg_ms = 0.0
        if world > 1 and not tp:
            x_all = None
            out_all = None
            if rank == 0:
                x_all = [synthetic_case(b, s, d, 100000, pad, r, world)[0].to(dev)
                         for r in range(world)]
                out_all = [torch.empty((b, s, d), dtype=torch.float32, device=dev)
                           for _ in range(world)]
            x_sg = torch.empty_like(x)

            def sg_step():
                dist.scatter(x_sg, x_all, src=0)
                dist.gather(model(x_sg, mask), out_all, dst=0)

            for _ in range(2):
                sg_step()
            torch.cuda.synchronize(dev)
            barrier()
            sg_start = torch.cuda.Event(enable_timing=True)
            sg_end = torch.cuda.Event(enable_timing=True)
            sg_start.record(stream)
            for _ in range(args.steps):
                sg_step()
                flush.zero_()
            sg_end.record(stream)
            torch.cuda.synchronize(dev)
            barrier()
            sg_ms = sg_start.elapsed_time(sg_end) / args.steps
            del x_all, out_all

        # -------------------------------------- per-kernel timing (eager)
        ksteps = max(3, min(args.steps, 20))
        # Per-kernel rates come from the unfused form of the plan (each
        # kernel family on its own: GEMMs, attention, FFN, LayerNorm); the
        # launch count and the rates of the plan's own kernels (the fused
        # GEMM + LayerNorm among them) from eager forwards of the plan itself.
        plans.set_override(plans.Plan(compute_dtype=plan.compute_dtype,
                                      delta_dtype=plan.delta_dtype, cuda_graph=False,
                                      fuse_layernorm=False, label="instrumented"))
        model(x, mask)
        torch.cuda.synchronize(dev)
        timer = KernelTimer(K, {"lengths": lengths, "valid_tokens": sum(lengths)})
        with timer:
            for _ in range(ksteps):
                model(x, mask)
                flush.zero_()
        kern = timer.summary(ksteps)
        plans.set_override(dataclasses.replace(plan, cuda_graph=False))
        model(x, mask)
        torch.cuda.synchronize(dev)
        counter = KernelTimer(K, {"lengths": lengths, "valid_tokens": sum(lengths)})
        with counter:
            for _ in range(ksteps):
                model(x, mask)
                flush.zero_()
        kern_plan = counter.summary(ksteps)
        launches_real = sum(v["launches_per_step"] for v in kern_plan.values())
        plans.set_override(None)

    status_local = float(K.device_status(clear=True))  # synchronises; after all timing
    step_max, e2e_max, sg_max, status_max = max_over_ranks([step_ms, e2e_ms, sg_ms,
                                                            status_local])
    device_status = int(status_max)
    launches_per_step = launches_real

    if rank == 0:
        peaks = load_peaks()
        tokens = b * s * (1 if tp else world)
        value = tokens / (step_max / 1e3)
        gemm_ms = (kern["gemm_bias"]["ms_per_step"] + kern["fused_ffn"]["ms_per_step"])
        gemm_flops = (kern["gemm_bias"]["flops_per_call"] * kern["gemm_bias"]["calls_per_step"]
                      + kern["fused_ffn"]["flops_per_call"] * kern["fused_ffn"]["calls_per_step"])
        gemm_launches = (kern["gemm_bias"]["launches_per_step"]
                         + kern["fused_ffn"]["launches_per_step"])
        achieved = gemm_flops / (gemm_ms / 1e3) / 1e12
        peak = peaks["tflops_sustained"]
        attn = kern["flash_attention"]
        ln = kern["fused_add_layernorm"]
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_max,
            "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": {torch.float16: "f16", torch.bfloat16: "bf16"}[plan.compute_dtype],
            "data": "synthetic (seeded N(0,1) inputs, default-init weights)",
            "config": dict(workload_config(args.config, world, tp),
                           plan=plan.to_json()),
            "roofline": {
                "bound": "tensor", "kernel": "gemm_kernel (tcgen05, all GEMM launches)",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_note": f"{peaks['source']} sustained bf16/f16 dense "
                             f"(burst {peaks['tflops']})",
                "flops_per_launch": gemm_flops / gemm_launches,
                "ms_per_launch": gemm_ms / gemm_launches,
                "traffic": None,
                "attn_tflops": attn["tflops"], "attn_frac": attn["tflops"] / peak,
                "ffn_tflops": kern["fused_ffn"]["tflops"],
                "ffn_frac": kern["fused_ffn"]["tflops"] / peak,
                # The plan's fused GEMM + add + LayerNorm (when it runs one).
                "gemm_ln_tflops": kern_plan.get("gemm_add_layernorm", {}).get("tflops"),
                "layernorm_gbs": ln["gbs"], "layernorm_frac": ln["gbs"] / peaks["hbm_gbs"],
                "eager_step_ms": sum(v["ms_per_step"] for v in kern.values()),
            },
            "kernels": kern,
            "kernels_plan": kern_plan,
            "e2e": {"value": tokens / (e2e_max / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_cpu.numel() * 4 + mask_cpu.numel(),
                    "d2h_bytes_per_step": b * s * d * 4, "ms_per_step": e2e_max,
                    "overlap": "uploads and downloads on two copy streams, 2 buffer sets; "
                               "L2 flush between forwards included"},
            "gpu_launches": int(round(launches_per_step * args.steps)),
            "clocks": clocks.summary(),
            # Sticky device status word: nonzero if any kernel's bounded wait
            # ran out during the run (the numbers are then not valid).
            "device_status": device_status,
        }
        if world > 1 and not tp:
            line["scatter_gather"] = {
                "value": tokens / (sg_max / 1e3), "unit": "tokens/s", "ms_per_step": sg_max,
                "bytes_per_step": 2 * (world - 1) * b * s * d * 4,
                "note": "inputs start on GPU 0; per step NCCL scatter of the shards and "
                        "gather of the outputs, max over ranks"}
        if device_status != 0:
            print(json.dumps(line), flush=True)
            raise SystemExit(f"a kernel recorded device status {device_status} "
                             "(bounded wait ran out): run invalid")
        if world == 1 and not args.no_cpu_baseline:
            sb, sl, calls = cpu_sample_plan(args.config)
            rate, info = cpu_forward_rate(args.config, sb, sl, calls)
            line["cpu_baseline"] = {"value": rate, "unit": "tokens/s", "cores": info["cores"],
                                    "kind": "port", "sample": info["sample"]}
        print(json.dumps(line), flush=True)

    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

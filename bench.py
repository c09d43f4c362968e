#!/usr/bin/env python3
"""Forward tokens/s of the sm_100a tjkernels engine (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--impl tjb|reference|reference-gpu]
    python bench.py --kernel KIND DIMS... [options]     (one kernel, see below)

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
  roofline  the dominant kernel of the plan that was timed (the tcgen05 GEMM,
            ``gemm_kernel``), each of its launches bracketed by CUDA events in
            eager forwards of that same plan over the same input; divided by
            the measured BURST peak (the launches are tens of microseconds
            inside a short eager pass).  ``kernels_plan`` gives every kernel
            family of the plan the same way, ``gemm_shapes`` the GEMM per
            shape.
  gpu_launches  library kernels launched in the timed steps (the plan's
            launches per forward times the steps).
  cpu_baseline  the reference PyTorch CPU forward (the fp32 oracle
            restatement) on a bounded sample, rank 0 at N=1.
  clocks    SM clock median and throttle reasons sampled during the timed
            region (NVML).

``--impl reference`` times the reference's CPU forward alone (rank 0 only),
on a bounded sample of the workload (one sequence), and reports what it
timed.  ``--impl reference-gpu`` runs the reference's own GPU path -- its
``tjkernels`` engine (Triton attention and LayerNorm, cuBLAS GEMMs, its CUDA
graph), unmodified, from ``baseline/_ref`` -- on the same workload through
the harness's ``UserOptimizedTransformer``, and times its Triton attention
(``flash_attention``) and add+LayerNorm (``fused_add_layernorm``) kernels at
the config's shapes; ``--kernel attn|ln`` times this build's kernels at the
same shapes the same way.

``--kernel`` runs one library kernel on seeded fp16 inputs of a given shape,
``--launches`` times with the L2 flushed before each, and prints the median
CUDA-event time of all but the first launch (the command the single-kernel
ncu captures are taken with):
    --kernel gemm M N K [--act gelu] [--out f16|f32] [--stream-k]
    --kernel attn B S H HD [--lengths full|prefix]
    --kernel ln ROWS D
    --kernel ffn T D F            (two launches)
    --kernel ffn_single T D F     (one kernel, hidden on chip; d <= 1024)
    --kernel gemm_ln M N K
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import sys
import types
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
PKG_DIR = ROOT / "tiktok-techjam-2026_b200"
REF_DIR = ROOT / "baseline" / "_ref"

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

# DRAM traffic of the dominant kernel family (the tcgen05 GEMM) per launch, averaged over
# the launches of one forward of the config's tuned plan: sum of
# dram__bytes_read.sum + dram__bytes_write.sum over those launches / their
# number, from one ncu capture of this bench's own command (a one-pass
# metric set on the full workload).  None where no capture was taken.
# Config 2: 12 launches, all on CTA pairs: QKV and FFN1 (17.7-18.1 and
# 20.1-20.8 MB), FFN2 with stream-K over the pairs (64.4-68.4 MB); the
# outputs mostly stay in the 126 MB L2 during a launch, so the figure sits
# below the algorithmic bytes (A + W read, C written).
GEMM_TRAFFIC_PER_LAUNCH = {2: 34.73e6}


def use_package() -> None:
    if str(PKG_DIR) not in sys.path:
        sys.path.insert(0, str(PKG_DIR))


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
        # (name, shape, start_event, end_event, flops, bytes, launches)
        self.records = []
        self._orig = {}

    def _wrap(self, name, fn, cost):
        def wrapped(*args, **kwargs):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kwargs)
            e.record()
            flops, nbytes, launches, shape = cost(args, kwargs, out)
            self.records.append((name, shape, s, e, flops, nbytes, launches))
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
            shape = f"M{a.shape[0]} N{w.shape[0]} K{a.shape[1]}"
            return 2.0 * rows_of(a, kwargs) * a.shape[1] * w.shape[0], 0.0, 1, shape

        def ffn_cost(args, kwargs, out):
            h, w1 = args[0], args[1]
            shape = f"T{h.shape[0]} d{h.shape[1]} F{w1.shape[0]}"
            return 4.0 * rows_of(h, kwargs) * h.shape[1] * w1.shape[0], 0.0, 2, shape

        def ln_cost(args, kwargs, out):
            res, delta = args[0], args[1]
            n = rows_of(res, kwargs) * res.shape[1]
            nbytes = n * 4 + (0 if delta is None else n * delta.element_size())
            if delta is not None and kwargs.get("write_residual", True):
                nbytes += n * 4
            nbytes += n * out[1].element_size()
            return 0.0, float(nbytes), 1, f"rows{res.shape[0]} d{res.shape[1]}"

        def attn_cost(args, kwargs, out):
            qkv = args[0]
            b, s, _, h, hd = qkv.shape
            lengths = self.cfg["lengths"]
            flops = sum(4.0 * h * hd * n * (n + 1) / 2 for n in lengths)
            return flops, 0.0, 1, f"B{b} S{s} H{h} hd{hd}"

        def mask_cost(args, kwargs, out):
            return 0.0, 0.0, 1, ""

        def small_cost(args, kwargs, out):
            # The whole forward in one launch: GEMM FLOPs on the valid tokens
            # plus causal attention; bytes = parameters + input + output.
            model, x, heads = args[0], args[1], args[3]
            b, s, d = x.shape
            hd = d // heads
            lengths = self.cfg["lengths"]
            flops = 2.0 * sum(lengths) * model.gemm_params
            flops += model.count * sum(4.0 * heads * hd * n * (n + 1) / 2 for n in lengths)
            nbytes = float(model.param_bytes + 2 * x.numel() * 4)
            return flops, nbytes, 1, f"B{b} S{s} d{d} L{model.count}"

        for name, cost in (("gemm_bias", gemm_cost), ("fused_ffn", ffn_cost),
                           ("gemm_add_layernorm", gemm_cost),
                           ("fused_add_layernorm", ln_cost), ("flash_attention", attn_cost),
                           ("mask_lengths", mask_cost), ("row_tiles", mask_cost),
                           ("mask_lengths_tiles", mask_cost), ("forward_small", small_cost)):
            self._orig[name] = getattr(K, name)
            setattr(K, name, self._wrap(name, self._orig[name], cost))
        return self

    def __exit__(self, *exc):
        for name, fn in self._orig.items():
            setattr(self.K, name, fn)

    @staticmethod
    def _aggregate(records, key):
        agg = {}
        for rec in records:
            name, shape, s, e, flops, nbytes, launches = rec
            a = agg.setdefault(key(rec), {"ms": 0.0, "flops": 0.0, "bytes": 0.0, "calls": 0,
                                          "launches": 0})
            a["ms"] += s.elapsed_time(e)
            a["flops"] += flops
            a["bytes"] += nbytes
            a["calls"] += 1
            a["launches"] += launches
        return agg

    @staticmethod
    def _rates(agg, steps):
        out = {}
        for k, a in agg.items():
            sec = a["ms"] / 1e3
            out[k] = {
                "ms_per_step": a["ms"] / steps,
                "calls_per_step": a["calls"] / steps,
                "launches_per_step": a["launches"] / steps,
                "tflops": a["flops"] / sec / 1e12 if a["flops"] else None,
                "gbs": a["bytes"] / sec / 1e9 if a["bytes"] else None,
                "flops_per_call": a["flops"] / a["calls"],
                "bytes_per_call": a["bytes"] / a["calls"],
                "ms_per_call": a["ms"] / a["calls"],
            }
        return out

    def summary(self, steps):
        torch.cuda.synchronize()
        return self._rates(self._aggregate(self.records, lambda r: r[0]), steps)

    def gemm_shapes(self, steps):
        """gemm_kernel launches (gemm_bias calls) per shape."""
        recs = [r for r in self.records if r[0] == "gemm_bias"]
        return self._rates(self._aggregate(recs, lambda r: r[1]), steps)


# ---------------------------------------------------------------- CPU reference

def cpu_reference_model(cfg_id, sample_batch, sample_layers):
    """The reference CPU forward (fp32 oracle restatement of
    BaselineTransformer) on a bounded sample of the config: ``sample_batch``
    sequences and ``sample_layers`` of its layers.  Built once."""
    from oracle.model import ModelConfig, build_model

    b, s, d, h, f, layers, pad = CONFIGS[cfg_id]
    torch.set_num_threads(os.cpu_count() or 1)
    torch.set_float32_matmul_precision("highest")
    cfg = ModelConfig(sample_batch, s, d, h, f, sample_layers, True)
    return cfg, build_model(cfg, 0)


def cpu_sample_plan(cfg_id):
    """(batch, layers, calls) so one sample costs a few seconds on the host."""
    return {0: (2, 4, 5), 1: (1, 4, 5), 2: (1, 4, 3), 3: (1, 1, 2), 4: (1, 1, 1)}[cfg_id]


def cpu_forward_rate(cfg_id, calls, seed=100000):
    """tokens/s of the full-depth forward, from the bounded sample's median
    time scaled by layers / sample layers; returns (rate, info)."""
    from oracle.model import generate_case

    b, s, d, h, f, layers, pad = CONFIGS[cfg_id]
    sb, sl, _ = cpu_sample_plan(cfg_id)
    cfg, model = cpu_reference_model(cfg_id, sb, sl)
    x, mask = generate_case(cfg, seed, pad)
    times = []
    with torch.inference_mode():
        model(x, mask)  # warm-up
        for _ in range(calls):
            t0 = time.perf_counter_ns()
            model(x, mask)
            times.append((time.perf_counter_ns() - t0) / 1e9)
    sec = statistics.median(times) * layers / sl
    info = {
        "cores": torch.get_num_threads(),
        "sample": f"{sb} sequence(s) x S={s}, {sl} of {layers} layers "
                  f"(time scaled to {layers}), median of {calls} call(s) after 1 warm-up",
    }
    return sb * s / sec, info


def run_reference(args, rank, world):
    """The reference arm: the reference's CPU forward on the host cores, rank
    0 only.  Each step is one forward of the bounded sample (built once);
    ``steps``/``ms_per_step`` describe exactly those timed forwards, and
    ``value`` is their tokens/s scaled to the full depth."""
    if rank != 0:
        return
    from oracle.model import generate_case

    b, s, d, h, f, layers, pad = CONFIGS[args.config]
    sb, sl, _ = cpu_sample_plan(args.config)
    cfg, model = cpu_reference_model(args.config, sb, sl)
    x, mask = generate_case(cfg, 100000, pad)
    times = []
    with torch.inference_mode():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter_ns()
            model(x, mask)
            if i >= args.warmup:
                times.append((time.perf_counter_ns() - t0) / 1e9)
    ms_sample = statistics.median(times) * 1e3
    value = sb * s / (ms_sample / 1e3 * layers / sl)
    sample = (f"{sb} sequence(s) x S={s}, {sl} of {layers} layers per step "
              f"(tokens/s scaled to {layers} layers), model built once")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_sample, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(workload_config(args.config, world),
                       timed_step=f"one CPU forward of the sample: {sample}"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
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


# ---------------------------------------------------------------- shared timing

def time_launches(fn, launches, flush=None):
    """Median CUDA-event time (ms) of launches 2..n of ``fn`` (the first is a
    warm-up); the L2 is flushed before each launch when ``flush`` is given."""
    fn()
    times = []
    for _ in range(max(1, launches - 1)):
        if flush is not None:
            flush.zero_()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end))
    return sorted(times)[len(times) // 2]


def timed_steps(fwd, x, mask, steps, stream, flush):
    """Mean device time (ms) of ``steps`` calls of fwd(x, mask), each
    bracketed by CUDA events, L2 flushed between them (outside the events)."""
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    for i in range(steps):
        starts[i].record(stream)
        fwd(x, mask)
        ends[i].record(stream)
        flush.zero_()
    torch.cuda.synchronize()
    return sum(a.elapsed_time(e) for a, e in zip(starts, ends)) / steps


def e2e_leg(fwd, x_cpu, mask_cpu, steps, dev, stream, flush, barrier):
    """Per-step ms of fwd fed from pinned host memory: every step copies its
    input in and its output back, inside the timed region.  The copies run on
    their own streams with two buffer sets, so step i+1's upload and step
    i-1's download overlap step i's forward (what a serving loop does); the
    L2 flush between forwards stays inside the timed region."""
    x_host = x_cpu.pin_memory()
    m_host = mask_cpu.pin_memory()
    depth = 2
    out_host = [torch.empty(x_cpu.shape, dtype=torch.float32).pin_memory()
                for _ in range(depth)]
    x_dev = [torch.empty(x_cpu.shape, dtype=x_cpu.dtype, device=dev) for _ in range(depth)]
    m_dev = [torch.empty(mask_cpu.shape, dtype=mask_cpu.dtype, device=dev)
             for _ in range(depth)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(depth)]
    ev_comp = [torch.cuda.Event() for _ in range(depth)]

    def run(n):
        for i in range(n):
            k = i % depth
            with torch.cuda.stream(s_in):
                if i >= depth:
                    s_in.wait_event(ev_comp[k])  # forward i-2 is done with x_dev[k]
                x_dev[k].copy_(x_host, non_blocking=True)
                m_dev[k].copy_(m_host, non_blocking=True)
                ev_in[k].record(s_in)
            stream.wait_event(ev_in[k])
            out = fwd(x_dev[k], m_dev[k])
            ev_comp[k].record(stream)
            flush.zero_()
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_comp[k])
                out_host[k].copy_(out, non_blocking=True)
                out.record_stream(s_out)

    run(2 * depth)
    torch.cuda.synchronize(dev)
    e_start = torch.cuda.Event(enable_timing=True)
    e_end = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    e_start.record(s_in)
    s_out.wait_event(e_start)
    stream.wait_event(e_start)
    run(steps)
    e_end.record(s_out)
    torch.cuda.synchronize(dev)
    barrier()
    return e_start.elapsed_time(e_end) / steps


class PeerBuffers:
    """GPU 0's scatter/gather buffers mapped into every rank (CUDA IPC), so
    that each rank's copy engine pulls its input shard from GPU 0 and pushes
    its output shard back over NVLink with plain cudaMemcpyAsync calls: no
    SM of GPU 0 is taken from its own forward, as an NCCL scatter/gather
    kernel would.  Rank 0 owns one cudaMalloc block for the inputs of every
    rank and one for `depth` sets of outputs; the others open their handles
    in their own device's context (peer access over NVLink).  `ok` is False
    on every rank when any rank failed to set up (the caller then uses
    NCCL); every rank takes the same collective steps either way."""

    def __init__(self, dist, rank, world, dev, shard_bytes, depth, inputs):
        self.rank, self.world, self.shard, self.depth = rank, world, shard_bytes, depth
        self.ok = False
        self.x_base = self.o_base = None
        self._owned = []
        self._opened = []
        try:
            from cuda.bindings import runtime as rt
        except Exception:
            rt = None
        self.rt = rt
        handles = [None, None]
        # BENCH_SG_NCCL=1 keeps the NCCL scatter/gather (for comparisons).
        good = rt is not None and os.environ.get("BENCH_SG_NCCL") != "1"
        if rank == 0 and good:
            try:
                for i, nbytes in enumerate((world * shard_bytes, depth * world * shard_bytes)):
                    err, ptr = rt.cudaMalloc(nbytes)
                    good = good and err == rt.cudaError_t.cudaSuccess
                    if not good:
                        break
                    self._owned.append(ptr)
                    err, h = rt.cudaIpcGetMemHandle(ptr)
                    good = good and err == rt.cudaError_t.cudaSuccess
                    handles[i] = bytes(h.reserved) if good else None
                if good:
                    self.x_base, self.o_base = self._owned
                    for r, t in enumerate(inputs):
                        (err,) = rt.cudaMemcpy(self.x_base + r * shard_bytes, t.data_ptr(),
                                               shard_bytes,
                                               rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice)
                        good = good and err == rt.cudaError_t.cudaSuccess
            except Exception:
                good = False
        box = [handles if good else None]
        dist.broadcast_object_list(box, src=0, device=dev)
        if rank != 0:
            good = rt is not None and box[0] is not None and os.environ.get("BENCH_SG_NCCL") != "1"
            if good:
                try:
                    bases = []
                    for raw in box[0]:
                        h = rt.cudaIpcMemHandle_t()
                        h.reserved = raw
                        err, ptr = rt.cudaIpcOpenMemHandle(h, rt.cudaIpcMemLazyEnablePeerAccess)
                        good = good and err == rt.cudaError_t.cudaSuccess
                        if not good:
                            break
                        self._opened.append(ptr)
                        bases.append(ptr)
                    if good:
                        self.x_base, self.o_base = bases
                except Exception:
                    good = False
        flag = torch.tensor([1 if good else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        self.ok = bool(flag.item())

    def pull_input(self, dst: torch.Tensor, stream: torch.cuda.Stream) -> None:
        rt = self.rt
        (err,) = rt.cudaMemcpyAsync(dst.data_ptr(), self.x_base + self.rank * self.shard,
                                    self.shard, rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                    stream.cuda_stream)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"peer input copy failed: {err}")

    def push_output(self, src: torch.Tensor, k: int, stream: torch.cuda.Stream) -> None:
        rt = self.rt
        dst = self.o_base + (k * self.world + self.rank) * self.shard
        (err,) = rt.cudaMemcpyAsync(dst, src.data_ptr(), self.shard,
                                    rt.cudaMemcpyKind.cudaMemcpyDeviceToDevice,
                                    stream.cuda_stream)
        if err != rt.cudaError_t.cudaSuccess:
            raise RuntimeError(f"peer output copy failed: {err}")

    def close(self, dist, dev) -> None:
        """Peers unmap first; rank 0 frees after a barrier."""
        torch.cuda.synchronize(dev)
        for ptr in self._opened:
            self.rt.cudaIpcCloseMemHandle(ptr)
        dist.barrier(device_ids=[dev.index])
        for ptr in self._owned:
            self.rt.cudaFree(ptr)
        self._opened, self._owned = [], []


# -------------------------------------------------------- reference GPU path

def run_reference_gpu(args, rank, world):
    """The reference's own GPU implementation on this GPU, unmodified: the
    harness's ``UserOptimizedTransformer`` whose forward is the reference's
    ``tjkernels.forward`` (default plan on CUDA: fp16 compute, Triton causal
    flash attention and add+LayerNorm, cuBLAS GEMMs, whole-forward graph when
    the input is <= 64 MB), imported from ``baseline/_ref`` in a process
    where this build's package is not on the path.  Rank 0 only."""
    if rank != 0:
        return
    if not (REF_DIR / "tjkernels").is_dir() or not (REF_DIR / "torch_transformer_benchmark.py").exists():
        print(json.dumps({"impl": "reference-gpu",
                          "unavailable": "baseline/_ref holds no install of the reference"}),
              flush=True)
        return
    sys.path[:] = [p for p in sys.path if Path(p or ".").resolve() != PKG_DIR]
    sys.path.insert(0, str(REF_DIR))
    import torch_transformer_benchmark as H  # the reference harness (imports its tjkernels)
    import tjkernels as ref_tj
    import tjkernels.kernels as ref_k
    if Path(ref_tj.__file__).resolve().parent.parent != REF_DIR.resolve():
        raise SystemExit(f"reference-gpu: imported tjkernels from {ref_tj.__file__}")

    b, s, d, h, f, layers, pad = CONFIGS[args.config]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    # The harness's defaults (TF32 on for fp32 matmuls: --allow-tf32).
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.backends.cudnn.allow_tf32 = True
    torch.manual_seed(0)
    model = H.UserOptimizedTransformer(H.TransformerConfig(b, s, d, h, f, layers, True))
    model = model.to(dev).eval()
    x_cpu, mask_cpu = synthetic_case(b, s, d, 100000, pad)
    x, mask = x_cpu.to(dev), mask_cpu.to(dev)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    with torch.inference_mode():
        for _ in range(args.warmup):
            model(x, mask)
        torch.cuda.synchronize()
        plan = ref_tj.get_engine(model).plan
        with ClockSampler(0) as clocks:
            step_ms = timed_steps(model, x, mask, args.steps, stream, flush)
        e2e_ms = e2e_leg(model, x_cpu, mask_cpu, args.steps, dev, stream, flush, lambda: None)

        # The reference's two Triton kernels at this config's shapes, full
        # lengths (its attention kernel has no length skipping), fp16.
        g = torch.Generator(device=dev).manual_seed(0)
        hd = d // h
        qkv = torch.randn(b, s, 3, h, hd, device=dev, generator=g).half()
        attn_ms = time_launches(lambda: ref_k.flash_attention(qkv, h, causal=True), 5, flush)
        attn_flops = b * 4.0 * h * hd * s * (s + 1) / 2
        res = torch.randn(b * s, d, device=dev, generator=g)
        delta = torch.randn(b * s, d, device=dev, generator=g).half()
        w, bvec = torch.ones(d, device=dev), torch.zeros(d, device=dev)
        ln_ms = time_launches(lambda: ref_k.fused_add_layernorm(
            res, delta, w, bvec, 1e-5, out_dtype=torch.float16), 5, flush)
        ln_bytes = b * s * d * (4 + 2 + 4 + 2)
    tokens = b * s
    line = {
        "impl": "reference-gpu", "metric": METRIC, "value": tokens / (step_ms / 1e3),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": str(plan.compute_dtype).replace("torch.", ""),
        "data": "synthetic (the same seeded inputs and default-init weights as this build's arm)",
        "config": dict(workload_config(args.config, 1), plan=plan.to_json()),
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": x_cpu.numel() * 4 + mask_cpu.numel(),
                "d2h_bytes_per_step": tokens * d * 4, "ms_per_step": e2e_ms},
        "kernels": {
            "flash_attention": {"shape": f"B{b} S{s} H{h} hd{hd} causal full lengths fp16",
                                "us": attn_ms * 1e3,
                                "tflops": attn_flops / (attn_ms / 1e3) / 1e12},
            "fused_add_layernorm": {"shape": f"rows{b * s} d{d} fp32 res, fp16 delta/out",
                                    "us": ln_ms * 1e3,
                                    "gbs": ln_bytes / (ln_ms / 1e3) / 1e9},
            "timing": "median of 4 launches after 1 warm-up, L2 flushed before each",
        },
        "clocks": clocks.summary(),
        "source": "reference tjkernels + harness, unmodified, from baseline/_ref",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- single kernel

def kernel_main(argv) -> int:
    """One library kernel on seeded fp16 inputs (the profiling driver)."""
    use_package()
    import tjkernels.kernels as K

    ap = argparse.ArgumentParser(prog="bench.py --kernel")
    ap.add_argument("kernel", choices=["gemm", "attn", "ln", "ffn", "ffn_single", "gemm_ln",
                                       "small"])
    ap.add_argument("dims", type=int, nargs="+")
    ap.add_argument("--act", choices=["none", "gelu"], default="none")
    ap.add_argument("--out", choices=["f16", "f32"], default="f16")
    ap.add_argument("--lengths", choices=["full", "prefix"], default="full")
    ap.add_argument("--stream-k", action="store_true", help="gemm: pass a stream-K workspace")
    ap.add_argument("--launches", type=int, default=5)
    args = ap.parse_args(argv)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    flush = torch.empty(FLUSH_BYTES // 4, dtype=torch.float32, device=dev)

    def randn(*shape, scale=1.0):
        return (torch.randn(*shape, device=dev, generator=g) * scale).half()

    nbytes = 0.0
    if args.kernel == "gemm":
        m, n, k = args.dims
        a, w = randn(m, k), randn(n, k, scale=k ** -0.5)
        bias = torch.randn(n, device=dev, generator=g)
        out_dtype = torch.float16 if args.out == "f16" else torch.float32
        act = K.ACT_GELU if args.act == "gelu" else K.ACT_NONE
        ws = K.gemm_workspace(dev) if args.stream_k else None
        fn = lambda: K.gemm_bias(a, w, bias, act=act, out_dtype=out_dtype, workspace=ws)
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
                      sched=torch.zeros(2, dtype=torch.int32, device=dev),
                      skip_dead_rows=True)
            n_list = lengths.tolist()
        else:
            n_list = [s] * b
        fn = lambda: K.flash_attention(qkv, h, causal=True, **kw)
        flops = sum(4.0 * h * hd * n * (n + 1) / 2 for n in n_list)
    elif args.kernel == "ln":
        rows, d = args.dims
        res = torch.randn(rows, d, device=dev, generator=g)
        delta = randn(rows, d)
        w = torch.ones(d, device=dev)
        bvec = torch.zeros(d, device=dev)
        fn = lambda: K.fused_add_layernorm(res, delta, w, bvec, 1e-5, out_dtype=torch.float16,
                                           residual_out=res)
        flops, nbytes = 0.0, rows * d * (4.0 + 2 + 4 + 2)
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
        fn = lambda: K.gemm_add_layernorm(a, w, bias, res, gamma, beta, 1e-5,
                                          residual_out=res, out=out, workspace=ws)
        flops = 2.0 * m * n * k
    elif args.kernel == "small":
        # The whole forward in one launch (tjb_forward_small): dims B S d H F L,
        # default-like random weights, all tokens valid, causal.
        b, s, d, h, f, layers = args.dims
        one = lambda n: torch.ones(n, device=dev)
        zero = lambda n: torch.zeros(n, device=dev)
        blocks = [types.SimpleNamespace(
            wqkv=randn(3 * d, d, scale=d ** -0.5), wo=randn(d, d, scale=d ** -0.5),
            w1=randn(f, d, scale=d ** -0.5), w2=randn(d, f, scale=f ** -0.5),
            bqkv=zero(3 * d), bo=zero(d), b1=zero(f), b2=zero(d), ln1_w=one(d), ln1_b=zero(d),
            ln2_w=one(d), ln2_b=zero(d), ln1_eps=1e-5, ln2_eps=1e-5) for _ in range(layers)]
        small = K.SmallModel(blocks, (one(d), zero(d), 1e-5))
        x = torch.randn(b, s, d, device=dev, generator=g)
        ws = K.forward_small_workspace(b, s, d, f, dev)
        out = torch.empty_like(x)
        fn = lambda: K.forward_small(small, x, None, h, f, True, ws, out=out)
        flops = 2.0 * b * s * small.gemm_params + layers * 4.0 * d * b * s * (s + 1) / 2
        nbytes = float(small.param_bytes + 2 * x.numel() * 4)
    else:
        # ffn: the two GEMM launches through a hidden scratch; ffn_single: the
        # one-kernel form whose hidden activations stay on chip.
        t, d, f = args.dims
        h = randn(t, d)
        w1, w2 = randn(f, d, scale=d ** -0.5), randn(d, f, scale=f ** -0.5)
        b1 = torch.zeros(f, device=dev)
        b2 = torch.zeros(d, device=dev)
        if args.kernel == "ffn":
            fn = lambda: K.fused_ffn(h, w1, b1, w2, b2, out_dtype=torch.float16)
        else:
            fn = lambda: K.ffn_single_kernel(h, w1, b1, w2, b2, out_dtype=torch.float16)
        flops = 4.0 * t * d * f
    ms = time_launches(fn, args.launches, flush)
    rate = f"  {flops / ms / 1e9:.0f} TFLOP/s" if flops else ""
    if nbytes:
        rate += f"  {nbytes / ms / 1e6:.0f} GB/s"
    print(f"{args.kernel} {args.dims}: {ms * 1e3:.1f} us{rate}", flush=True)
    return 0


# --------------------------------------------------------------------- main

def main():
    if "--kernel" in sys.argv[1:]:
        argv = list(sys.argv[1:])
        argv.remove("--kernel")
        sys.exit(kernel_main(argv))
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2, choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="tjb", choices=["tjb", "reference", "reference-gpu"])
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
    if args.impl == "reference-gpu":
        run_reference_gpu(args, rank, world)
        return

    use_package()
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
    # Default initialisation, drawn on the GPU itself (config 4's 2.4 B
    # parameters take tens of seconds to initialise on the host).
    with torch.device(dev):
        model = Encoder(cfg).eval()
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
        barrier()
        torch.cuda.synchronize(dev)
        with ClockSampler(local) as clocks:
            step_ms = timed_steps(model, x, mask, args.steps, stream, flush)
        barrier()

        # ------------------------------------------------------- end to end
        e2e_ms = e2e_leg(model, x_cpu, mask_cpu, args.steps, dev, stream, flush, barrier)

        # ------------------------- scatter/gather from GPU 0 (N > 1 only)
        # The same steps with the inputs starting on GPU 0: each step's
        # shards are scattered from GPU 0 over NVLink (NCCL), every GPU runs
        # its forward, and the outputs are gathered back to GPU 0.  As in a
        # serving loop, the collectives run on their own stream with two
        # buffer sets: step i+1's scatter and step i's gather overlap the
        # forwards (every rank issues them in the same order).
        sg_ms = 0.0
        sg_transport = None
        if world > 1 and not tp:
            depth = 2
            x_all = None
            out_all = [None] * depth
            if rank == 0:
                x_all = [synthetic_case(b, s, d, 100000, pad, r, world)[0].to(dev)
                         for r in range(world)]
            shard_bytes = b * s * d * 4
            peers = PeerBuffers(dist, rank, world, dev, shard_bytes, depth, x_all or [])
            sg_transport = "p2p" if peers.ok else "nccl"
            if not peers.ok and rank == 0:
                out_all = [[torch.empty((b, s, d), dtype=torch.float32, device=dev)
                            for _ in range(world)] for _ in range(depth)]
            x_sg = [torch.empty_like(x) for _ in range(depth)]
            comm = torch.cuda.Stream(dev)
            ev_in = [torch.cuda.Event() for _ in range(depth)]
            ev_done = [torch.cuda.Event() for _ in range(depth)]

            def scatter_into(dst):
                if peers.ok:
                    peers.pull_input(dst, comm)
                else:
                    dist.scatter(dst, x_all, src=0)

            def gather_from(out, k):
                if peers.ok:
                    peers.push_output(out, k, comm)
                else:
                    dist.gather(out, out_all[k], dst=0)

            def sg_steps(n):
                with torch.cuda.stream(comm):
                    comm.wait_stream(stream)
                    scatter_into(x_sg[0])
                    ev_in[0].record(comm)
                for i in range(n):
                    k, kn = i % depth, (i + 1) % depth
                    if i + 1 < n:
                        with torch.cuda.stream(comm):
                            if i >= 1:
                                comm.wait_event(ev_done[kn])  # forward i-1 read x_sg[kn]
                            scatter_into(x_sg[kn])
                            ev_in[kn].record(comm)
                    stream.wait_event(ev_in[k])
                    out = model(x_sg[k], mask)
                    ev_done[k].record(stream)
                    flush.zero_()
                    with torch.cuda.stream(comm):
                        comm.wait_event(ev_done[k])
                        gather_from(out, k)
                        out.record_stream(comm)
                stream.wait_stream(comm)

            sg_steps(2 * depth)
            torch.cuda.synchronize(dev)
            barrier()
            sg_start = torch.cuda.Event(enable_timing=True)
            sg_end = torch.cuda.Event(enable_timing=True)
            sg_start.record(stream)
            sg_steps(args.steps)
            sg_end.record(stream)
            torch.cuda.synchronize(dev)
            barrier()
            sg_ms = sg_start.elapsed_time(sg_end) / args.steps
            peers.close(dist, dev)
            del x_all, out_all

        # -------------------------------- per-kernel timing of the plan (eager)
        # Eager forwards of the plan that was timed (graph off): each library
        # call bracketed by CUDA events; gives the roofline's dominant kernel,
        # the other families' rates and the launch count per forward.
        ksteps = max(3, min(args.steps, 20))
        plans.set_override(dataclasses.replace(plan, cuda_graph=False))
        model(x, mask)
        torch.cuda.synchronize(dev)
        timer = KernelTimer(K, {"lengths": lengths, "valid_tokens": sum(lengths)})
        with timer:
            for _ in range(ksteps):
                model(x, mask)
                flush.zero_()
        kern_plan = timer.summary(ksteps)
        gemm_shapes = timer.gemm_shapes(ksteps)
        launches_per_step = sum(v["launches_per_step"] for v in kern_plan.values())
        plans.set_override(None)

    status_local = float(K.device_status(clear=True))  # synchronises; after all timing
    step_max, e2e_max, sg_max, status_max = max_over_ranks([step_ms, e2e_ms, sg_ms,
                                                            status_local])
    device_status = int(status_max)

    if rank == 0:
        peaks = load_peaks()
        tokens = b * s * (1 if tp else world)
        value = tokens / (step_max / 1e3)
        # The dominant kernel family: the tcgen05 GEMM (CTA-pair or single-CTA
        # form), launched by gemm_bias (one launch per call) and fused_ffn (two).
        fams = [kern_plan[n] for n in ("gemm_bias", "fused_ffn") if n in kern_plan]
        gemm_ms = sum(v["ms_per_step"] for v in fams)
        gemm_flops = sum(v["flops_per_call"] * v["calls_per_step"] for v in fams)
        gemm_launches = sum(v["launches_per_step"] for v in fams)
        peak = peaks["tflops"]
        achieved = gemm_flops / (gemm_ms / 1e3) / 1e12 if gemm_ms > 0 else None
        traffic = GEMM_TRAFFIC_PER_LAUNCH.get(args.config) if not tp else None

        def rate(name, key="tflops"):
            return kern_plan.get(name, {}).get(key)

        def frac(v, p):
            return None if v is None else v / p

        whole = kern_plan.get("forward_small")
        if whole is not None:
            # One launch runs the whole forward (tjb_forward_small): at these
            # token counts it streams the parameters, so its roofline is HBM.
            roofline = {
                "bound": "hbm",
                "kernel": "forward_small_kernel: the whole forward in one cooperative launch",
                "achieved": whole["gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": whole["gbs"] / peaks["hbm_gbs"],
                "peak_note": f"{peaks['source']} HBM copy bandwidth; bytes = parameters + "
                             "input + output per forward",
                "bytes_per_launch": whole["bytes_per_call"],
                "ms_per_launch": whole["ms_per_call"],
                "tflops": whole["tflops"], "tflops_frac": frac(whole["tflops"], peak),
                "traffic": None,
                "eager_step_ms": sum(v["ms_per_step"] for v in kern_plan.values()),
            }
        else:
            roofline = {
                "bound": "tensor",
                "kernel": "tcgen05 GEMM: gemm_pair_kernel (CTA pairs) and gemm_kernel "
                          "(single CTA, stream-K), every launch in the timed plan",
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak,
                "peak_note": f"{peaks['source']} burst bf16/f16 dense (sustained "
                             f"{peaks['tflops_sustained']}); FLOPs on valid tokens",
                "flops_per_launch": gemm_flops / gemm_launches,
                "ms_per_launch": gemm_ms / gemm_launches,
                "traffic": traffic,
                "traffic_note": "dram__bytes_read.sum + dram__bytes_write.sum per GEMM "
                                "launch, mean over one forward's launches, one ncu capture "
                                "of this command" if traffic else None,
                "attn_tflops": rate("flash_attention"),
                "attn_frac": frac(rate("flash_attention"), peak),
                "ffn_tflops": rate("fused_ffn"), "ffn_frac": frac(rate("fused_ffn"), peak),
                "gemm_ln_tflops": rate("gemm_add_layernorm"),
                "gemm_ln_frac": frac(rate("gemm_add_layernorm"), peak),
                "layernorm_gbs": rate("fused_add_layernorm", "gbs"),
                "layernorm_frac": frac(rate("fused_add_layernorm", "gbs"), peaks["hbm_gbs"]),
                "eager_step_ms": sum(v["ms_per_step"] for v in kern_plan.values()),
            }

        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_max,
            "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": {torch.float16: "f16", torch.bfloat16: "bf16"}[plan.compute_dtype],
            "data": "synthetic (seeded N(0,1) inputs, default-init weights)",
            "config": dict(workload_config(args.config, world, tp),
                           plan=plan.to_json()),
            "roofline": roofline,
            "kernels_plan": kern_plan,
            "gemm_shapes": gemm_shapes,
            "e2e": {"value": tokens / (e2e_max / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": x_cpu.numel() * 4 + mask_cpu.numel(),
                    "d2h_bytes_per_step": b * s * d * 4, "ms_per_step": e2e_max,
                    "h2d_gbs_per_rank": (x_cpu.numel() * 4 + mask_cpu.numel()) / e2e_max / 1e6,
                    "d2h_gbs_per_rank": b * s * d * 4 / e2e_max / 1e6,
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
                "transport": sg_transport,
                "note": "inputs start on GPU 0; per step every rank pulls its input shard "
                        "from GPU 0 and pushes its output shard back with copy-engine "
                        "cudaMemcpyAsync over NVLink through CUDA IPC mappings (transport "
                        "p2p; NCCL scatter/gather if the mapping is not available), on a "
                        "side stream, step i+1's scatter and step i's gather overlapping "
                        "the forwards (two buffer sets); max over ranks"}
        if device_status != 0:
            print(json.dumps(line), flush=True)
            raise SystemExit(f"a kernel recorded device status {device_status} "
                             "(bounded wait ran out): run invalid")
        if world == 1 and not args.no_cpu_baseline:
            rate_cpu, info = cpu_forward_rate(args.config, cpu_sample_plan(args.config)[2])
            line["cpu_baseline"] = {"value": rate_cpu, "unit": "tokens/s",
                                    "cores": info["cores"], "kind": "port",
                                    "sample": info["sample"]}
        print(json.dumps(line), flush=True)

    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

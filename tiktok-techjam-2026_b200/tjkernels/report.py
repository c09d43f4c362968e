"""Benchmark sweep and report: every config (and GPU count) through bench.py.

    python -m tjkernels.report run [--configs 0 1 2 3 4] [--gpus 1 2 4 8]
                                   [--steps K] [--warmup W] [--with-reference]
                                   [--out results.json]
    python -m tjkernels.report render results.json [--md report.md]

``run`` launches ``bench.py`` once per (config, GPU count) in its own process
(``torch.distributed.run`` on 127.0.0.1 for N > 1), each under a time limit,
and keeps the JSON line each prints, so one crashed or timed-out config
leaves the others' results; ``--with-reference`` adds the reference arm
(``bench.py --impl reference``, the CPU forward) per config.  ``render``
turns the collected lines into a Markdown table: tokens/s on the device and
end to end, ms per forward, the GEMM roofline fraction, the attention / FFN
/ LayerNorm fractions, the CPU baseline and the ratio against it, and the
clocks seen.  Same flow as the reference's ``bench/run_all.py`` (per-case
subprocess sweep into JSON) and ``bench/make_report.py`` (JSON to Markdown).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time
from pathlib import Path
from typing import Dict, Iterable, List, Optional, Sequence

REPO = Path(__file__).resolve().parents[2]
BENCH = REPO / "bench.py"


def bench_command(config: int, gpus: int, steps: int, warmup: int, impl: str = "tjb",
                  port: int = 29531, extra: Sequence[str] = ()) -> List[str]:
    """The command line that runs bench.py for one (config, GPU count)."""
    args = [str(BENCH), "--gpus", str(gpus), "--steps", str(steps), "--warmup", str(warmup),
            "--config", str(config), "--impl", impl, *extra]
    if gpus == 1:
        return [sys.executable, *args]
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
            f"--nproc-per-node={gpus}", "--master-addr", "127.0.0.1",
            "--master-port", str(port), *args]


def last_json_line(text: str) -> Optional[Dict[str, object]]:
    """The last line of ``text`` that parses as a JSON object."""
    for line in reversed(text.splitlines()):
        line = line.strip()
        if line.startswith("{"):
            try:
                obj = json.loads(line)
            except json.JSONDecodeError:
                continue
            if isinstance(obj, dict):
                return obj
    return None


def run(configs: Iterable[int], gpus: Iterable[int], steps: int, warmup: int,
        with_reference: bool = False, timeout_s: float = 900.0,
        extra: Sequence[str] = ()) -> List[Dict[str, object]]:
    """Run every (config, GPU count) and return one record per run."""
    records = []
    port = 29531
    for cfg in configs:
        arms = [("tjb", n) for n in gpus]
        if with_reference:
            arms.insert(0, ("reference", 1))
        for impl, n in arms:
            cmd = bench_command(cfg, n, steps, warmup, impl, port, extra)
            port += 1
            t0 = time.time()
            rec: Dict[str, object] = {"config": cfg, "gpus": n, "impl": impl,
                                      "command": " ".join(cmd)}
            try:
                proc = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True,
                                      timeout=timeout_s, env=dict(os.environ))
                rec["returncode"] = proc.returncode
                rec["result"] = last_json_line(proc.stdout)
                if proc.returncode != 0 or rec["result"] is None:
                    rec["stderr_tail"] = proc.stderr[-2000:]
            except subprocess.TimeoutExpired:
                rec["returncode"] = None
                rec["result"] = None
                rec["error"] = f"timed out after {timeout_s:.0f} s"
            rec["wall_s"] = round(time.time() - t0, 1)
            records.append(rec)
            print(json.dumps({k: rec[k] for k in ("config", "gpus", "impl", "returncode",
                                                  "wall_s")}), flush=True)
    return records


def _fmt(v: Optional[float], unit: str = "", digits: int = 3) -> str:
    if v is None:
        return "—"
    if unit == "M":  # tokens/s: millions on the GPU, plain for the CPU's thousands
        return f"{v / 1e6:.{digits}g} M" if v >= 1e5 else f"{v:.4g}"
    if unit == "%":
        return f"{100 * v:.0f} %"
    return f"{v:.{digits}g}"


def render(records: List[Dict[str, object]]) -> str:
    """Markdown table of the records (one row per run)."""
    ref_rate: Dict[int, float] = {}
    for rec in records:
        res = rec.get("result") or {}
        if rec.get("impl") == "reference" and isinstance(res, dict) and "value" in res:
            ref_rate[int(rec["config"])] = float(res["value"])
    head = ("| cfg | GPUs | impl | tokens/s | e2e tokens/s | ms / fwd | GEMM % peak | "
            "attn % | FFN % | LN % HBM | CPU tokens/s | e2e ÷ CPU | SM MHz (reasons) |")
    ncol = head.count("|") - 1
    lines = [head, "|" + "---|" * ncol]
    for rec in records:
        cfg, n, impl = rec["config"], rec["gpus"], rec["impl"]
        res = rec.get("result")
        if not isinstance(res, dict) or "value" not in res:
            why = rec.get("error") or (res or {}).get("unavailable") or \
                f"exit {rec.get('returncode')}"
            lines.append(f"| {cfg} | {n} | {impl} | {why} |" + " — |" * (ncol - 4))
            continue
        e2e = res.get("e2e") if isinstance(res.get("e2e"), dict) else {}
        roof = res.get("roofline") if isinstance(res.get("roofline"), dict) else {}
        cpu = res.get("cpu_baseline") if isinstance(res.get("cpu_baseline"), dict) else {}
        clocks = res.get("clocks") if isinstance(res.get("clocks"), dict) else {}
        cpu_rate = cpu.get("value") if impl != "reference" else None
        base = ref_rate.get(int(cfg)) or cpu_rate
        e2e_v = e2e.get("value")
        ratio = (float(e2e_v) / float(base)) if (e2e_v and base and impl != "reference") else None
        mhz = clocks.get("sm_mhz")
        reasons = ",".join(clocks.get("reasons") or []) or "none"
        lines.append(
            f"| {cfg} | {n} | {impl} | {_fmt(res.get('value'), 'M')} | {_fmt(e2e_v, 'M')} | "
            f"{_fmt(res.get('ms_per_step'), digits=4)} | {_fmt(roof.get('frac'), '%')} | "
            f"{_fmt(roof.get('attn_frac'), '%')} | {_fmt(roof.get('ffn_frac'), '%')} | "
            f"{_fmt(roof.get('layernorm_frac'), '%')} | {_fmt(cpu_rate, 'M')} | "
            f"{_fmt(ratio, digits=4)}{'×' if ratio else ''} | "
            f"{'—' if mhz is None else f'{mhz:.0f}'} ({reasons}) |")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="cmd", required=True)
    r = sub.add_parser("run")
    r.add_argument("--configs", type=int, nargs="+", default=[0, 1, 2, 3, 4])
    r.add_argument("--gpus", type=int, nargs="+", default=[1])
    r.add_argument("--steps", type=int, default=20)
    r.add_argument("--warmup", type=int, default=5)
    r.add_argument("--with-reference", action="store_true")
    r.add_argument("--timeout", type=float, default=900.0)
    r.add_argument("--out", default="results.json")
    r.add_argument("--dry-run", action="store_true", help="print the commands only")
    d = sub.add_parser("render")
    d.add_argument("results")
    d.add_argument("--md", default=None)
    args = ap.parse_args(argv)
    if args.cmd == "run":
        if args.dry_run:
            port = 29531
            for cfg in args.configs:
                for n in args.gpus:
                    print(" ".join(bench_command(cfg, n, args.steps, args.warmup, port=port)))
                    port += 1
            return 0
        records = run(args.configs, args.gpus, args.steps, args.warmup, args.with_reference,
                      args.timeout)
        Path(args.out).write_text(json.dumps(records, indent=1))
        print(render(records))
        return 0 if all(rec.get("returncode") == 0 for rec in records) else 1
    records = json.loads(Path(args.results).read_text())
    table = render(records)
    if args.md:
        Path(args.md).write_text(table)
    print(table)
    return 0


if __name__ == "__main__":
    sys.exit(main())

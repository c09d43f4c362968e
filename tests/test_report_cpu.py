"""The sweep/report tool on the CPU: commands it would run, JSON-line
parsing and the Markdown table (no GPU, no subprocess)."""

import json

from tjkernels import report


def test_bench_commands():
    one = report.bench_command(2, 1, 10, 3)
    assert one[1].endswith("bench.py") and one[one.index("--config") + 1] == "2"
    assert one[one.index("--impl") + 1] == "tjb"
    eight = report.bench_command(4, 8, 5, 3, port=29600)
    assert eight[1:3] == ["-m", "torch.distributed.run"]
    assert "--nproc-per-node=8" in eight and "127.0.0.1" in eight and "29600" in eight
    assert eight[eight.index("--gpus") + 1] == "8"


def test_last_json_line():
    text = 'warming up\n{"a": 1}\nnoise {\n{"metric": "x", "value": 2.0}\ntrailing text\n'
    assert report.last_json_line(text) == {"metric": "x", "value": 2.0}
    assert report.last_json_line("no json here\n{broken") is None


def _line(value, e2e, cpu=None):
    line = {"metric": "forward tokens/sec", "value": value, "ms_per_step": 0.9,
            "e2e": {"value": e2e}, "roofline": {"frac": 0.58, "attn_frac": 0.13,
                                                "ffn_frac": 0.6, "layernorm_frac": 0.75},
            "clocks": {"sm_mhz": 1965.0, "reasons": []}}
    if cpu is not None:
        line["cpu_baseline"] = {"value": cpu}
    return line


def test_render_table():
    records = [
        {"config": 2, "gpus": 1, "impl": "reference", "returncode": 0,
         "result": {"impl": "reference", "value": 1000.0, "ms_per_step": 8000.0}},
        {"config": 2, "gpus": 1, "impl": "tjb", "returncode": 0,
         "result": _line(9.1e6, 8.0e6, cpu=1200.0)},
        {"config": 3, "gpus": 2, "impl": "tjb", "returncode": None, "result": None,
         "error": "timed out after 900 s"},
    ]
    md = report.render(json.loads(json.dumps(records)))
    rows = md.strip().splitlines()
    assert len(rows) == 5 and rows[1].count("---") == rows[0].count("|") - 1
    assert all(r.count("|") == rows[0].count("|") for r in rows)
    assert "9.1 M" in rows[3] and "58 %" in rows[3] and "8000×" in rows[3]
    assert "| 1000 |" in rows[2] and "| 1200 |" in rows[3]
    assert "timed out" in rows[4]

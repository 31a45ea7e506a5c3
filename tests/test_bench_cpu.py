"""bench.py's contract on a machine without a GPU: the reference arm (the
CPU implementation of the path) prints one JSON line with the metric, the
cpu_baseline block and an e2e block with zero copies, and the B200 arm's
argument parser knows the profiling and comparator switches."""

import json
import os
import subprocess
import sys

from conftest import ROOT

sys.path.insert(0, ROOT)
import bench  # noqa: E402


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_attention_line():
    d = _run("--impl", "reference", "--config", "cfg0", "--steps", "2", "--warmup", "1")
    assert d["impl"] == "reference" and d["unit"] == "TFLOP/s" and d["value"] > 0
    assert d["higher_is_better"] is True and d["config"]["D"] == 64
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_mlp_line():
    d = _run("--impl", "reference", "--config", "cfg3", "--steps", "1", "--warmup", "1")
    assert d["impl"] == "reference" and d["metric"] == "MLP block TFLOP/s" and d["value"] > 0


def test_parser_knows_profiling_switches():
    a = bench.parse_args(["--config", "cfg2", "--pairs", "32", "--kernel-only", "--no-sdpa",
                          "--no-secondary"])
    assert a.pairs == 32 and a.kernel_only and a.no_sdpa and a.no_secondary
    a = bench.parse_args(["--config", "ln", "--rows", "16384"])
    assert a.config == "ln" and a.rows == 16384
    assert bench.parse_args([]).config == "cfg2"

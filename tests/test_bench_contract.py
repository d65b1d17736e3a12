"""The benchmark's JSON line for the reference arm (CPU only: the reference arm times the CPU port).

The driver reads one JSON line per run; these checks pin the keys it reads and the consistency between the
steps a line claims and the time its run took (steps x ms_per_step fits the timed region), on the small
cfg1 workload so that the test takes seconds.
"""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _reference_line(*extra):
    cmd = [sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference", "--config", "cfg1", "--steps", "2",
           "--warmup", "1", "--no-reference-cuda", *extra]
    out = subprocess.run(cmd, cwd=REPO, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_line_keys_and_timed_region():
    d = _reference_line()
    for key in ("metric", "value", "unit", "impl", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "dtype", "data", "config", "cpu_baseline", "e2e", "what_ran"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 1
    assert d["higher_is_better"] is False and d["unit"] == "ms"
    assert d["value"] > 0 and d["ms_per_step"] > 0
    # the value scales one sample to the whole grid, so it is at least the sample's own time
    assert d["value"] >= d["ms_per_step"]
    # the steps the line claims fit the region that was timed
    assert d["steps"] * d["ms_per_step"] <= d["what_ran"]["timed_region_s"] * 1e3 * 1.05
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1

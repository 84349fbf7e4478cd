"""bench.py's reference arm runs on the host cores and prints the driver's JSON line
(CPU only): hayate's own CPU attention path from baseline/_ref on a bounded sample of
config 2, with config 1 beside it, or the NumPy restatement where the reference is absent."""

from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    proc = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1",
                           "--warmup", "0"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr[-2000:]
    line = json.loads(proc.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in line, key
    assert line["metric"] == "decode attn HBM GB/s (% of peak)" and line["unit"] == "GB/s"
    assert line["value"] > 0 and line["steps"] == 1
    installed = os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "hayate"))
    assert line["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    assert line["cpu_baseline"]["cores"] >= 1
    if installed:
        assert line["config1"]["kind"] == "reference" and line["config1"]["value"] > 0
        assert "config 1" in line["config1"]["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_longdecode_defaults_to_config5_steps():
    sys.path.insert(0, ROOT)
    import bench

    old = sys.argv
    try:
        sys.argv = ["bench.py", "--workload", "longdecode"]
        assert bench.parse_args().steps == 128
        sys.argv = ["bench.py"]
        assert bench.parse_args().steps == 2000
    finally:
        sys.argv = old


def test_reference_cpu_path_puts_the_compiled_wrapper_back():
    """The CPU timing swaps the reference module's compiled FlexAttention for the eager one;
    the GPU comparisons that run later in the same bench process must see the compiled
    wrapper again (the eager path scores the whole pool: slower, and out of memory on long
    prefixes)."""
    import pytest

    if not os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "hayate")):
        pytest.skip("reference not installed in baseline/_ref")
    sys.path.insert(0, ROOT)
    import bench

    mods, why = bench.import_reference()
    assert mods is not None, why
    paged_cache = mods[0]
    before = paged_cache._compiled_flex_attention
    out = bench.reference_cpu_path("config1", steps=1, warmup=0, budget_s=0.0)
    assert out["kind"] == "reference" and out["value"] > 0
    assert paged_cache._compiled_flex_attention is before

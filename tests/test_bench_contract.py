"""CPU checks of bench.py's JSON contract: the reference arm (the CPU port of
ref_kernel, timed on host cores) prints one line with the driver's keys, and
the peak selection picks the sustained figure only for long timed regions."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


@pytest.mark.parametrize("config", ["gemv", "dual"])
def test_reference_arm_line(config):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "0",
                          "--config", config], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["warmup"] >= 3 and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["config"]["workload"] == config


def test_peak_selection():
    import bench
    hbm, bf16_burst, src = bench.load_peaks(long_run=False)
    _, bf16_sust, src_long = bench.load_peaks(long_run=True)
    assert hbm > 0 and bf16_burst > 0 and bf16_sust > 0
    assert bf16_sust <= bf16_burst
    assert ("sustained" in src_long) or src_long == "fallback"

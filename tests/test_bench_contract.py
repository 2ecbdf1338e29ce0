"""bench.py's CPU-side contract: the reference arm's JSON line and the clock summary.

The reference arm times the CPU restatement of the reference's attention oracle
(the reference's own kernels need Metal), so it runs here without a GPU.
"""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def test_reference_arm_prints_one_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                        "--steps", "3", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 3 and d["warmup"] == 3
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["config"]["workload"] == "fa_f16_causal_B4_H16_S2048_D128"


def test_clock_summary_flags_throttle_reasons():
    import bench
    s = bench.ClockSampler(0)
    s.samples = [
        ["0", "1965", "1965", "400.0", "0x0", "Not Active", "Not Active", "Not Active", "Not Active"],
        ["0", "1590", "1965", "990.0", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
        ["0", "1600", "1965", "980.0", "0x4", "Not Active", "Not Active", "Not Active", "Active"],
    ]
    out = s.summary()
    assert out["sm_mhz"] == 1600.0
    assert out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == ["sw_power_cap"]
    assert out["samples"] == 3
    assert bench.ClockSampler(0).summary()["reasons"] == ["unsampled"]

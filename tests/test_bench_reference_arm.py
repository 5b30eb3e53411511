"""The bench's reference arm (`bench.py --impl reference`) runs on host cores
only: it must print one JSON line with the contract's keys on rank 0 and exit
0 without work on the other ranks -- on a machine with no GPU too."""

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "2",
                           "--warmup", "1"], capture_output=True, text=True, env=env, timeout=600)


def test_reference_arm_prints_contract_line():
    r = _run({"WORLD_SIZE": "1", "RANK": "0"})
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"WORLD_SIZE": "2", "RANK": "1"})
    assert r.returncode == 0 and r.stdout.strip() == "", (r.stdout, r.stderr[-2000:])


def test_submetrics_summarise_the_suite():
    """The compact `submetrics` key: each BASELINE sub-metric with its
    fraction of the measured peak (GB/s of HBM, TFLOP/s of dense bf16)."""
    import sys
    sys.path.insert(0, str(ROOT))
    import bench
    hbm, tf, _ = bench.measured_peaks()
    suite = {"qkv_m1": {"us_per_launch": 7.0, "GB/s": hbm / 2},
             "qkv_m2048": {"us_per_launch": 60.0, "TFLOP/s": tf / 4},
             "mla_b32_l32768": {"us_per_step": 229.0, "GB/s": hbm * 0.75},
             "mla_sideband_fill_b32_l32768": {"us": 575.0, "x_decode_step": 2.5, "TFLOP/s": 700.0}}
    sm = bench.submetrics(suite)
    assert sm["qkv_m1"]["frac"] == 0.5 and sm["qkv_m1"]["us"] == 7.0
    assert sm["qkv_m2048"]["frac"] == 0.25
    assert sm["mla_b32_l32768"]["frac"] == 0.75 and sm["mla_b32_l32768"]["us"] == 229.0
    assert sm["mla_sideband_fill_b32_l32768"]["x_decode_step"] == 2.5
    assert "gate_up_m1" not in sm  # absent parts are left out, not invented

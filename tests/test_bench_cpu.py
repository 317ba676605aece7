"""bench.py on the CPU: the algorithmic work counts behind the roofline figures
and the reference arm's JSON line (it runs on the host cores only)."""
import json
import os
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402


def test_dcn_work_counts():
    # cfg2 / cfg3: 2*M*N*K = 41.05 GFLOP; unique bytes 23.01 MB / 38.69 MB (fp16/bf16)
    f2, b2 = bench.dcn_work(bench.DCN_CFGS["cfg2"])
    f3, b3 = bench.dcn_work(bench.DCN_CFGS["cfg3"])
    assert abs(f2 - 41.05e9) / 41.05e9 < 1e-3 and abs(f3 - 41.05e9) / 41.05e9 < 1e-3
    assert abs(b2 - 23.01e6) / 23.01e6 < 1e-3 and abs(b3 - 38.69e6) / 38.69e6 < 1e-3
    # cfg1: 75.5 MFLOP, fp32, with its bias
    f1, b1 = bench.dcn_work(bench.DCN_CFGS["cfg1"])
    assert abs(f1 - 75.5e6) / 75.5e6 < 1e-2 and 0.7e6 < b1 < 0.8e6


def test_msda_byte_counts():
    # cfg4 194.56 MB, cfg5 435.15 MB (fp32); fp16/bf16 halve them
    assert abs(bench.msda_bytes(bench.MSDA_CFGS["cfg4"]) - 194.56e6) < 0.01e6
    assert abs(bench.msda_bytes(bench.MSDA_CFGS["cfg5"]) - 435.15e6) < 0.01e6
    assert bench.msda_bytes(bench.MSDA_CFGS["cfg5"], 2) * 2 == bench.msda_bytes(
        bench.MSDA_CFGS["cfg5"])


def test_compact_rounding():
    assert bench._r(45.3256) == 45.3 and bench._r(None) is None and bench._r(0) == 0.0
    assert bench._r(0.54759) == 0.548


@pytest.mark.timeout(300)
def test_reference_arm_line():
    env = dict(os.environ)
    for k in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(k, None)
    out = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "3"], env=env, capture_output=True,
                         text=True, timeout=280, cwd=REPO)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC
    assert line["unit"] == "TFLOP/s" and line["higher_is_better"] is True
    assert line["steps"] == 2 and line["warmup"] == 3 and line["value"] > 0
    # the same config dict as our arm's headline, so the two lines compare
    assert line["config"] == bench.headline_config(1)
    cb = line["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0

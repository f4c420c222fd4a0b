"""The JSON line bench.py prints (the contract the benchmark driver reads)."""

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config"}


def _line(args):
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                          timeout=900, cwd=ROOT)
    assert proc.returncode == 0, proc.stdout[-2000:] + proc.stderr[-2000:]
    lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, proc.stdout
    return json.loads(lines[0])


def test_reference_arm_prints_the_contract_line(oracle_lib):
    d = _line(["--impl", "reference", "--workload", "test", "--steps", "1", "--warmup", "1", "--cpu-stories", "2"])
    assert BASE_KEYS <= set(d)
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert set(d["cpu_baseline"]) >= {"value", "unit", "cores", "kind", "sample"}
    assert d["cpu_baseline"]["kind"] == "port"
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert "workload" in d["config"]
    assert "oracle" not in d["config"]["workload"]


@pytest.mark.gpu
def test_gpu_arm_prints_the_contract_line(native_lib, oracle_lib):
    d = _line(["--workload", "test", "--steps", "1", "--warmup", "3", "--cpu-stories", "2", "--big-workload", "test",
               "--big-batches", "1"])
    assert BASE_KEYS <= set(d)
    assert d["n_gpus"] == 1 and d["value"] > 0
    r = d["roofline"]
    assert set(r) >= {"bound", "achieved", "peak", "unit", "frac", "traffic"}
    assert r["bound"] == "hbm" and r["unit"] == "GB/s" and r["peak"] > 0
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-5
    assert set(d["e2e"]) == {"value", "unit", "h2d_bytes_per_step", "d2h_bytes_per_step"}
    assert d["e2e"]["h2d_bytes_per_step"] > 0 and d["e2e"]["d2h_bytes_per_step"] > 0
    assert d["gpu_launches"] > 0
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= set(d["clocks"])
    assert set(d["cpu_baseline"]) >= {"value", "unit", "cores", "kind", "sample"}
    assert d["replay_off"]["value"] > 0 and d["replay_off"]["unit"] == d["unit"]
    assert d["execution_steps_per_second"] >= d["steps_per_second"] > 0
    big = d["config3"]
    assert big["value"] > 0 and big["unit"] == d["unit"] and big["timed_batches"] == 1
    assert big["roofline"]["frac"] > 0

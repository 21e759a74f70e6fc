"""The benchmark's JSON line (bench.py result_line) built from fabricated
measurements, on the CPU: every key the line promises is present and the
throughput, roofline and byte counts follow from the inputs."""
import argparse
import importlib.util
import json
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_encoder_frames(bench):
    assert bench.encoder_frames(160000) == 499        # 10 s at 16 kHz
    assert bench.encoder_frames(16000) == 49          # 1 s
    assert bench.encoder_frames(9) == 0 and bench.encoder_frames(0) == 0


def test_result_line_contract(bench):
    args = argparse.Namespace(batch=64, seconds=10.0, steps=30, warmup=3, e2e_steps=10, dtype="q8_0", world=2)
    prof = {"gemm_encoder": {"ms": 53.0, "launches": 480, "flops": 5.42e13},
            "attention": {"ms": 13.0, "launches": 120, "flops": 5.9e12}}
    clocks = [{"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 12},
              {"sm_mhz": 1880.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 12}]
    cpu = {"value": 4.4, "unit": bench.UNIT, "cores": 16, "kind": "reference", "sample": "a bounded sample"}
    line = bench.result_line(args, 2, 360.0, prof, 10, 100, clocks, 12.5, cpu)
    json.dumps(line)
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "roofline", "e2e", "gpu_launches", "clocks",
                "cpu_baseline"):
        assert key in line, key
    assert line["value"] == pytest.approx(2 * 30 * 640 / 0.360)      # whole job: both ranks' audio
    assert line["ms_per_step"] == pytest.approx(12.0)
    assert line["gpu_launches"] == 100 * 30 * 2
    assert line["higher_is_better"] is True and line["scaling"] == "weak"
    r = line["roofline"]
    for key in ("bound", "achieved", "peak", "unit", "frac", "traffic"):
        assert key in r, key
    assert r["achieved"] == pytest.approx(5.42e13 / 0.053 / 1e12)
    assert r["frac"] == pytest.approx(r["achieved"] / r["peak"])
    e = line["e2e"]
    assert e["value"] == pytest.approx(2 * 10 * 640 / 12.5)
    assert e["h2d_bytes_per_step"] == 64 * 160000 * 4
    assert e["d2h_bytes_per_step"] == 499 * 64 * 3 * 4 + 64 * 4 + 4
    assert line["clocks"]["reasons"] == ["sw_power_cap"]
    assert line["clocks"]["per_rank_sm_mhz"] == [1900.0, 1880.0]
    assert line["config"]["global_batch"] == 128
    assert line["breakdown_ms_per_step"]["attention"] == pytest.approx(1.3)
    assert line["cpu_baseline"] is cpu


def test_result_line_without_e2e(bench):
    args = argparse.Namespace(batch=16, seconds=5.0, steps=4, warmup=3, e2e_steps=10, dtype="f16", world=1)
    prof = {"gemm_encoder": {"ms": 0.0, "launches": 0, "flops": 0.0}}
    line = bench.result_line(args, 1, 40.0, prof, 4, 90, [{"sm_mhz": None, "reasons": []}], None, None)
    assert "e2e" not in line and "cpu_baseline" not in line
    assert line["roofline"]["achieved"] == 0.0
    assert line["roofline"]["traffic"] is None        # ncu traffic only for the default workload
    assert "249 frames each" in line["config"]["workload"]

"""The benchmark's JSON line (bench.py result_line) built from fabricated
measurements, on the CPU: every key the line promises is present and the
throughput, roofline and byte counts follow from the inputs; the workload
helpers and the parity report behave."""
import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["bench_under_test"] = mod          # dataclasses look their module up here
    spec.loader.exec_module(mod)
    return mod


def test_encoder_frames(bench):
    assert bench.encoder_frames(160000) == 499        # 10 s at 16 kHz
    assert bench.encoder_frames(320000) == 999        # 20 s
    assert bench.encoder_frames(16000) == 49          # 1 s
    assert bench.encoder_frames(9) == 0 and bench.encoder_frames(0) == 0


def test_result_line_contract(bench):
    wl = bench.WORKLOADS[bench.DEFAULT_WORKLOAD]
    args = argparse.Namespace(steps=30, warmup=3, e2e_steps=10, world=2)
    prof = {"gemm_encoder": {"ms": 53.0, "launches": 480, "flops": 5.42e13},
            "attention": {"ms": 13.0, "launches": 120, "flops": 5.9e12}}
    clocks = [{"sm_mhz": 1900.0, "sm_max_mhz": 1965.0, "reasons": [], "samples": 12},
              {"sm_mhz": 1880.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap"], "samples": 12}]
    cpu = {"value": 0.26, "unit": bench.UNIT, "cores": 16, "kind": "reference", "sample": "a bounded sample"}
    e2e = {"seconds": 12.5, "audio": 6400.0, "h2d": 64 * 160000 * 4, "d2h": 499 * 64 * 3 * 4 + 64 * 4 + 4}
    line = bench.result_line(args, wl, 2, 360.0, 30 * 640.0, prof, 10, 100, clocks, e2e, cpu)
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
    assert r["traffic"] == pytest.approx(np.mean(list(bench.ENCODER_GEMM_DRAM_BYTES.values())))
    e = line["e2e"]
    assert e["value"] == pytest.approx(2 * 6400 / 12.5)
    assert e["h2d_bytes_per_step"] == 64 * 160000 * 4
    assert e["d2h_bytes_per_step"] == 499 * 64 * 3 * 4 + 64 * 4 + 4
    assert line["clocks"]["reasons"] == ["sw_power_cap"]
    assert line["clocks"]["per_rank_sm_mhz"] == [1900.0, 1880.0]
    assert line["config"]["global_batch"] == 128
    assert "499 frames each" in line["config"]["workload"]
    assert line["breakdown_ms_per_step"]["attention"] == pytest.approx(1.3)
    assert line["cpu_baseline"] is cpu


def test_result_line_ragged_without_e2e(bench):
    wl = bench.WORKLOADS["xlsr1b-f16-b16-5to30s"]
    args = argparse.Namespace(steps=4, warmup=3, e2e_steps=10, world=1)
    prof = {"gemm_encoder": {"ms": 0.0, "launches": 0, "flops": 0.0}}
    lens = [bench.batch_lengths(wl, 0, j) for j in range(wl.n_rot)]
    audio = sum(sum(lens[j % wl.n_rot]) for j in range(4)) / bench.SR
    line = bench.result_line(args, wl, 1, 40.0, audio, prof, 4, 90, [{"sm_mhz": None, "reasons": []}], None, None,
                             lens)
    assert "e2e" not in line and "cpu_baseline" not in line
    assert line["value"] == pytest.approx(audio / 0.040)
    assert line["roofline"]["achieved"] == 0.0
    assert line["roofline"]["traffic"] is None        # ncu traffic only for the default workload
    assert "XLS-R-1B F16" in line["config"]["workload"] and "5-30 s" in line["config"]["workload"]


def test_workload_lengths(bench):
    wl = bench.WORKLOADS["xlsr1b-f16-b16-5to30s"]
    a, b2 = bench.batch_lengths(wl, 0, 0), bench.batch_lengths(wl, 0, 0)
    assert a == b2 and len(a) == 16                              # seeded: reproducible
    assert a != bench.batch_lengths(wl, 1, 0)                    # ranks get different utterances
    assert all(5 * 16000 <= n <= 30 * 16000 and n % 320 == 0 for n in a)
    assert bench.batch_lengths(bench.WORKLOADS["large-q8_0-b32-20s"], 0, 0) == [320000] * 32
    sw = bench.sweep_lengths(4096, 2.0, 30.0)
    assert len(sw) == 4096 and min(sw) >= 32000 and max(sw) <= 480000
    assert 15.0 < np.mean(sw) / 16000 < 17.0


def test_rank_seeds_disjoint(bench):
    a = {s for b in bench.rank_seeds(0, 4, 64) for s in b}
    b2 = {s for b in bench.rank_seeds(1, 4, 64) for s in b}
    assert len(a) == 256 and not a & b2
    assert bench.rank_seeds(0, 4, 64)[0] == list(range(64))


def test_collapse_ids(bench):
    assert bench.collapse_ids([0, 3, 3, 0, 3, 5, 5, 0]).tolist() == [3, 3, 5]
    assert bench.collapse_ids([]).tolist() == []
    assert bench.collapse_ids([0, 0]).tolist() == []


def test_parity_report_arithmetic(bench):
    """A fabricated fixture: reference logits, a copy with a small error, one
    utterance whose low-margin frame flips."""
    rng = np.random.default_rng(0)
    n, T, V = 6, 40, 8
    ex = rng.standard_normal((n, T, V)).astype(np.float32)
    gg = ex + rng.standard_normal((n, T, V)).astype(np.float32) * 1e-3
    got = [x + 1e-4 for x in ex]
    srt = np.sort(ex, 2)
    margin = srt[:, :, -1] - srt[:, :, -2]
    # utterance 2: swap the top two logits of its smallest-margin frame
    t = int(margin[2].argmin())
    row = got[2][t]
    i1, i2 = np.argsort(row)[-1], np.argsort(row)[-2]
    row[i1], row[i2] = row[i2], row[i1]
    fx = {"seeds": np.arange(n), "ids_exact": ex.argmax(2), "ids_ggml": gg.argmax(2), "margin_exact": margin,
          "full_seeds": np.array([0, 5]), "logits_exact_full": ex[[0, 5]], "logits_ggml_full": gg[[0, 5]]}
    r = bench.parity_report(got, fx)
    assert r["utterances"] == n
    assert r["logits_max_abs_vs_exact"] == pytest.approx(1e-4, rel=1e-2)
    assert r["frame_argmax_agree_vs_exact"] == pytest.approx(1 - 1 / (n * T))
    # the flipped frame had the smallest margin; unless that margin exceeds 2e-4 it is not a violation
    assert r["margin_rule_violations"] == int(margin[2, t] > 2 * r["logits_max_abs_vs_exact"])
    seq_same = np.array_equal(bench.collapse_ids(got[2].argmax(1)), bench.collapse_ids(ex[2].argmax(1)))
    assert r["greedy_sequences_identical_vs_exact"] == pytest.approx((n - 1 + seq_same) / n)

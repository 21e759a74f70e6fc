#!/usr/bin/env python3
"""Benchmark: wav2vec2 CTC inference in audio-seconds per second.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                  [--workload NAME]

Workloads (seeded synthetic audio, seeded random-init weights):
  base-q8_0-b64-10s     (default) wav2vec2-base, Q8_0 linears, 64 utterances
                        x 10 s per GPU (499 frames each), greedy CTC.
  base-q8_0-b1-10s      the same model, one 10 s utterance per step (latency;
                        L2 flushed between timed steps).
  base-q4_0-b64-10s     wav2vec2-base with Q4_0 linears, 64 x 10 s.
  large-q8_0-b32-20s    wav2vec2-large / XLS-R-300M architecture (LayerNorm
                        extractor, 24 pre-LN layers, hidden 1024), Q8_0,
                        32 utterances x 20 s (999 frames each).
  xlsr1b-f16-b16-5to30s XLS-R-1B architecture (48 pre-LN layers, hidden
                        1280, head dim 80), F16, 16 utterances per batch with
                        seeded lengths uniform in 5-30 s.
  sweep-base-q8_0-4096-2to30s
                        4096 utterances, lengths uniform in 2-30 s, through
                        wav2vec2_transcribe_batch on ONE context spanning
                        devices 0..N-1 (the library's own length bucketing and
                        multi-device scheduler), greedy and beam width 5.

A step is one forward pass (waveform -> conv extractor -> projection ->
positional conv -> encoder -> CTC head -> greedy CTC spans) over one batch.
`value` is timed with CUDA events on the forward's stream over exactly K
steps with the inputs already in HBM (distinct batches rotate; together they
exceed the 126 MB L2, and each step also streams its activations); `e2e`
times the public C API (wav2vec2_transcribe_batch) from pinned host arrays to
transcripts, host<->device copies included.  Multi-GPU: one process per GPU
(torchrun), utterances sharded (weak scaling, no collective on the data
path); barriers and the max-over-ranks timing use torch.distributed.

`--impl reference` times the reference's own CPU implementation (its sources
built against the oracle's ggml-API shim, oracle/_ref): the reference CLI,
one WAV per call with -t <usable host cores>, as the reference is run.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from dataclasses import dataclass
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "oracle"))
METRIC = "audio-sec/sec (inverse RTF), base Q8_0 batch 64, 1/2/4/8 B200; % MMA peak"
UNIT = "audio-sec/sec"
SR = 16000
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
PARITY_FIXTURE = ROOT / "tests" / "golden" / "ref_base_q8_0_10s_b64.npz"


@dataclass(frozen=True)
class Workload:
    name: str
    arch: str
    dtype: str
    batch: int
    seconds: float = 0.0               # fixed utterance length (0: ragged)
    ragged: tuple = ()                 # (min_s, max_s): seeded uniform lengths per batch
    n_rot: int = 4                     # distinct device batches rotated over the timed steps
    flush_l2: bool = False             # flush L2 before every timed step (time each step alone)
    sweep: int = 0                     # >0: utterances of the multi-device library sweep


WORKLOADS = {w.name: w for w in [
    Workload("base-q8_0-b64-10s", "base", "q8_0", 64, 10.0),
    Workload("base-q8_0-b1-10s", "base", "q8_0", 1, 10.0, n_rot=8, flush_l2=True),
    Workload("base-q4_0-b64-10s", "base", "q4_0", 64, 10.0),
    Workload("large-q8_0-b32-20s", "large", "q8_0", 32, 20.0),
    Workload("xlsr1b-f16-b16-5to30s", "xlsr1b", "f16", 16, ragged=(5.0, 30.0), n_rot=8),
    Workload("sweep-base-q8_0-4096-2to30s", "base", "q8_0", 64, ragged=(2.0, 30.0), sweep=4096),
]}
DEFAULT_WORKLOAD = "base-q8_0-b64-10s"
ARCH_LABEL = {"base": "wav2vec2-base", "large": "wav2vec2-large / XLS-R-300M", "xlsr1b": "XLS-R-1B"}


def pkg():
    from importlib import util
    if "w2v_b200" in sys.modules:
        return sys.modules["w2v_b200"]
    init = ROOT / "wav2vec2.cpp_b200" / "__init__.py"
    spec = util.spec_from_file_location("w2v_b200", init, submodule_search_locations=[str(init.parent)])
    mod = util.module_from_spec(spec)
    sys.modules["w2v_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured (MEASURED_PEAKS.json)"
    return PEAKS_FALLBACK, "fallback (profiling recipe)"


def encoder_frames(n_samples: int) -> int:
    """Encoder frames of an utterance under the wav2vec2 conv stack
    (kernel, stride) = (10, 5), (3, 2) x 4, (2, 2) x 2 (all three
    architectures share it)."""
    n = n_samples
    for k, s in ((10, 5), (3, 2), (3, 2), (3, 2), (3, 2), (2, 2), (2, 2)):
        n = (n - k) // s + 1 if n >= k else 0
    return n


def batch_lengths(wl: Workload, rank: int, j: int) -> list[int]:
    """Sample counts of rank `rank`'s rotating batch j: fixed, or seeded
    uniform lengths in wl.ragged seconds (whole 20 ms frames)."""
    if not wl.ragged:
        return [int(wl.seconds * SR)] * wl.batch
    rng = np.random.default_rng(100_000 + rank * 1000 + j)
    s = rng.uniform(wl.ragged[0], wl.ragged[1], wl.batch)
    return [int(round(v * 50)) * (SR // 50) for v in s]


def workload_config(wl: Workload, world: int, lens_rot=None) -> dict:
    if wl.ragged:
        per = f"{wl.batch} utterances per batch, lengths seeded uniform {wl.ragged[0]:g}-{wl.ragged[1]:g} s"
        if lens_rot:
            allv = [n for b in lens_rot for n in b]
            per += f" (mean {np.mean(allv) / SR:.2f} s over the rotated batches)"
    else:
        n = int(wl.seconds * SR)
        per = f"{wl.batch} utterances x {wl.seconds:g} s per GPU ({n} samples, {encoder_frames(n)} frames each)"
    cfg = {"workload": f"{ARCH_LABEL[wl.arch]} {wl.dtype.upper()} (seeded random init), {per}, greedy CTC",
           "name": wl.name, "per_gpu_batch": wl.batch, "global_batch": wl.batch * world,
           "linears": wl.dtype,
           "parallelism": f"dp{world} (utterances sharded per GPU, no collective on the data path)"}
    if wl.seconds:
        cfg["utterance_seconds"] = wl.seconds
    cfg["l2"] = ("L2 flushed (256 MB write) before every timed step; each step timed alone" if wl.flush_l2 else
                 f"inputs rotate over {wl.n_rot} distinct device batches (together > 126 MB L2); each step also "
                 f"streams >1 GB of activations")
    cfg["launch"] = (f"each of the {wl.n_rot} input batches runs twice before the warm-up steps (the library captures "
                     "the forward as a CUDA graph on its second sight of an input); timed steps replay the graphs")
    return cfg


# ── clocks sampling (nvidia-smi during the timed region) ─────────────────────

class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu_id, self.proc, self.lines = gpu_id, None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", self.gpu_id, f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, pw, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 8:
                continue
            try:
                sm.append(float(f[0])); mx.append(float(f[1]))
                pw.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(pw) if pw else None, "samples": len(sm), "reasons": sorted(reasons)}


def gpu_selector(local: int) -> str:
    import torch
    props = torch.cuda.get_device_properties(local)
    gid = str(getattr(props, "uuid", "")) or str(local)
    return gid if gid.startswith("GPU-") or gid == str(local) else f"GPU-{gid}"


# ── reference CPU implementation ──────────────────────────────────────────────

def usable_cores() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def ref_cli_run(model_path, seconds: float, calls: int, warmup: int = 0, seed: int = 0) -> dict:
    """The reference CLI (oracle/_ref/wav2vec2-cli, its examples/main/main.cpp
    built from source) as the reference is run: one float32 WAV per call,
    -t <usable host cores>, wall time per call (model load and WAV decode
    included, as for any CLI user).  Linears through the ggml-API shim in its
    ggml-emulation mode (activations re-quantised to Q8_0)."""
    import oracle as O
    import w2v_b200.synth as s
    cores = usable_cores()
    n = int(round(seconds * 50)) * (SR // 50)
    env = dict(os.environ, W2V_ORACLE_LINEAR="ggml")
    times = []
    with tempfile.TemporaryDirectory() as td:
        wav = Path(td) / "u.wav"
        s.write_wav_f32(wav, s.make_audio(n, seed))
        for i in range(warmup + calls):
            t0 = time.perf_counter()
            subprocess.run([str(O.REF_CLI), "-m", str(model_path), "-f", str(wav), "-t", str(cores)], check=True,
                           env=env, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            if i >= warmup:
                times.append(time.perf_counter() - t0)
    audio = n / SR
    return {"value": calls * audio / sum(times), "ms_per_step": 1000 * sum(times) / calls, "cores": cores,
            "sample": f"reference CLI -t {cores}, one {audio:g} s WAV per call (utterance seed {seed}), "
                      f"{calls} call(s); linears through the ggml-API shim (Q8_0 activation re-quantisation)"}


def ref_parallel_run(model_path, budget_s: float, seed0: int = 0) -> dict:
    """Throughput of the reference library on all usable cores: one context
    per worker thread (the reference context is not re-entrant,
    src/wav2vec2.cpp:94-97), each transcribing its own utterance prefix with
    n_threads = 1 (ctypes releases the GIL during the call)."""
    import oracle as O
    import w2v_b200.synth as s
    from concurrent.futures import ThreadPoolExecutor
    P = max(1, min(usable_cores(), 32))
    ctxs = [O.RefOracle(model_path, n_threads=1) for _ in range(P)]
    utts = [s.make_audio(int(10 * SR), seed0 + i) for i in range(P)]
    with ThreadPoolExecutor(P) as pool:
        def one_round(n):
            t0 = time.perf_counter()
            list(pool.map(lambda i: ctxs[i].transcribe(utts[i][:n], 1, O.GGML), range(P)))
            return time.perf_counter() - t0
        cal_n = int(0.5 * SR)
        rate = (P * cal_n / SR) / one_round(cal_n)
        sample_s = float(np.clip(budget_s * rate / P, 0.5, 10.0))
        n = int(round(sample_s * 50)) * SR // 50
        dt = one_round(n)
    return {"value": P * n / SR / dt, "unit": UNIT, "cores": P,
            "sample": f"{P} worker threads x first {n / SR:g} s of utterances {seed0}..{seed0 + P - 1} (10 s "
                      f"each, seeded), reference library n_threads=1 each, ggml-shim linears"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    pkg()
    import w2v_b200.synth as s
    wl = WORKLOADS[args.workload]
    line = {"metric": METRIC, "impl": "reference", "unit": UNIT, "higher_is_better": True, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "scaling": "weak", "dtype": "fp32", "data": "synthetic",
            "config": workload_config(wl, args.world), "vs_baseline": None}
    if not O.ref_available():
        line.update({"unavailable": "reference CPU build oracle/_ref is absent (build here with make -C oracle ref)"})
        print(json.dumps(line), flush=True)
        return
    p = s.cached_model(args.cache, wl.arch, wl.dtype)
    # each step one CLI call; the WAV is as long as the workload's utterances
    # unless K + W calls of that length would exceed the budget
    probe = ref_cli_run(p, 1.0, 1)
    per_audio_s = probe["ms_per_step"] / 1000.0          # wall seconds per audio second (upper bound)
    full = wl.seconds or wl.ragged[1]
    secs = float(np.clip(args.ref_budget / max(1, args.steps + args.warmup) / per_audio_s, 1.0, full))
    r = ref_cli_run(p, secs, args.steps, args.warmup)
    line.update({"value": r["value"], "ms_per_step": r["ms_per_step"],
                 "cpu_baseline": {"value": r["value"], "unit": UNIT, "cores": r["cores"], "kind": "reference",
                                  "sample": r["sample"]},
                 "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
    if not args.no_parallel_baseline:
        line["cpu_parallel"] = ref_parallel_run(p, args.parallel_budget)
    print(json.dumps(line), flush=True)


# ── sharding helpers (one process per GPU, weak scaling) ─────────────────────

def rank_seeds(rank: int, n_rot: int, batch: int) -> list[list[int]]:
    """Utterance seeds of this rank's n_rot batches: disjoint across ranks, so
    N ranks process N different sets of utterances (no shared state)."""
    base = rank * n_rot * batch
    return [[base + j * batch + i for i in range(batch)] for j in range(n_rot)]


def max_over_ranks(values, world: int, device=None):
    """Element-wise max of per-rank timings (the whole job is as slow as its
    slowest rank); identity when world == 1."""
    import torch
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


# ── parity at the default workload (against the reference's golden outputs) ──

def collapse_ids(ids, blank: int = 0) -> np.ndarray:
    """Greedy CTC token sequence of per-frame argmax ids: runs collapsed,
    blank dropped (the reference's src/ops.h:132-149, src/wav2vec2.cpp:500-502)."""
    ids = np.asarray(ids)
    if ids.size == 0:
        return ids
    keep = np.ones(ids.size, bool)
    keep[1:] = ids[1:] != ids[:-1]
    r = ids[keep]
    return r[r != blank]


def parity_report(logits: list, fx) -> dict:
    """Agreement of this engine's logits for the fixture's utterances with the
    reference's forward pass in its two linear modes (exact fp32 linears, and
    ggml-emulated activation re-quantisation): greedy-sequence identity rate,
    per-frame argmax agreement, logit max-abs error (on the utterances whose
    full logits the fixture keeps) and the margin rule (frames whose exact
    reference top-1/top-2 margin exceeds twice that error must agree)."""
    seeds = [int(s) for s in fx["seeds"]]
    ids = np.stack([lg.argmax(1) for lg in logits])
    ex, gg = fx["ids_exact"], fx["ids_ggml"]
    full = [seeds.index(int(s)) for s in fx["full_seeds"]]
    err_ex = max(float(np.abs(logits[i] - fx["logits_exact_full"][k]).max()) for k, i in enumerate(full))
    err_gg = max(float(np.abs(logits[i] - fx["logits_ggml_full"][k]).max()) for k, i in enumerate(full))
    ref_gap = max(float(np.abs(fx["logits_ggml_full"][k] - fx["logits_exact_full"][k]).max())
                  for k in range(len(full)))
    seq = lambda a, b: float(np.mean([np.array_equal(collapse_ids(x), collapse_ids(y)) for x, y in zip(a, b)]))
    safe = fx["margin_exact"] > 2 * err_ex
    return {"utterances": len(seeds), "reference": "oracle/_ref golden outputs (tests/golden/ref_base_q8_0_10s_b64.npz)",
            "greedy_sequences_identical_vs_exact": seq(ids, ex),
            "greedy_sequences_identical_vs_ggml": seq(ids, gg),
            "reference_exact_vs_ggml_sequences_identical": seq(ex, gg),
            "frame_argmax_agree_vs_exact": float((ids == ex).mean()),
            "frame_argmax_agree_vs_ggml": float((ids == gg).mean()),
            "logits_max_abs_vs_exact": err_ex, "logits_max_abs_vs_ggml": err_gg,
            "reference_ggml_vs_exact_max_abs": ref_gap,
            "logits_max_abs_utterances": len(full),
            "margin_rule_frames": int(safe.sum()), "margin_rule_violations": int((safe & (ids != ex)).sum())}


# ── our engine ────────────────────────────────────────────────────────────────

def flush_l2(buf):
    buf.zero_()


def run_ours(args):
    import torch
    import torch.distributed as dist
    wl = WORKLOADS[args.workload]
    rank, world, local = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), \
        int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"), timeout=timedelta(seconds=300))
    pkg()
    import w2v_b200.binding as b
    import w2v_b200.synth as s

    def barrier():
        if world > 1:
            dist.barrier()

    # model: generated once per machine (rank 0 writes, the others wait)
    if rank == 0:
        mp = s.cached_model(args.cache, wl.arch, wl.dtype)
    barrier()
    mp = s.cached_model(args.cache, wl.arch, wl.dtype)
    m = b.Model(mp, devices=[local])

    seeds = rank_seeds(rank, wl.n_rot, wl.batch)
    lens_rot = [batch_lengths(wl, rank, j) for j in range(wl.n_rot)]
    host_batches = [[s.make_audio(n, sd) for n, sd in zip(lens, sds)] for lens, sds in zip(lens_rot, seeds)]
    dev_batches = [torch.from_numpy(np.concatenate(hb)).cuda() for hb in host_batches]
    stream = torch.cuda.Stream()

    def step(j):
        m.forward_device(dev_batches[j % wl.n_rot].data_ptr(), lens_rot[j % wl.n_rot], stream.cuda_stream)

    with torch.cuda.stream(stream):
        # The library captures the forward of a (device input, lengths) pair as
        # a CUDA graph the second time it sees it and replays it after that:
        # run every input batch twice before the warm-up steps, so that no
        # capture falls inside the timed steps.
        for j in range(2 * wl.n_rot):
            step(j)
        for j in range(args.warmup):
            step(j)
    stream.synchronize()
    launches = m.launches_per_forward()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if wl.flush_l2 else None
    sampler = ClockSampler(gpu_selector(local))
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    if flush is None:
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for j in range(args.steps):
                step(j)
            ev1.record(stream)
        stream.synchronize()
        elapsed_ms = ev0.elapsed_time(ev1)
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)]
        with torch.cuda.stream(stream):
            for j in range(args.steps):
                flush_l2(flush)
                evs[j][0].record(stream)
                step(j)
                evs[j][1].record(stream)
        stream.synchronize()
        elapsed_ms = sum(a.elapsed_time(c) for a, c in evs)
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    audio_timed = sum(sum(lens_rot[j % wl.n_rot]) for j in range(args.steps)) / SR
    # per-phase breakdown: a separate pass with an event pair around every
    # launch, outside the timed steps
    steps_prof = max(1, min(args.steps, 10))
    m.profile(True)
    with torch.cuda.stream(stream):
        for j in range(steps_prof):
            step(j)
    stream.synchronize()
    prof = m.profile_read()
    m.profile(False)

    # end-to-end through the public API: pinned host arrays in (each step's
    # host->device copy happens inside the call), transcripts out
    e2e = None
    if not args.no_e2e:
        pinned = [[torch.from_numpy(x).pin_memory() for x in hb] for hb in host_batches]
        e2e_batches = [[t.numpy() for t in hb] for hb in pinned]
        for j in range(2):
            m.transcribe_batch(e2e_batches[j % wl.n_rot])
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for j in range(args.e2e_steps):
            m.transcribe_batch(e2e_batches[j % wl.n_rot])
        e2e_s = time.perf_counter() - t0
        barrier()
        idx = [j % wl.n_rot for j in range(args.e2e_steps)]
        e2e = {"seconds": e2e_s, "audio": sum(sum(lens_rot[j]) for j in idx) / SR,
               "h2d": sum(4 * sum(lens_rot[j]) for j in idx) / args.e2e_steps,
               "d2h": sum(12 * sum(encoder_frames(n) for n in lens_rot[j]) + 4 * wl.batch + 4
                          for j in idx) / args.e2e_steps}

    # parity of the default workload's first batch (seeds 0..63 on rank 0)
    # against the reference's golden outputs
    parity = None
    if (rank == 0 and wl.name == DEFAULT_WORKLOAD and not args.no_parity and PARITY_FIXTURE.exists()):
        fx = np.load(PARITY_FIXTURE)
        if [int(v) for v in fx["seeds"]] == seeds[0]:
            parity = parity_report(m.logits(host_batches[0]), fx)

    t_max = max_over_ranks([elapsed_ms, e2e["seconds"] if e2e else 0.0], world, device="cuda")
    elapsed_ms = t_max[0]
    if e2e:
        e2e["seconds"] = t_max[1]
    all_clocks = [None] * world
    if world > 1:
        dist.all_gather_object(all_clocks, clocks)
    else:
        all_clocks = [clocks]

    cpu = None
    if rank == 0 and world == 1 and wl.name == DEFAULT_WORKLOAD and not args.no_cpu_baseline:
        import oracle as O
        if O.ref_available():
            r = ref_cli_run(mp, wl.seconds, 1)
            cpu = {"value": r["value"], "unit": UNIT, "cores": r["cores"], "kind": "reference",
                   "sample": r["sample"]}
            if not args.no_parallel_baseline:
                cpu["parallel"] = ref_parallel_run(mp, args.parallel_budget)
        else:
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                   "sample": "unavailable: oracle/_ref build absent"}

    if rank == 0:
        line = result_line(args, wl, world, elapsed_ms, audio_timed, prof, steps_prof, launches, all_clocks, e2e,
                           cpu, lens_rot)
        if parity:
            line["parity"] = parity
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def result_line(args, wl, world, elapsed_ms, audio_timed, prof, steps_prof, launches, all_clocks, e2e, cpu,
                lens_rot=None) -> dict:
    """The benchmark's JSON line from its measurements: elapsed_ms over
    args.steps timed steps that carried audio_timed seconds of audio per rank
    (max over ranks), prof the per-category event times of steps_prof
    profiled steps ({name: {"ms", "launches", "flops"}}), launches per
    forward, one clock record per rank, e2e {"seconds", "audio", "h2d",
    "d2h"} for args.e2e_steps calls of the public batch API per rank (None:
    not measured), cpu the CPU-baseline record or None."""
    value = world * audio_timed / (elapsed_ms / 1000.0)
    pk, pk_src = peaks()
    g = prof.get("gemm_encoder", {"ms": 0, "launches": 0, "flops": 0})
    achieved = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] else 0.0
    peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    total_flops = sum(v["flops"] for v in prof.values())
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)", "data": "synthetic",
        "config": workload_config(wl, world, lens_rot),
        "roofline": {"bound": "tensor",
                     "kernel": ("qgemm_kernel on the encoder linears (dequant-fused tcgen05 GEMM, "
                                f"{wl.dtype} weights expanded into TMEM)" if wl.dtype in ("q8_0", "q4_0") else
                                "gemm_tc_kernel / gemm2_tc_kernel on the encoder linears (tcgen05, TMEM)"),
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if peak else None,
                     "traffic": encoder_gemm_traffic(wl),
                     "traffic_source": ENCODER_GEMM_TRAFFIC_SOURCE,
                     "peak_source": f"bf16 dense sustained, {pk_src}",
                     "frac_of_burst_peak": achieved / pk["bf16_tflops"] if pk.get("bf16_tflops") else None,
                     "launches": g["launches"], "avg_launch_ms": g["ms"] / max(1, g["launches"]),
                     "flops_per_launch": g["flops"] / max(1, g["launches"])},
        "step_tflops": total_flops / steps_prof / (elapsed_ms / args.steps / 1000.0) / 1e12,
        "breakdown_ms_per_step": {k: v["ms"] / steps_prof for k, v in prof.items()},
        "gpu_launches": launches * args.steps * world,
        "clocks": {"sm_mhz": all_clocks[0].get("sm_mhz"), "sm_max_mhz": all_clocks[0].get("sm_max_mhz"),
                   "reasons": sorted(set(r for c in all_clocks for r in c.get("reasons", []))),
                   "samples": all_clocks[0].get("samples"),
                   "per_rank_sm_mhz": [c.get("sm_mhz") for c in all_clocks]},
    }
    if e2e and e2e.get("seconds"):
        # per step: the pinned float32 audio in; spans (3 ints per frame), span counts and the
        # device error word out
        line["e2e"] = {"value": world * e2e["audio"] / e2e["seconds"], "unit": UNIT,
                       "h2d_bytes_per_step": int(e2e["h2d"]), "d2h_bytes_per_step": int(e2e["d2h"]),
                       "steps": args.e2e_steps,
                       "api": "wav2vec2_transcribe_batch (pinned host float32 in, text out)"}
    if cpu:
        line["cpu_baseline"] = cpu
    return line


# DRAM bytes per launch of the four encoder linears of wav2vec2-base at 64 x
# 499 rows on Q8_0 weights through the dequant-fused GEMM (QKV, attention
# out-projection + LayerNorm residual, FFN up + GELU, FFN down + LayerNorm
# residual), from one ncu capture of each on B200 (profiles/qgemm_encoder_traffic_b64.md
# gives the commands and the per-linear figures).
ENCODER_GEMM_DRAM_BYTES = {"qkv": 146.2e6, "out_proj": 189.2e6, "ffn_up": 194.2e6, "ffn_down": 365.4e6}
ENCODER_GEMM_TRAFFIC_SOURCE = ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of each encoder "
                               "linear through the dequant-fused GEMM on Q8_0 weights at 64 x 499 rows, mean per "
                               "launch (profiles/qgemm_encoder_traffic_b64.md)")


def encoder_gemm_traffic(wl: Workload):
    """Mean DRAM traffic per encoder-GEMM launch for the default workload
    (None for other workloads, which were not captured)."""
    if wl.name != DEFAULT_WORKLOAD:
        return None
    return sum(ENCODER_GEMM_DRAM_BYTES.values()) / len(ENCODER_GEMM_DRAM_BYTES)


# ── the whole-box sweep through the library's own multi-device scheduler ─────

def sweep_lengths(n: int, lo: float, hi: float, seed: int = 4096) -> list[int]:
    rng = np.random.default_rng(seed)
    return [int(round(v * 50)) * (SR // 50) for v in rng.uniform(lo, hi, n)]


def run_sweep(args):
    """4096 ragged utterances through wav2vec2_transcribe_batch on one context
    over devices 0..N-1: the library length-buckets them into batches of <= 64
    and feeds the devices from one queue (one host thread + stream each).
    Greedy CTC on the GPU, then beam width 5 on the host pool from GPU logits.
    Wall time of the API call (host audio in, transcripts out)."""
    import torch
    from concurrent.futures import ThreadPoolExecutor
    wl = WORKLOADS[args.workload]
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:       # one process drives every device
        return
    n_dev = args.gpus
    pkg()
    import w2v_b200.binding as b
    import w2v_b200.synth as s
    mp = s.cached_model(args.cache, wl.arch, wl.dtype)
    lens = sweep_lengths(wl.sweep, *wl.ragged)
    with ThreadPoolExecutor(min(32, usable_cores())) as pool:
        audio = list(pool.map(lambda i: s.make_audio(lens[i], 500_000 + i), range(len(lens))))
    total_s = sum(lens) / SR
    m = b.Model(mp, devices=list(range(n_dev)), max_batch=wl.batch)
    # warm-up: one untimed pass over the same utterances, so every batch worker
    # (two per device on several devices) has allocated its workspace and pinned
    # staging for the batch sizes it will see
    m.transcribe_batch(audio)
    torch.cuda.synchronize()
    cores = usable_cores()
    out = {"metric": METRIC, "workload": wl.name, "n_gpus": n_dev, "unit": UNIT, "higher_is_better": True,
           "utterances": len(lens), "audio_seconds": total_s, "data": "synthetic",
           "config": {"workload": f"wav2vec2-base Q8_0 (seeded random init), {len(lens)} utterances, lengths "
                                  f"seeded uniform {wl.ragged[0]:g}-{wl.ragged[1]:g} s, length-bucketed into "
                                  f"batches of <= {wl.batch} by the library, one context over {n_dev} device(s)",
                      "api": "wav2vec2_transcribe_batch (pageable host float32 in, text out)",
                      "busy": "per device, the device time of its batches summed over its engines (two per device "
                              "on a context over several devices, whose batches overlap: the fraction may exceed 1)"}}
    sampler = ClockSampler("0")
    sampler.start()
    for beam in (1, 5):
        m.device_stats(reset=True)
        t0 = time.perf_counter()
        res = m.transcribe_batch(audio, beam_size=beam, n_threads=cores)
        wall = time.perf_counter() - t0
        st = m.device_stats()
        busy = [d["busy_ms"] / 1000.0 for d in st]
        out[f"beam{beam}"] = {
            "value": total_s / wall, "wall_s": wall, "decoder_threads": cores if beam > 1 else 0,
            "per_gpu_busy_s": busy, "per_gpu_batches": [d["batches"] for d in st],
            "per_gpu_audio_s": [d["samples"] / SR for d in st],
            "gpu_busy_frac_of_wall": [x / wall for x in busy],
            "transcripts": len(res)}
    out["clocks_gpu0"] = sampler.stop()
    out["value"] = out["beam1"]["value"]
    m.close()
    print(json.dumps(out), flush=True)


def run_kernel_case(args):
    """One kernel at a representative size (for ncu captures and micro-timing):
    gemm: M rows x K -> N with the given epilogue (default the encoder FFN-up
          shape, K=768 -> N=3072, fp16 out, GELU epilogue);
    attention: 64 utterances x 499 frames, 12 heads x 64;
    pos_conv: the same batch, hidden 768, kernel 128, 16 groups;
    layer_norm: M rows of --ln-dim (fp32 in, fp16 + row statistics out)."""
    import torch
    pkg()
    import w2v_b200.binding as b
    K = b.kernels
    torch.manual_seed(0)
    st = torch.cuda.current_stream().cuda_stream
    M = args.rows
    if args.kernel == "gemm":
        N, Kd, epi = (int(v) for v in args.gemm_shape.split(","))
        A = torch.randn(M, Kd, device="cuda").half()
        W = (torch.randn(N, Kd, device="cuda") * 0.05).half()
        bias = torch.randn(N, device="cuda")
        f16 = epi in (0, 1)
        out = torch.zeros(M, N, device="cuda", dtype=torch.float16 if f16 else torch.float32)
        res = out.data_ptr() if epi == 3 else 0
        fn = lambda: K.gemm(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, out.data_ptr(), N, M, M,
                            bias.data_ptr(), res, N, epi, args.block_n, 0, st)
        if args.weights != "f16":
            # the same shape on quantised weights through the dequant-fused GEMM
            import w2v_b200.synth as s
            gt = 8 if args.weights == "q8_0" else 2
            wq = (np.random.default_rng(0).standard_normal((N, Kd)) * 0.02).astype(np.float32)
            raw = s.quantize_q8_0(wq) if gt == 8 else s.quantize_q4_0(wq)
            raw_d = torch.from_numpy(np.frombuffer(raw, np.uint8).copy()).cuda()
            ld = (N + 7) // 8 * 8
            codes = torch.empty(N * Kd // (1 if gt == 8 else 2), dtype=torch.uint8, device="cuda")
            scales = torch.zeros(Kd // 32, ld, dtype=torch.int16, device="cuda")
            K.repack_q(raw_d.data_ptr(), gt, N, Kd, codes.data_ptr(), scales.data_ptr(), ld, st)
            fn = lambda: K.gemm_q(A.data_ptr(), Kd, M, codes.data_ptr(), scales.data_ptr(), ld, gt, N, out.data_ptr(),
                                  N, bias.data_ptr(), res, N, epi, args.block_n, 0, st)
        if epi == 4:
            # residual normalised on the fly from per-row (mean, rstd), in place over C
            stats = torch.stack([torch.randn(M), torch.rand(M) + 0.5], 1).cuda()
            lw, lb = torch.ones(N, device="cuda"), torch.zeros(N, device="cuda")
            fn = lambda: K.gemm_ln_resid(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, out.data_ptr(),
                                         N, M, M, bias.data_ptr(), out.data_ptr(), N, stats.data_ptr(),
                                         lw.data_ptr(), lb.data_ptr(), block_n=args.block_n, stream=st)
            if args.weights != "f16":
                fn = lambda: K.gemm_q_ln_resid(A.data_ptr(), Kd, M, codes.data_ptr(), scales.data_ptr(), ld, gt, N,
                                               out.data_ptr(), N, bias.data_ptr(), out.data_ptr(), N,
                                               stats.data_ptr(), lw.data_ptr(), lb.data_ptr(), args.block_n, 0, st)
        flops = 2.0 * M * N * Kd
    elif args.kernel == "attention":
        H, nh, T, B = 768, 12, 499, 64
        qkv = torch.randn(B * T, 3 * H, device="cuda").half()
        out = torch.empty(B * T, H, device="cuda", dtype=torch.float16)
        off = torch.arange(B, device="cuda", dtype=torch.int64) * T
        Tt = torch.full((B,), T, device="cuda", dtype=torch.int32)
        fn = lambda: K.attention(qkv.data_ptr(), out.data_ptr(), off.data_ptr(), Tt.data_ptr(), B, H, nh, T, B * T, 0, st)
        flops = 4.0 * B * T * T * H
    elif args.kernel == "layer_norm":
        # post-LN encoder LayerNorm: fp32 rows in, fp16 normalised rows + (mean, rstd) out
        H, M = args.ln_dim, args.rows
        x = torch.randn(M, H, device="cuda")
        xh = torch.empty(M, H, device="cuda", dtype=torch.float16)
        stats = torch.empty(M, 2, device="cuda")
        lw, lb = torch.randn(H, device="cuda"), torch.randn(H, device="cuda")
        fn = lambda: K.layer_norm_stats(x.data_ptr(), M, H, lw.data_ptr(), lb.data_ptr(), xh.data_ptr(),
                                        stats.data_ptr(), st)
        flops = 0.0
        nbytes = M * H * (4 + 2) + M * 8
    else:
        H, G, Kp, T, B = 768, 16, 128, 499, 64
        x = torch.randn(B * T, H, device="cuda")
        out = torch.empty_like(x)
        wt = (torch.randn(G, Kp, H // G, H // G, device="cuda") * 0.02).half()
        bias = torch.randn(H, device="cuda")
        off = torch.arange(B, device="cuda", dtype=torch.int64) * T
        Tt = torch.full((B,), T, device="cuda", dtype=torch.int32)
        fn = lambda: K.pos_conv(out.data_ptr(), x.data_ptr(), off.data_ptr(), Tt.data_ptr(), B, H, Kp, G,
                                wt.data_ptr(), bias.data_ptr(), T, 0, st)
        flops = 2.0 * B * T * Kp * (H // G) * H
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    rec = {"kernel": args.kernel, "rows": M, "ms": ms, "tflops": flops / ms / 1e9}
    if args.kernel == "layer_norm":
        rec = {"kernel": args.kernel, "rows": M, "ms": ms, "gbs": nbytes / ms / 1e6}
    if args.kernel == "gemm":
        rec.update(shape=args.gemm_shape, block_n=args.block_n, weights=args.weights)
    print(json.dumps(rec), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default=DEFAULT_WORKLOAD)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parallel-baseline", action="store_true")
    ap.add_argument("--parallel-budget", type=float, default=10.0,
                    help="seconds of the all-cores reference throughput sample")
    ap.add_argument("--ref-budget", type=float, default=150.0, help="seconds for the --impl reference CLI calls")
    ap.add_argument("--cache", default=os.environ.get("W2V_MODEL_CACHE", "/tmp/w2v_models"))
    ap.add_argument("--kernel", choices=["gemm", "attention", "pos_conv", "layer_norm"], default=None,
                    help="time one kernel at a representative size instead of the whole step")
    ap.add_argument("--rows", type=int, default=32768, help="GEMM rows for --kernel gemm")
    ap.add_argument("--gemm-shape", default="3072,768,1",
                    help="N,K,epilogue for --kernel gemm (epilogue 0 fp16, 1 fp16+GELU, 2 fp32, 3 fp32+residual, "
                         "4 fp32+LayerNorm-normalised residual)")
    ap.add_argument("--weights", choices=["f16", "q8_0", "q4_0"], default="f16",
                    help="B operand of --kernel gemm: fp16 rows, or quantised through the dequant-fused GEMM")
    ap.add_argument("--ln-dim", type=int, default=768, help="row width for --kernel layer_norm")
    ap.add_argument("--block-n", type=int, default=0,
                    help="GEMM tile for --kernel gemm: 0 automatic, 64/128/256 one CTA, -128/-256 CTA pair")
    args = ap.parse_args()
    if args.kernel:
        run_kernel_case(args)
        return
    args.world = int(os.environ.get("WORLD_SIZE", args.gpus))
    if args.impl == "reference":
        run_reference(args)
    elif WORKLOADS[args.workload].sweep:
        run_sweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

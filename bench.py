#!/usr/bin/env python3
"""Benchmark: wav2vec2-base (random-init, seeded) Q8_0, 64 utterances x 10 s
per GPU (499 frames each), greedy CTC -- audio-seconds per second.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one forward pass (waveform -> conv extractor -> projection ->
positional conv -> 12 encoder layers -> CTC head -> greedy CTC spans) over one
batch of 64 utterances.  `value` is timed with CUDA events on the forward's
stream over exactly K steps with the inputs already in HBM (4 distinct
batches rotate, 164 MB > 126 MB L2); `e2e` times the public C API
(wav2vec2_transcribe_batch) from host arrays to transcripts, host<->device
copies included.  Multi-GPU: one process per GPU (torchrun), utterances
sharded (weak scaling, no collective on the data path); barriers and the
max-over-ranks timing use torch.distributed.

`--impl reference` times the reference's own CPU implementation (its
wav2vec2.cpp built from its sources against the oracle's ggml-API shim,
oracle/_ref) on the host cores, utterances in parallel on all usable cores.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "oracle"))
METRIC = "audio-sec/sec (inverse RTF), base Q8_0 batch 64, 1/2/4/8 B200; % MMA peak"
UNIT = "audio-sec/sec"
SR = 16000
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


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
    """Encoder frames of an utterance under the base model's conv stack
    (kernel, stride) = (10, 5), (3, 2) x 4, (2, 2) x 2."""
    n = n_samples
    for k, s in ((10, 5), (3, 2), (3, 2), (3, 2), (3, 2), (2, 2), (2, 2)):
        n = (n - k) // s + 1 if n >= k else 0
    return n


def workload(args) -> dict:
    n = int(args.seconds * SR)
    return {"workload": f"wav2vec2-base {args.dtype.upper()} (seeded random init), {args.batch} utterances x "
                        f"{args.seconds:g} s per GPU ({n} samples, {encoder_frames(n)} frames each), greedy CTC",
            "per_gpu_batch": args.batch, "global_batch": args.batch * args.world,
            "utterance_seconds": args.seconds, "linears": args.dtype,
            "parallelism": f"dp{args.world} (utterances sharded per GPU, no collective on the data path)",
            "l2": "inputs rotate over 4 distinct device batches (4 x 41 MB > 126 MB L2); each step also streams "
                  ">2 GB of activations"}


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


# ── reference CPU implementation ──────────────────────────────────────────────

def ref_cpu_run(model_path, seconds_total_budget: float, steps: int, warmup: int, batch_seed: int = 0):
    """Time the reference's own CPU path on all usable host cores: one context
    per worker thread (the reference context is not re-entrant,
    src/wav2vec2.cpp:94-97), each worker transcribing its own sample with
    n_threads = 1 (ctypes releases the GIL during the call)."""
    import oracle as O
    import w2v_b200.synth as s
    from concurrent.futures import ThreadPoolExecutor
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    P = max(1, min(cores, 32))
    ctxs = [O.RefOracle(model_path, n_threads=1) for _ in range(P)]
    utts = [s.make_audio(int(10 * SR), batch_seed + i) for i in range(P)]
    pool = ThreadPoolExecutor(P)

    def one_round(n):
        t0 = time.perf_counter()
        list(pool.map(lambda i: ctxs[i].transcribe(utts[i][:n], 1, O.GGML), range(P)))
        return time.perf_counter() - t0

    # calibrate on a short sample, then size each step to the budget
    cal_n = int(0.5 * SR)
    rate = (P * cal_n / SR) / one_round(cal_n)                # audio-s per wall-s, all workers
    per_step = seconds_total_budget / max(1, steps + warmup)
    sample_s = float(np.clip(per_step * rate / P, 0.5, 10.0))
    n = int(round(sample_s * 50)) * SR // 50                  # whole 20 ms frames
    for _ in range(warmup):
        one_round(n)
    times = [one_round(n) for _ in range(steps)]
    pool.shutdown()
    audio = P * n / SR
    total = sum(times)
    return {"value": steps * audio / total, "ms_per_step": 1000 * total / steps, "cores": P,
            "sample": f"{P} workers x first {n / SR:g} s of utterances 0..{P - 1} (10 s each, seeded), "
                      f"1 thread each, ggml-shim Q8_0 activation re-quantisation in the linears",
            "audio_s_per_step": audio}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    pkg()
    import w2v_b200.synth as s
    line = {"metric": METRIC, "impl": "reference", "unit": UNIT, "higher_is_better": True, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "scaling": "weak", "dtype": "fp32", "data": "synthetic",
            "config": workload(args), "vs_baseline": None}
    if not O.ref_available():
        line.update({"unavailable": "reference CPU build oracle/_ref/libw2v_ref.so is absent (build here with "
                                    "make -C oracle ref)"})
        print(json.dumps(line), flush=True)
        return
    p = s.cached_model(args.cache, "base", args.dtype)
    r = ref_cpu_run(p, args.ref_budget, args.steps, args.warmup)
    line.update({"value": r["value"], "ms_per_step": r["ms_per_step"],
                 "cpu_baseline": {"value": r["value"], "unit": UNIT, "cores": r["cores"], "kind": "reference",
                                  "sample": r["sample"]},
                 "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}})
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


# ── our engine ────────────────────────────────────────────────────────────────

def run_ours(args):
    import torch
    import torch.distributed as dist
    rank, world, local = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), \
        int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"), timeout=timedelta(seconds=300))
    P = pkg()
    import w2v_b200.binding as b
    import w2v_b200.synth as s

    def barrier():
        if world > 1:
            dist.barrier()

    # model: generated once per machine (rank 0 writes, the others wait)
    if rank == 0:
        mp = s.cached_model(args.cache, "base", args.dtype)
    barrier()
    mp = s.cached_model(args.cache, "base", args.dtype)
    m = b.Model(mp, devices=[local])

    n = int(args.seconds * SR)
    n_rot = 4
    host_batches = [[s.make_audio(n, sd) for sd in seeds] for seeds in rank_seeds(rank, n_rot, args.batch)]
    dev_batches = [torch.from_numpy(np.concatenate(hb)).cuda() for hb in host_batches]
    lens = [n] * args.batch
    stream = torch.cuda.Stream()

    def step(j):
        m.forward_device(dev_batches[j % n_rot].data_ptr(), lens, stream.cuda_stream)

    with torch.cuda.stream(stream):
        for j in range(args.warmup):
            step(j)
    stream.synchronize()
    launches = m.launches_per_forward()
    props = torch.cuda.get_device_properties(local)
    gid = str(getattr(props, "uuid", "")) or str(local)
    sampler = ClockSampler(gid if gid.startswith("GPU-") or gid == str(local) else f"GPU-{gid}")
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for j in range(args.steps):
            step(j)
        ev1.record(stream)
    stream.synchronize()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop()
    elapsed_ms = ev0.elapsed_time(ev1)
    # per-phase breakdown: a separate pass with an event pair around every
    # launch (which also runs the encoder on one stream), outside the timed steps
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
    e2e_s = None
    if not args.no_e2e:
        pinned = [[torch.from_numpy(x).pin_memory() for x in hb] for hb in host_batches]
        e2e_batches = [[t.numpy() for t in hb] for hb in pinned]
        for j in range(2):
            m.transcribe_batch(e2e_batches[j % n_rot])
        barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for j in range(args.e2e_steps):
            m.transcribe_batch(e2e_batches[j % n_rot])
        e2e_s = time.perf_counter() - t0
        barrier()

    elapsed_ms, e2e_s = max_over_ranks([elapsed_ms, e2e_s or 0.0], world, device="cuda")
    if world > 1:
        all_clocks = [None] * world
        dist.all_gather_object(all_clocks, clocks)
    else:
        all_clocks = [clocks]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle as O
        if O.ref_available():
            r = ref_cpu_run(mp, args.cpu_budget, 1, 0)
            cpu = {"value": r["value"], "unit": UNIT, "cores": r["cores"], "kind": "reference",
                   "sample": r["sample"]}
        else:
            cpu = {"value": None, "unit": UNIT, "cores": 0, "kind": "reference",
                   "sample": "unavailable: oracle/_ref build absent"}

    if rank == 0:
        print(json.dumps(result_line(args, world, elapsed_ms, prof, steps_prof, launches, all_clocks, e2e_s, cpu)),
              flush=True)
    m.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def result_line(args, world, elapsed_ms, prof, steps_prof, launches, all_clocks, e2e_s, cpu) -> dict:
    """The benchmark's JSON line from its measurements: elapsed_ms over
    args.steps timed steps (max over ranks), prof the per-category event
    times of steps_prof profiled steps ({name: {"ms", "launches", "flops"}}),
    launches per forward, one clock record per rank, e2e_s seconds for
    args.e2e_steps calls of the public batch API (0 or None: not measured),
    cpu the CPU-baseline record or None."""
    n = int(args.seconds * SR)
    audio_per_step = args.batch * args.seconds
    value = world * args.steps * audio_per_step / (elapsed_ms / 1000.0)
    pk, pk_src = peaks()
    g = prof.get("gemm_encoder", {"ms": 0, "launches": 0, "flops": 0})
    achieved = g["flops"] / (g["ms"] / 1000.0) / 1e12 if g["ms"] else 0.0
    peak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    total_flops = sum(v["flops"] for v in prof.values())
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp16 (fp32 accumulate)", "data": "synthetic",
        "config": workload(args),
        "roofline": {"bound": "tensor",
                     "kernel": "gemm_tc_kernel / gemm2_tc_kernel on the encoder linears (tcgen05, TMEM)",
                     "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak if peak else None,
                     "traffic": encoder_gemm_traffic(args),
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch of each "
                                       "encoder linear at this workload, mean per launch",
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
    if e2e_s:
        # per step: the pinned float32 audio in; spans (3 ints per frame), span counts and the
        # device error word out
        line["e2e"] = {"value": world * args.e2e_steps * audio_per_step / e2e_s, "unit": UNIT,
                       "h2d_bytes_per_step": args.batch * n * 4,
                       "d2h_bytes_per_step": encoder_frames(n) * args.batch * 3 * 4 + args.batch * 4 + 4,
                       "steps": args.e2e_steps, "api": "wav2vec2_transcribe_batch (pinned host float32 in, text out)"}
    if cpu:
        line["cpu_baseline"] = cpu
    return line


# DRAM bytes per launch of the four encoder linears of wav2vec2-base at 64 x
# 499 rows (QKV, attention out-projection + residual, FFN up + GELU, FFN down +
# residual), measured with ncu on B200 on one launch each.
ENCODER_GEMM_DRAM_BYTES = {"qkv": 147.9e6, "out_proj": 188.4e6, "ffn_up": 197.4e6, "ffn_down": 372.5e6}


def encoder_gemm_traffic(args):
    """Mean DRAM traffic per encoder-GEMM launch for the default workload
    (None for other workloads, which were not captured)."""
    if (args.dtype, args.batch, args.seconds) != ("q8_0", 64, 10.0):
        return None
    return sum(ENCODER_GEMM_DRAM_BYTES.values()) / len(ENCODER_GEMM_DRAM_BYTES)


def run_kernel_case(args):
    """One kernel at a representative size (for ncu captures and micro-timing):
    gemm: M rows x K -> N with the given epilogue (default the encoder FFN-up
          shape, K=768 -> N=3072, fp16 out, GELU epilogue);
    attention: 64 utterances x 499 frames, 12 heads x 64;
    pos_conv: the same batch, hidden 768, kernel 128, 16 groups."""
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
        if epi == 4:
            # residual normalised on the fly from per-row (mean, rstd), in place over C
            stats = torch.stack([torch.randn(M), torch.rand(M) + 0.5], 1).cuda()
            lw, lb = torch.ones(N, device="cuda"), torch.zeros(N, device="cuda")
            fn = lambda: K.gemm_ln_resid(A.data_ptr(), Kd, 1, 1, Kd, M, 1, M * Kd, W.data_ptr(), N, out.data_ptr(),
                                         N, M, M, bias.data_ptr(), out.data_ptr(), N, stats.data_ptr(),
                                         lw.data_ptr(), lb.data_ptr(), block_n=args.block_n, stream=st)
        flops = 2.0 * M * N * Kd
    elif args.kernel == "attention":
        H, nh, T, B = 768, 12, 499, 64
        qkv = torch.randn(B * T, 3 * H, device="cuda").half()
        out = torch.empty(B * T, H, device="cuda", dtype=torch.float16)
        off = torch.arange(B, device="cuda", dtype=torch.int64) * T
        Tt = torch.full((B,), T, device="cuda", dtype=torch.int32)
        fn = lambda: K.attention(qkv.data_ptr(), out.data_ptr(), off.data_ptr(), Tt.data_ptr(), B, H, nh, T, B * T, 0, st)
        flops = 4.0 * B * T * T * H
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
    if args.kernel == "gemm":
        rec.update(shape=args.gemm_shape, block_n=args.block_n)
    print(json.dumps(rec), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=60)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dtype", choices=["q8_0", "q4_0", "f16"], default="q8_0")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--seconds", type=float, default=10.0)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0, help="seconds of CPU work for cpu_baseline")
    ap.add_argument("--ref-budget", type=float, default=150.0, help="seconds for the whole --impl reference run")
    ap.add_argument("--cache", default=os.environ.get("W2V_MODEL_CACHE", "/tmp/w2v_models"))
    ap.add_argument("--kernel", choices=["gemm", "attention", "pos_conv"], default=None,
                    help="time one kernel at a representative size instead of the whole step")
    ap.add_argument("--rows", type=int, default=32768, help="GEMM rows for --kernel gemm")
    ap.add_argument("--gemm-shape", default="3072,768,1",
                    help="N,K,epilogue for --kernel gemm (epilogue 0 fp16, 1 fp16+GELU, 2 fp32, 3 fp32+residual, "
                         "4 fp32+LayerNorm-normalised residual)")
    ap.add_argument("--block-n", type=int, default=0,
                    help="GEMM tile for --kernel gemm: 0 automatic, 64/128/256 one CTA, -128/-256 CTA pair")
    args = ap.parse_args()
    if args.kernel:
        run_kernel_case(args)
        return
    args.world = int(os.environ.get("WORLD_SIZE", args.gpus))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()

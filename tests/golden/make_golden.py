"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run here, where the reference checkout exists (it does not on GPU machines;
W2V_REFERENCE overrides its location):

    make -C oracle ref && python tests/golden/make_golden.py [--jobs N] [case ...]

Outputs (committed):
  quant_golden.npz  -- bytes of the reference converter's quantize_q8_0 /
                       quantize_q4_0 (scripts/convert_to_gguf.py:63-97) on a
                       seeded array.
  ref_<case>.npz    -- logits of the reference's own forward pass
                       (src/wav2vec2.cpp built by oracle/Makefile against the
                       oracle's ggml-API shim) in both linear modes, the
                       reference's greedy spans (src/ops.h:132-149), its
                       public-API transcript, the audio seed/length and the
                       sha256 of the synthetic GGUF the case was run on.
  ref_base_q8_0_10s_b64.npz -- the benchmark's first batch (wav2vec2-base
                       Q8_0, utterances seeded 0..63, 10 s each): per-frame
                       argmax ids of the reference's logits in both linear
                       modes, the exact-mode top-1 minus top-2 margin of every
                       frame, and the full logits of four utterances spread
                       over the batch.

Every case is computed by the reference in worker processes (spawned, one
reference thread each); the extractor output is computed once per utterance
and fed to both linear modes (w2vref_logits_from_features).
"""
from __future__ import annotations

import argparse
import hashlib
import multiprocessing as mp
import os
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))
import oracle as O  # noqa: E402

REF = Path(os.environ.get("W2V_REFERENCE", "/root/reference"))
OUT = Path(__file__).resolve().parent
MODELS = Path(os.environ.get("W2V_GOLDEN_MODELS", "/tmp/w2v_golden_models"))

# (case, arch, dtype, model kwargs, audio seconds, audio seed)
CASES = [
    ("base_q8_0_2s", "base", "q8_0", {}, 2.0, 0),
    ("base_q4_0_2s", "base", "q4_0", {}, 2.0, 1),
    ("base_f16_1s", "base", "f16", {}, 1.0, 2),
    ("base_q8_0_10s", "base", "q8_0", {}, 10.0, 0),
    ("large_q8_0_1s", "large", "q8_0", {}, 1.0, 3),
    ("tiny_f16_1s", "tiny", "f16", {"bias_std": 0.02, "gain_jitter": 0.1}, 1.0, 4),
    ("tiny_pre_q4_0_1s", "tiny_pre", "q4_0", {"bias_std": 0.02, "gain_jitter": 0.1}, 1.0, 5),
    ("tiny_q8_0_short", "tiny", "q8_0", {"bias_std": 0.02, "gain_jitter": 0.1}, 0.05, 6),
    ("tiny80_f16_1s", "tiny80", "f16", {"bias_std": 0.02, "gain_jitter": 0.1}, 1.0, 7),
    # wav2vec2-large / XLS-R-300M at its benchmark utterance length (20 s, 999 frames)
    ("large_q8_0_20s", "large", "q8_0", {}, 20.0, 8),
    # XLS-R-1B F16: two utterances of different lengths (a ragged batch in the tests)
    ("xlsr1b_f16_5s", "xlsr1b", "f16", {}, 5.0, 9),
    ("xlsr1b_f16_7s", "xlsr1b", "f16", {}, 7.3, 10),
]

BATCH_CASE = "base_q8_0_10s_b64"
BATCH_SEEDS = list(range(64))
BATCH_FULL = (0, 21, 42, 63)        # utterances whose full logits are kept


def load_synth():
    from importlib import util
    if "w2v_b200" not in sys.modules:
        spec = util.spec_from_file_location("w2v_b200", ROOT / "wav2vec2.cpp_b200" / "__init__.py",
                                            submodule_search_locations=[str(ROOT / "wav2vec2.cpp_b200")])
        mod = util.module_from_spec(spec)
        sys.modules["w2v_b200"] = mod
        spec.loader.exec_module(mod)
    import w2v_b200.synth as synth
    return synth


def quant_golden():
    sys.path.insert(0, str(REF / "scripts"))
    import convert_to_gguf as conv  # the reference converter (imports numpy only)
    rng = np.random.default_rng(1234)
    a = (rng.standard_normal(32 * 64) * 0.02).astype(np.float32)
    a[:32] = 0.0                                     # an all-zero block
    a[32:64] = np.arange(32, dtype=np.float32) / 2   # exact halves / ties
    np.savez_compressed(OUT / "quant_golden.npz", x=a,
                        q8_0=np.frombuffer(conv.quantize_q8_0(a), np.uint8),
                        q4_0=np.frombuffer(conv.quantize_q4_0(a), np.uint8))


_refs: dict = {}


def _ref(path):
    if str(path) not in _refs:
        _refs[str(path)] = O.RefOracle(path, n_threads=1)
    return _refs[str(path)]


def ref_logits_both(ref, x):
    """Reference logits of x in exact and ggml linear mode, the extractor run once."""
    f = np.ascontiguousarray(ref.features(x))
    T, V = f.shape[0], ref.cfg["vocab"]
    out = []
    for mode in (O.EXACT, O.GGML):
        lg = np.zeros((T, V), np.float32)
        with O.linear_mode(mode):
            rc = ref.lib().w2vref_logits_from_features(ref.h, O._p(f), T, ref.nt, O._p(lg))
        if rc < 0:
            raise RuntimeError("reference logits failed")
        out.append(lg)
    return out


def task_case(case, arch, dtype, kw, secs, seed):
    synth = load_synth()
    path = synth.cached_model(MODELS, arch, dtype, **kw)
    sha = hashlib.sha256(path.read_bytes()).hexdigest()
    x = synth.make_audio(int(secs * 16000), seed)
    ref = _ref(path)
    t0 = time.time()
    le, lg = ref_logits_both(ref, x)
    spans = np.array(O.greedy_spans(lg), np.int32).reshape(-1, 3)
    text = ref.transcribe(x, 1, O.GGML)
    np.savez_compressed(OUT / f"ref_{case}.npz", logits_ggml=lg, logits_exact=le,
                        spans_ggml=spans, transcript=np.array(text), arch=np.array(arch),
                        dtype=np.array(dtype), kwargs=np.array(repr(sorted(kw.items()))),
                        seconds=np.array(secs), seed=np.array(seed), gguf_sha256=np.array(sha))
    return f"{case}: T={lg.shape[0]} {time.time() - t0:.1f}s text={text[:40]!r}"


def task_batch_utt(seed):
    synth = load_synth()
    path = synth.cached_model(MODELS, "base", "q8_0")
    x = synth.make_audio(160000, seed)
    le, lg = ref_logits_both(_ref(path), x)
    return seed, le, lg


def top2_margin(lg):
    s = np.sort(lg, axis=1)
    return (s[:, -1] - s[:, -2]).astype(np.float32)


def run(fn, args):
    return fn(*args)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=max(1, (os.cpu_count() or 2) - 2))
    ap.add_argument("cases", nargs="*")
    a = ap.parse_args()
    if not O.ref_available():
        sys.exit("build the reference oracle first: make -C oracle ref")
    only = set(a.cases)
    synth = load_synth()
    quant_golden()
    tasks = []
    for c in CASES:
        if not only or c[0] in only:
            synth.cached_model(MODELS, c[1], c[2], **c[3])     # generate models before forking work
            tasks.append((task_case, c))
    if not only or BATCH_CASE in only:
        synth.cached_model(MODELS, "base", "q8_0")
        tasks += [(task_batch_utt, (s,)) for s in BATCH_SEEDS]
    # longest first
    tasks.sort(key=lambda t: -(t[1][4] * {"base": 1, "large": 7, "xlsr1b": 22}.get(t[1][1], 0.1)
                               if t[0] is task_case else 10))
    batch = {}
    with mp.get_context("spawn").Pool(a.jobs) as pool:
        for r in pool.starmap(run, tasks):
            if isinstance(r, str):
                print(r, flush=True)
            else:
                batch[r[0]] = r[1:]
    if batch:
        path = synth.cached_model(MODELS, "base", "q8_0")
        seeds = sorted(batch)
        ex = np.stack([batch[s][0] for s in seeds])
        gg = np.stack([batch[s][1] for s in seeds])
        full = np.array([s for s in BATCH_FULL if s in batch], np.int32)
        np.savez_compressed(OUT / f"ref_{BATCH_CASE}.npz", seeds=np.array(seeds, np.int32),
                            ids_exact=ex.argmax(2).astype(np.uint8), ids_ggml=gg.argmax(2).astype(np.uint8),
                            margin_exact=np.stack([top2_margin(m) for m in ex]),
                            full_seeds=full, logits_exact_full=ex[[seeds.index(s) for s in full]],
                            logits_ggml_full=gg[[seeds.index(s) for s in full]],
                            arch=np.array("base"), dtype=np.array("q8_0"), kwargs=np.array(repr([])),
                            seconds=np.array(10.0), gguf_sha256=np.array(hashlib.sha256(path.read_bytes()).hexdigest()))
        print(f"{BATCH_CASE}: {len(seeds)} utterances", flush=True)


if __name__ == "__main__":
    main()

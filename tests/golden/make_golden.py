"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Run here, where the reference checkout exists (it does not on GPU machines):

    make -C oracle ref && python tests/golden/make_golden.py

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
"""
from __future__ import annotations

import hashlib
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "oracle"))
sys.path.insert(0, str(ROOT))
import oracle as O  # noqa: E402

REF = Path("/root/reference")
OUT = Path(__file__).resolve().parent
MODELS = Path("/tmp/w2v_golden_models")

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
]


def load_synth():
    from importlib import util
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


def main(only=None):
    if not O.ref_available():
        sys.exit("build the reference oracle first: make -C oracle ref")
    synth = load_synth()
    quant_golden()
    for case, arch, dtype, kw, secs, seed in CASES:
        if only and case not in only:
            continue
        path = synth.cached_model(MODELS, arch, dtype, **kw)
        sha = hashlib.sha256(path.read_bytes()).hexdigest()
        x = synth.make_audio(int(secs * 16000), seed)
        ref = O.RefOracle(path)
        t0 = time.time()
        lg = ref.logits(x, O.GGML)
        le = ref.logits(x, O.EXACT)
        spans = np.array(O.greedy_spans(lg), np.int32).reshape(-1, 3)
        text = ref.transcribe(x, 1, O.GGML)
        np.savez_compressed(OUT / f"ref_{case}.npz", logits_ggml=lg, logits_exact=le,
                            spans_ggml=spans, transcript=np.array(text), arch=np.array(arch),
                            dtype=np.array(dtype), kwargs=np.array(repr(sorted(kw.items()))),
                            seconds=np.array(secs), seed=np.array(seed), gguf_sha256=np.array(sha))
        print(f"{case}: T={lg.shape[0]} {time.time() - t0:.1f}s text={text[:40]!r}")


if __name__ == "__main__":
    main(sys.argv[1:] or None)

"""Seeded WAV file images for the audio-ingestion parity tests.

Each case is (name, image bytes, reference-comparable).  Cases marked not
comparable have no defined reference result: the reference's reader loops
forever on a file without a "data" chunk and reads indeterminate values past
a truncated one; they are checked against this reader's documented behaviour
only."""
from __future__ import annotations

import struct
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]


def _synth():
    if "w2v_b200" not in sys.modules:
        import importlib.util
        pkg = ROOT / "wav2vec2.cpp_b200"
        spec = importlib.util.spec_from_file_location("w2v_b200", pkg / "__init__.py",
                                                      submodule_search_locations=[str(pkg)])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["w2v_b200"] = mod
        spec.loader.exec_module(mod)
    import w2v_b200.synth as s
    return s


def _tone(n, ch, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n)[:, None]
    f = rng.uniform(0.001, 0.2, size=(1, ch))
    x = 0.6 * np.sin(2 * np.pi * f * t + rng.uniform(0, 6.28, size=(1, ch))) + rng.normal(0, 0.05, (n, ch))
    return np.clip(x, -0.999, 0.999)


def cases():
    wb = _synth().wav_bytes
    out = [
        ("pcm16_mono_16k", wb(_tone(3000, 1, 1), 16000, "pcm16"), True),
        ("pcm16_stereo_44k", wb(_tone(4410, 2, 2), 44100, "pcm16"), True),
        ("pcm32_mono_8k", wb(_tone(800, 1, 3), 8000, "pcm32"), True),
        ("f32_stereo_48k_list_fmt18", wb(_tone(4800, 2, 4), 48000, "f32", fmt_size=18,
                                         chunks_before=((b"LIST", b"INFOxxxx" * 3),)), True),
        ("pcm16_3ch_22k", wb(_tone(2205, 3, 5), 22050, "pcm16"), True),
        ("f32_mono_16k", wb(_tone(1600, 1, 6), 16000, "f32"), True),
        ("pcm16_mono_11k_odd", wb(_tone(1103, 1, 7), 11025, "pcm16"), True),
        ("one_sample_44k", wb(_tone(1, 1, 8), 44100, "pcm16"), True),
        ("empty_data", wb(np.zeros((0, 1)), 16000, "pcm16"), True),
        ("short_data_decl", wb(_tone(10, 2, 9), 16000, "pcm16", data_size=3), True),
        # errors (reference messages)
        ("not_riff", b"RIFX" + wb(_tone(10, 1, 0))[4:], True),
        ("not_wave", wb(_tone(10, 1, 0))[:8] + b"WAVX" + wb(_tone(10, 1, 0))[12:], True),
        ("adpcm", _patch_fmt(wb(_tone(10, 1, 0)), code=2), True),
        ("pcm8", _patch_fmt(wb(_tone(10, 1, 0)), bits=8), True),
        ("pcm24", _patch_fmt(wb(_tone(12, 1, 0)), bits=24), True),
        ("data_before_fmt", _data_first(), True),
        # this reader's defined behaviour only
        ("no_data_chunk", wb(_tone(10, 1, 0))[:36], False),
        ("zero_channels", _patch_fmt(wb(_tone(10, 1, 0)), ch=0), False),
        ("truncated", wb(_tone(100, 2, 10), 16000, "pcm16", truncate=7), False),
    ]
    return out


def _wb(*a, **k):
    return _synth().wav_bytes(*a, **k)


def _patch_fmt(img: bytes, code=None, ch=None, bits=None) -> bytes:
    b = bytearray(img)
    if code is not None:
        b[20:22] = struct.pack("<H", code)
    if ch is not None:
        b[22:24] = struct.pack("<H", ch)
    if bits is not None:
        b[34:36] = struct.pack("<H", bits)
    return bytes(b)


def _data_first() -> bytes:
    data = np.zeros(8, "<i2").tobytes()
    body = b"WAVE" + b"data" + struct.pack("<I", len(data)) + data
    body += b"fmt " + struct.pack("<IHHIIHH", 16, 1, 1, 16000, 32000, 2, 16)
    return b"RIFF" + struct.pack("<I", len(body)) + body

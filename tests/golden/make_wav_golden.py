"""Generate tests/golden/wav_golden.npz from the REFERENCE CLI's WAV reader.

Run here, where the reference checkout exists:

    make -C oracle ref && python tests/golden/make_wav_golden.py

For every reference-comparable case of wav_cases.py the fixture stores the
WAV image and either the reference's decoded samples at 16 kHz
(examples/main/main.cpp:20-82, compiled from its source by oracle/Makefile)
or its exception message.
"""
from __future__ import annotations

import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
sys.path.insert(0, str(HERE.parents[1] / "oracle"))
import oracle as O  # noqa: E402
import wav_cases  # noqa: E402


def main():
    out = {}
    with tempfile.TemporaryDirectory() as d:
        for name, img, comparable in wav_cases.cases():
            if not comparable:
                continue
            p = Path(d) / f"{name}.wav"
            p.write_bytes(img)
            out[f"{name}__wav"] = np.frombuffer(img, np.uint8)
            try:
                out[f"{name}__out"] = O.ref_load_wav(p, 16000)
            except RuntimeError as e:
                out[f"{name}__err"] = np.array(str(e))
    np.savez_compressed(HERE / "wav_golden.npz", **out)
    print(f"{len(out)} arrays -> {HERE / 'wav_golden.npz'}")


if __name__ == "__main__":
    main()

"""Audio ingestion (wav2vec2_b200_load_wav) against the reference CLI's WAV
reader (examples/main/main.cpp:20-82): committed fixtures made by that reader,
the reader itself where the reference checkout is present, and this reader's
defined behaviour where the reference's is undefined.  Samples must be
bit-identical to the reference build's.  Host code only."""
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle as O

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
import wav_cases  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden" / "wav_golden.npz"


@pytest.fixture(scope="module")
def B(pkg):
    import w2v_b200.binding as b
    b.lib()
    return b


def _same_bits(a, b):
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    return a.shape == b.shape and np.array_equal(a.view(np.uint32), b.view(np.uint32))


def _decode(B, tmp_path, name, img, sr=16000):
    p = tmp_path / f"{name}.wav"
    p.write_bytes(bytes(img))
    return B.load_wav(p, sr)


def test_fixture_matches_case_generator():
    z = np.load(GOLDEN)
    for name, img, comparable in wav_cases.cases():
        if comparable:
            assert bytes(z[f"{name}__wav"]) == img, name


@pytest.mark.parametrize("name", [c[0] for c in wav_cases.cases() if c[2]])
def test_against_reference_fixture(B, tmp_path, name):
    z = np.load(GOLDEN)
    img = z[f"{name}__wav"]
    if f"{name}__err" in z.files:
        with pytest.raises(B.EngineError, match=str(z[f"{name}__err"])):
            _decode(B, tmp_path, name, img)
        return
    ref = z[f"{name}__out"]
    got = _decode(B, tmp_path, name, img)
    assert _same_bits(got, ref), name


@pytest.mark.skipif(not O.ref_available(), reason="reference build (oracle/_ref) not present")
@pytest.mark.parametrize("sr", [16000, 8000, 22050])
def test_against_live_reference(B, tmp_path, sr):
    for name, img, comparable in wav_cases.cases():
        if not comparable:
            continue
        p = tmp_path / f"{name}.wav"
        p.write_bytes(img)
        try:
            ref = O.ref_load_wav(p, sr)
        except RuntimeError as e:
            with pytest.raises(B.EngineError, match=str(e)):
                B.load_wav(p, sr)
            continue
        got = B.load_wav(p, sr)
        assert _same_bits(got, ref), (name, sr)


def test_missing_file(B, tmp_path):
    p = tmp_path / "nope.wav"
    with pytest.raises(B.EngineError, match=f"Cannot open WAV: {p}"):
        B.load_wav(p)


def test_defined_where_reference_is_not(B, tmp_path):
    cases = {c[0]: c[1] for c in wav_cases.cases()}
    for name in ("no_data_chunk", "zero_channels"):
        with pytest.raises(B.EngineError, match="Malformed WAV"):
            _decode(B, tmp_path, name, cases[name])
    # a data chunk cut short yields the complete sample frames present
    t = _decode(B, tmp_path, "truncated", cases["truncated"])
    full = _decode(B, tmp_path, "full", cases["truncated"] + b"\0" * 7)
    frames = (len(cases["truncated"]) - 44) // 4
    assert t.shape == (frames,) and np.array_equal(t, full[:frames])


def test_load_wav_status_code(B, tmp_path):
    import ctypes as C
    p = C.c_void_p()
    n = C.c_int()
    bad = tmp_path / "bad.wav"
    bad.write_bytes(b"RIFF\0\0\0\0WAVE")
    assert B.lib().wav2vec2_b200_load_wav(str(bad).encode(), 16000, C.byref(p), C.byref(n)) == 5
    assert p.value is None and n.value == 0
    assert B.lib().wav2vec2_b200_load_wav(str(bad).encode(), 16000, None, C.byref(n)) == 1

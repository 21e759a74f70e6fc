"""Synthetic GGUF generator: byte-exact quantisers against the reference
converter's output (golden), a GGUF that the reference-format reader parses,
and seeded determinism."""
import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN


def test_quantizers_byte_exact_vs_reference_golden(synth):
    z = np.load(GOLDEN / "quant_golden.npz")
    assert synth.quantize_q8_0(z["x"]) == z["q8_0"].tobytes()
    assert synth.quantize_q4_0(z["x"]) == z["q4_0"].tobytes()


def test_dequantize_roundtrip(synth):
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((8, 64)) * 0.02).astype(np.float32)
    for gt, enc, tol in ((synth.GGUF_Q8_0, synth.quantize_q8_0, 1 / 127), (synth.GGUF_Q4_0, synth.quantize_q4_0, 1 / 7)):
        d = synth.dequantize(enc(a), gt, a.shape)
        amax = np.abs(a.reshape(-1, 32)).max(1).repeat(32).reshape(a.shape)
        # half a step plus the fp16 rounding of the scale (|q| <= 127 ulps of 2^-11)
        assert np.all(np.abs(d - a) <= amax * tol * 0.6 + 1e-6)


def test_audio_seeded_and_normalised(synth):
    a = synth.make_audio(16000, 5)
    b = synth.make_audio(16000, 5)
    assert a.dtype == np.float32 and np.array_equal(a, b)
    assert abs(np.abs(a).max() - 0.9) < 1e-6
    assert not np.array_equal(a, synth.make_audio(16000, 6))


def test_gguf_parses_with_expected_hparams(synth, tmp_path):
    p = tmp_path / "m.gguf"
    synth.write_model(p, "tiny_pre", "q4_0", seed=1)
    o = O.Oracle(p)
    a = synth.ARCHS["tiny_pre"]
    assert o.cfg == {"conv_dim": a.conv_dim, "hidden": a.hidden, "n_layers": a.n_layers,
                     "n_heads": a.n_heads, "ffn": a.ffn, "vocab": a.vocab, "pad_id": 0,
                     "stable": 1, "n_conv": 7, "group_norm": 0}
    w = o.weight("encoder.layers.1.feed_forward.intermediate_dense")
    t = synth.model_tensors(a, 1)["encoder.layers.1.feed_forward.intermediate_dense.weight"]
    assert w.shape == t.shape
    assert np.allclose(w, synth.dequantize(synth.quantize_q4_0(t), synth.GGUF_Q4_0, t.shape))


def test_gguf_deterministic(synth, tmp_path):
    h1 = synth.write_model(tmp_path / "a.gguf", "tiny", "q8_0", seed=2)
    h2 = synth.write_model(tmp_path / "b.gguf", "tiny", "q8_0", seed=2)
    assert h1 == h2


@pytest.mark.parametrize("corrupt", ["magic", "truncated", "missing_key"])
def test_oracle_loader_rejects_bad_files(synth, tmp_path, corrupt):
    data = bytearray(synth.gguf_bytes(synth.ARCHS["tiny"], synth.model_tensors(synth.ARCHS["tiny"], 0), "q8_0"))
    if corrupt == "magic":
        data[0] ^= 0xFF
    elif corrupt == "truncated":
        data = data[: len(data) // 2]
    else:
        key = b"wav2vec2.hidden_size"
        i = data.find(key)
        data[i:i + len(key)] = b"wav2vec2.hidden_sizX"
    p = tmp_path / "bad.gguf"
    p.write_bytes(bytes(data))
    with pytest.raises(RuntimeError):
        O.Oracle(p)

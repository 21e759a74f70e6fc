"""The CPU oracle, pinned against the reference's own known-answer tests
(tests/test_ops.cpp in the reference) and against golden outputs of the
reference's own forward pass (tests/golden/make_golden.py)."""
import ast
import hashlib

import numpy as np
import pytest

import oracle as O
from conftest import load_golden

GOLDEN_CASES = ["base_q8_0_2s", "base_q4_0_2s", "base_f16_1s", "large_q8_0_1s",
                "tiny_f16_1s", "tiny_pre_q4_0_1s", "tiny_q8_0_short"]


# ── known answers of reference tests/test_ops.cpp ────────────────────────────

def test_gelu_known_values():            # test_ops.cpp:8-17
    assert abs(O.gelu(0.0)) < 1e-6
    assert abs(O.gelu(10.0) - 10.0) < 1e-3
    assert -1.0 < O.gelu(-1.0) < 0.0
    assert abs(O.gelu(1.0) - 0.8413) < 1e-3


def test_softmax():                      # test_ops.cpp:20-41
    x = O.softmax([1.0, 2.0, 3.0])
    assert abs(x.sum() - 1) < 1e-6 and (x > 0).all() and x[2] > x[1] > x[0]
    y = O.softmax([2.0] * 4)
    assert np.allclose(y, 0.25, atol=1e-6)
    z = O.softmax([1000.0, 1001.0, 999.0])
    assert abs(z.sum() - 1) < 1e-5 and z[1] > z[0] > z[2]


def test_layer_norm():                   # test_ops.cpp:44-72
    x = O.layer_norm([[1, 2, 3, 4]], np.ones(4), np.zeros(4))
    assert abs(x.mean()) < 1e-5 and abs(np.sqrt((x ** 2).mean()) - 1) < 1e-3
    x2 = O.layer_norm([[0, 0, 0, 0]], np.full(4, 2.0), np.full(4, 5.0))
    assert np.allclose(x2, 5.0, atol=1e-3)
    x3 = O.layer_norm([[10, 20, 10, 20], [1, 1, 1, 1]], np.ones(4), np.zeros(4))
    assert abs(x3[0].mean()) < 1e-5


def test_group_norm():                   # test_ops.cpp:75-89
    x = O.group_norm([[1, 4], [2, 4], [3, 4]], np.ones(2), np.zeros(2))
    assert abs(x[:, 0].mean()) < 1e-5
    assert np.abs(x[:, 1]).max() < 1e-2


def test_conv1d():                       # test_ops.cpp:106-141
    x = np.arange(1, 6, dtype=np.float32)[:, None]
    assert np.allclose(O.conv1d(x, np.ones((1, 1, 1)), np.zeros(1))[:, 0], x[:, 0])
    x2 = np.arange(1, 5, dtype=np.float32)[:, None]
    assert np.allclose(O.conv1d(x2, np.ones((1, 1, 2)), np.zeros(1))[:, 0], [3, 5, 7])
    assert np.allclose(O.conv1d(x2, np.ones((1, 1, 2)), np.zeros(1), stride=2)[:, 0], [3, 7])
    x3 = np.arange(1, 4, dtype=np.float32)[:, None]
    assert np.allclose(O.conv1d(x3, np.ones((1, 1, 3)), np.zeros(1), pad=1)[:, 0], [3, 6, 5])


def test_conv1d_grouped_matches_numpy():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((37, 8)).astype(np.float32)
    w = rng.standard_normal((8, 2, 5)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    y = O.conv1d(x, w, b, stride=1, pad=2, groups=4)
    xp = np.pad(x, ((2, 2), (0, 0)))
    ref = np.zeros_like(y)
    for t in range(y.shape[0]):
        for co in range(8):
            g = co // 2
            ref[t, co] = b[co] + np.sum(xp[t:t + 5, 2 * g:2 * g + 2].T * w[co])
    assert np.allclose(y, ref, atol=1e-4)


def test_feature_extractor_output_length(synth):   # test_ops.cpp:144-154
    assert 45 <= synth.n_frames(16000) <= 55
    assert synth.n_frames(160000) == 499 and synth.n_frames(320000) == 999


def test_ctc_greedy_spans():             # test_ops.cpp:157-183
    lg = np.zeros((6, 4), np.float32)
    for t, v in enumerate([0, 1, 1, 0, 2, 0]):
        lg[t, v] = 10
    spans = O.greedy_spans(lg)
    assert [s[0] for s in spans] == [0, 1, 0, 2, 0]
    assert spans[1] == (1, 1, 3) and spans[-1] == (0, 5, 6)
    assert O.collapse(spans) == [1, 2]
    lg2 = np.array([[0, 10]] * 3, np.float32)
    assert [s[0] for s in O.greedy_spans(lg2)] == [1]


def test_ctc_greedy_ties_first_max_wins():          # strict '>' at ops.h:141
    lg = np.array([[1, 1, 0], [0, 2, 2]], np.float32)
    assert [s[0] for s in O.greedy_spans(lg)] == [0, 1]


def test_ctc_greedy_empty():
    assert O.greedy_spans(np.zeros((0, 5), np.float32)) == []


# ── oracle vs golden outputs of the reference forward pass ───────────────────

def _case_model(model_path, g):
    kw = dict(ast.literal_eval(g["kwargs"]))
    p = model_path(g["arch"], g["dtype"], **kw)
    sha = hashlib.sha256(p.read_bytes()).hexdigest()
    assert sha == g["gguf_sha256"], "synthetic GGUF generator drifted from the golden fixture"
    return p


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_matches_reference_golden_exact_mode(case, model_path, synth):
    g = load_golden(case)
    o = O.Oracle(_case_model(model_path, g))
    x = synth.make_audio(int(g["seconds"] * 16000), int(g["seed"]))
    lg = o.logits(x, O.EXACT)
    ref = g["logits_exact"]
    assert lg.shape == ref.shape
    # fp32 restatement vs fp32 reference: summation order only
    assert np.abs(lg - ref).max() < 5e-4, np.abs(lg - ref).max()


@pytest.mark.parametrize("case", ["tiny_f16_1s", "tiny_pre_q4_0_1s", "tiny_q8_0_short"])
def test_oracle_matches_reference_golden_ggml_mode(case, model_path, synth):
    g = load_golden(case)
    o = O.Oracle(_case_model(model_path, g))
    x = synth.make_audio(int(g["seconds"] * 16000), int(g["seed"]))
    lg = o.logits(x, O.GGML)
    # ggml mode re-quantizes every linear's activations to Q8_0; fp32-level
    # differences upstream (LN summation order) flip a few rounding decisions,
    # so agreement is bounded by the quantization step, not by fp32 rounding
    assert np.abs(lg - g["logits_ggml"]).max() < 2e-2


def test_reference_greedy_spans_match_oracle_decoder():
    for case in GOLDEN_CASES:
        g = load_golden(case)
        spans = np.array(O.greedy_spans(g["logits_ggml"]), np.int32).reshape(-1, 3)
        assert np.array_equal(spans, g["spans_ggml"])


@pytest.mark.skipif(not O.ref_available(), reason="reference oracle not built here")
def test_oracle_vs_reference_live_stagewise(model_path, synth):
    p = model_path("tiny_pre", "q4_0", bias_std=0.02, gain_jitter=0.1)
    o, r = O.Oracle(p), O.RefOracle(p, 4)
    x = synth.make_audio(12000, 11)
    fo, fr = o.features(x), r.features(x)
    assert np.abs(fo - fr).max() <= 1e-5 * max(1.0, np.abs(fr).max())
    so, sr = o.encode_stages(fr, O.EXACT), r.encode_stages(fr, O.EXACT)
    for a, b in zip(so, sr):
        assert np.abs(a - b).max() < 1e-4

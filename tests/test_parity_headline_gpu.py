"""Parity at the benchmark's own configuration: wav2vec2-base Q8_0, one batch
of 64 utterances x 10 s (M = 31936 encoder rows: the GEMM tiles the
benchmark times), through the batch API wav2vec2_b200_logits, against golden
outputs of the reference's own forward pass
(tests/golden/ref_base_q8_0_10s_b64.npz, made by make_golden.py from
oracle/_ref).

Checked:
  * batch rows equal single-utterance runs bit for bit (4 utterances spread
    over the batch; a single 499-row utterance runs other GEMM tiles);
  * logits within 2e-2 of the reference with exact fp32 linears
    (src/ggml_backend.h:78-120 through the oracle's exact mode);
  * the margin rule: every frame whose reference top-1/top-2 margin exceeds
    twice the measured logit error has the reference's argmax
    (src/ops.h:132-149, first max wins) -- on all 64 utterances;
  * greedy-sequence identity rates against both reference linear modes,
    asserted in the form random-init weights allow: at least as often as the
    reference's own two linear modes agree with each other."""
import ast
import hashlib

import numpy as np
import pytest

from conftest import load_golden

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

CASE = "base_q8_0_10s_b64"


def collapse(ids, blank=0):
    """Greedy CTC token sequence of per-frame ids: runs collapsed, blank dropped
    (src/ops.h:132-149, src/wav2vec2.cpp:500-502)."""
    ids = np.asarray(ids)
    if ids.size == 0:
        return ids
    keep = np.ones(ids.size, bool)
    keep[1:] = ids[1:] != ids[:-1]
    r = ids[keep]
    return r[r != blank]


@pytest.fixture(scope="module")
def run(pkg, model_path, synth):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import w2v_b200.binding as b
    g = load_golden(CASE)
    p = model_path(g["arch"], g["dtype"], **dict(ast.literal_eval(g["kwargs"])))
    assert hashlib.sha256(p.read_bytes()).hexdigest() == g["gguf_sha256"]
    m = b.Model(p)
    xs = [synth.make_audio(int(g["seconds"] * 16000), int(s)) for s in g["seeds"]]
    got = m.logits(xs)                       # one device batch of 64 (max_batch 64)
    yield m, g, xs, got
    m.close()


def test_batch_of_64_equals_single_utterances_bitwise(run):
    m, g, xs, got = run
    assert len(got) == 64 and all(x.shape == (499, 32) for x in got)
    for s in g["full_seeds"]:
        i = list(g["seeds"]).index(int(s))
        single = m.logits([xs[i]])[0]
        assert np.array_equal(got[i], single), (int(s), np.abs(got[i] - single).max())


def test_batch_of_64_logits_vs_reference_exact(run):
    m, g, xs, got = run
    seeds = list(g["seeds"])
    for k, s in enumerate(g["full_seeds"]):
        lg = got[seeds.index(int(s))]
        err = np.abs(lg - g["logits_exact_full"][k]).max()
        assert err < 2e-2, (int(s), err)
        # against the ggml-emulated path the reference's own ggml-vs-exact gap bounds any
        # implementation without bit-identical activation re-quantisation
        floor = np.abs(g["logits_ggml_full"][k] - g["logits_exact_full"][k]).max()
        assert np.abs(lg - g["logits_ggml_full"][k]).max() < max(2 * floor, 2e-2)


def test_margin_rule_on_all_64_utterances(run):
    m, g, xs, got = run
    seeds = list(g["seeds"])
    err = max(np.abs(got[seeds.index(int(s))] - g["logits_exact_full"][k]).max()
              for k, s in enumerate(g["full_seeds"]))
    ids = np.stack([x.argmax(1) for x in got])
    safe = g["margin_exact"] > 2 * err
    print(f"max logit error {err:.2e}; frames covered by the margin rule {safe.mean():.4f}")
    assert safe.mean() > 0.9
    bad = np.argwhere(safe & (ids != g["ids_exact"]))
    assert bad.size == 0, f"{len(bad)} frames flipped despite margin > 2 x {err:.2e}: {bad[:5].tolist()}"
    assert (ids == g["ids_exact"]).mean() > 0.99


def test_greedy_sequence_identity_rates(run):
    m, g, xs, got = run
    ids = [x.argmax(1) for x in got]
    same_exact = np.mean([np.array_equal(collapse(a), collapse(b)) for a, b in zip(ids, g["ids_exact"])])
    same_ggml = np.mean([np.array_equal(collapse(a), collapse(b)) for a, b in zip(ids, g["ids_ggml"])])
    ref_self = np.mean([np.array_equal(collapse(a), collapse(b)) for a, b in zip(g["ids_exact"], g["ids_ggml"])])
    print(f"greedy sequences identical: vs exact {same_exact:.3f}, vs ggml {same_ggml:.3f}; "
          f"reference exact vs its own ggml mode {ref_self:.3f}")
    assert same_exact >= ref_self

"""Host prefix beam search (wav2vec2_b200_ctc_beam_search, a prefix trie)
against the reference's own decoder (wv2_ctc_beam_search, src/ops.h:151-251,
compiled from its source into oracle/_ref) on the CPU: the reference's
known-answer cases (tests/test_ops.cpp:186-226), then seeded random logits
over vocabulary sizes, lengths, beam widths and logit scales."""
import numpy as np
import pytest

import oracle as O


@pytest.fixture(scope="module")
def B(pkg):
    import w2v_b200.binding as b
    b.lib()
    return b


def kat(rows, V):
    return np.array(rows, np.float32).reshape(-1, V)


def test_reference_known_answers(B):
    # blank, 1, 1, blank, 2, blank -> [1, 2]
    lg = kat([10, 0, 0, 0, 0, 10, 0, 0, 0, 10, 0, 0, 10, 0, 0, 0, 0, 0, 10, 0, 10, 0, 0, 0], 4)
    assert B.ctc_beam_search(lg, 0, 5) == [1, 2]
    # 1, blank, 1 -> [1, 1]
    assert B.ctc_beam_search(kat([0, 10, 0, 10, 0, 0, 0, 10, 0], 3), 0, 5) == [1, 1]
    # all blanks -> []
    assert B.ctc_beam_search(kat([10, 0] * 4, 2), 0, 5) == []
    # one token repeated without blanks -> [1]
    assert B.ctc_beam_search(kat([0, 10] * 3, 2), 0, 5) == [1]


def test_edge_cases(B):
    assert B.ctc_beam_search(np.zeros((0, 5), np.float32), 0, 3) == []
    lg = np.array([[0.0, 5.0, 0.0]], np.float32)
    assert B.ctc_beam_search(lg, 0, 1) == [1]
    assert B.ctc_beam_search(lg, 2, 4) == [1]                      # blank need not be id 0
    with pytest.raises(B.EngineError):
        B.ctc_beam_search(lg, 3, 4)                                 # blank out of range
    with pytest.raises(B.EngineError):
        B.ctc_beam_search(lg, 0, 0)                                 # no beam


@pytest.mark.skipif(not O.ref_available(), reason="reference oracle build absent")
def test_reference_known_answers_agree(B):
    for rows, V in (([10, 0, 0, 0, 0, 10, 0, 0, 0, 10, 0, 0, 10, 0, 0, 0, 0, 0, 10, 0, 10, 0, 0, 0], 4),
                    ([0, 10, 0, 10, 0, 0, 0, 10, 0], 3), ([10, 0] * 4, 2), ([0, 10] * 3, 2)):
        lg = kat(rows, V)
        assert B.ctc_beam_search(lg, 0, 5) == O.ref_beam_search(lg, 0, 5)


@pytest.mark.skipif(not O.ref_available(), reason="reference oracle build absent")
def test_matches_reference_decoder_on_random_logits(B):
    rng = np.random.default_rng(2024)
    n = 0
    for V in (2, 3, 5, 32, 64):
        for T in (1, 2, 7, 60, 400):
            for W in (1, 2, 5, 16):
                for scale in (0.5, 3.0, 12.0):
                    lg = (rng.standard_normal((T, V)) * scale).astype(np.float32)
                    blank = int(rng.integers(0, V)) if V > 2 else 0
                    got = B.ctc_beam_search(lg, blank, W)
                    ref = O.ref_beam_search(lg, blank, W)
                    assert got == ref, (V, T, W, scale, blank)
                    n += 1
    assert n == 300


@pytest.mark.skipif(not O.ref_available(), reason="reference oracle build absent")
def test_matches_reference_on_ctc_shaped_logits(B):
    """Logits shaped like a CTC head's: mostly blank, with bursts of a token."""
    rng = np.random.default_rng(7)
    for case in range(40):
        T, V = int(rng.integers(50, 800)), 32
        lg = rng.standard_normal((T, V)).astype(np.float32)
        lg[:, 0] += 4.0
        for t0 in rng.integers(0, T, T // 6):
            lg[t0: t0 + int(rng.integers(1, 4)), int(rng.integers(1, V))] += 8.0
        for W in (3, 5, 10):
            assert B.ctc_beam_search(lg, 0, W) == O.ref_beam_search(lg, 0, W), (case, W)


def test_exact_ties_take_the_smaller_sequence(B):
    """Equal logits make every candidate of a frame tie: the explicit rule keeps
    the lexicographically smaller prefixes and returns the smaller sequence."""
    lg = np.zeros((1, 4), np.float32)
    # one frame: prefixes [], [1], [2], [3] all have log-probability -log 4
    assert B.ctc_beam_search(lg, 0, 4) == []
    lg = np.array([[0.0, 3.0, 3.0]], np.float32)
    assert B.ctc_beam_search(lg, 0, 3) == [1]

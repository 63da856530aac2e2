"""Pins the CTC oracle: the reference's own ctc_decode.cpp (compiled in
place) and this repository's restatement both reproduce the reference's
known-answer tests (tests/recognition/test_ctc_decode.cpp:14-88)."""
import json

import numpy as np
import pytest

from conftest import ROOT
from oracle import ctc_oracle as co

KAT = json.loads((ROOT / "tests/golden/ctc_kat.json").read_text())


def expected_score(terms):
    if not terms:
        return 0.0
    s = np.float32(0)
    for t in terms:
        s = np.float32(s + np.float32(t))
    return float(np.float32(s / np.float32(len(terms))))


@pytest.mark.parametrize("case", KAT["decode"], ids=lambda c: c["name"])
def test_restatement_matches_kat(case):
    toks, score = co.collapse(case["indices"], case["scores"], KAT["num_labels"])
    assert toks == case["tokens"]
    assert score == pytest.approx(expected_score(case["score_terms"]), abs=1e-7)


@pytest.mark.parametrize("case", KAT["decode"], ids=lambda c: c["name"])
def test_reference_build_matches_kat(case):
    toks, score = co.ref_decode(case["indices"], case["scores"], KAT["num_labels"])
    assert toks == case["tokens"]
    assert score == pytest.approx(expected_score(case["score_terms"]), abs=1e-7)


@pytest.mark.parametrize("simd", [False, True])
@pytest.mark.parametrize("case", KAT["decode_raw"], ids=lambda c: c["name"])
def test_reference_raw_matches_kat(case, simd):
    x = np.array(case["logits"], dtype=np.float32).reshape(case["seq_len"], case["num_classes"])
    toks, score = co.ref_decode_raw(x, KAT["num_labels"], simd=simd)
    assert toks == case["tokens"]
    assert score == pytest.approx(expected_score(case["score_terms"]), abs=1e-7)


@pytest.mark.parametrize("simd", [False, True])
def test_restatement_agrees_with_reference_on_random_lines(simd):
    rng = np.random.default_rng(7)
    for _ in range(40):
        T, V = int(rng.integers(1, 60)), int(rng.integers(2, 300))
        logits = (rng.standard_normal((T, V)) * 4).astype(np.float16)
        # plant ties and blanks
        logits[:, 0] += np.float16(rng.integers(0, 2) * 3)
        probs = co.softmax_probs(logits)
        nl = int(rng.integers(1, V + 1))
        ref = co.ref_decode_raw(probs, nl, simd=simd)
        idx = probs.argmax(axis=1)  # numpy: first occurrence on ties
        own = co.collapse(idx, probs[np.arange(T), idx], nl)
        assert ref[0] == own[0]
        assert ref[1] == pytest.approx(own[1], abs=1e-7)

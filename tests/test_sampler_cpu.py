"""Token samplers of generation (GreedySampler / NucleusSampler / make_sampler, attnrank/src/
model.cpp:70-127) against golden token ids produced by the reference's own samplers
(tests/golden/make_sampler_fixtures.py). Host code only: no GPU.

Bit-exact: every case for the library's sampler (the same std::partial_sort order and
std::mt19937_64 draws), the tie-free cases for the oracle's restatement (oracle/sampler.py).
"""
from __future__ import annotations

import base64
import json
from pathlib import Path

import numpy as np
import pytest

CASES = json.loads((Path(__file__).resolve().parent / "golden" / "sampler_fixtures.json").read_text())["cases"]


def logits_of(case) -> np.ndarray:
    raw = base64.b64decode(case["logits_f32_b64"])
    return np.frombuffer(raw, dtype=np.float32).reshape(case["rows"], case["vocab"])


@pytest.mark.parametrize("case", CASES, ids=[c["name"] for c in CASES])
def test_library_sampler_matches_reference(case):
    import attnrank as ar
    sampler = ar.make_sampler(case["temperature"], case["top_p"], case["top_k"], case["seed"])
    assert sampler.greedy == (case["temperature"] <= 0.0)
    assert [sampler.select(row) for row in logits_of(case)] == case["tokens"]


TIE_FREE = [c for c in CASES if not c["ties"]]


@pytest.mark.parametrize("case", TIE_FREE, ids=[c["name"] for c in TIE_FREE])
def test_oracle_sampler_matches_reference(case):
    from oracle import sampler as S
    sampler = S.make_sampler(case["temperature"], case["top_p"], case["top_k"], case["seed"])
    assert [sampler.select(row) for row in logits_of(case)] == case["tokens"]


def test_mt19937_64_check_value():
    """The C++ standard's check value: output 10000 of mt19937_64 seeded with 5489."""
    from oracle import sampler as S
    generator = S.MT19937_64(5489)
    for _ in range(9999):
        generator.next()
    assert generator.next() == 9981545732273789042


def test_greedy_takes_the_first_maximum():
    import attnrank as ar
    logits = np.array([0.5, 2.0, -1.0, 2.0, 2.0], dtype=np.float32)
    assert ar.make_sampler(0.0).select(logits) == 1
    assert ar.make_sampler(-0.5).select(logits) == 1


def test_nucleus_draws_advance_and_depend_on_the_seed():
    import attnrank as ar
    logits = np.linspace(-1.0, 1.0, 64, dtype=np.float32)
    first = ar.make_sampler(1.0, 1.0, 0, 42)
    draws = [first.select(logits) for _ in range(32)]
    assert len(set(draws)) > 1
    again = ar.make_sampler(1.0, 1.0, 0, 42)
    assert [again.select(logits) for _ in range(32)] == draws
    other = ar.make_sampler(1.0, 1.0, 0, 43)
    assert [other.select(logits) for _ in range(32)] != draws


def test_sampler_errors():
    import attnrank as ar
    empty = np.zeros(0, dtype=np.float32)
    with pytest.raises(ar.AttnRankError, match="empty logits"):
        ar.make_sampler(0.7).select(empty)
    with pytest.raises(ar.AttnRankError, match="empty logits"):
        ar.make_sampler(0.0).select(empty)


def test_generate_needs_decode_for_stop_strings():
    """Host-side argument check of Engine.generate (no engine is created)."""
    import attnrank as ar
    from attnrank.core import _apply_stop_sequence
    assert _apply_stop_sequence("abc</s>def</s>", ["</s>"]) == (True, "abc")
    assert _apply_stop_sequence("abc", ["x", ""]) == (False, "abc")
    # the first stop in list order wins, wherever it occurs
    assert _apply_stop_sequence("one two three", ["three", "two"]) == (True, "one two ")
    settings = ar.GenerationSettings()
    assert (settings.max_new_tokens, settings.temperature, settings.top_p, settings.top_k, settings.seed) == \
        (128, 0.0, 0.9, 0, 1234)


@pytest.mark.parametrize("temperature,top_p,top_k,quantum", [(0.7, 0.9, 0, 0.0), (1.0, 0.95, 0, 0.25),
                                                              (0.5, 0.9, 50, 0.0), (1.3, 0.5, 0, 1.0)])
def test_library_sampler_matches_reference_at_full_vocabulary(reference_lib, temperature, top_p, top_k, quantum):
    """152064-wide logits (the Qwen vocabulary) against the reference's own sampler: the library's
    radix-sorted fast path must give the same ids, with and without tied logits."""
    if reference_lib is None:
        pytest.skip("oracle/_ref is not built")
    import attnrank as ar
    from oracle import reference
    rng = np.random.default_rng(int(temperature * 100) + top_k)
    rows = rng.normal(0.0, 2.0, size=(6, 152064))
    if quantum > 0.0:
        rows = np.round(rows / quantum) * quantum
    rows = rows.astype(np.float32)
    want = reference.sample(rows, temperature, top_p, top_k, 2024)
    sampler = ar.make_sampler(temperature, top_p, top_k, 2024)
    assert [sampler.select(row) for row in rows] == want

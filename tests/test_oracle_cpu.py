"""The CPU oracle itself: pinned to the reference before it is trusted as a checker.

  * the synthetic checkpoint generator: deterministic, the documented distribution;
  * the vectorised mass reduction against a literal loop transcription of the reference's
    reduce_document_attention_kernel (kernels.cu:202-236) on a small case;
  * the full forward against fixtures produced by the reference's own CUDA build on a B200
    (tests/golden/reference_small.json, made by tests/golden/make_reference_fixtures.py);
  * BASELINE config 1 (TinyLlama-shaped single layer, fp32, CPU only) end to end.
"""
from __future__ import annotations

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import forward as F
from oracle import weights as W

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_synthetic_weights_are_deterministic_and_distributed_as_documented():
    a = W.bf16_bits(1 << 16, 0, 3, W.QUERY)
    b = W.bf16_bits(1 << 16, 0, 3, W.QUERY)
    c = W.bf16_bits(1 << 16, 1, 3, W.QUERY)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    values = W.bf16_to_f32(W.bf16_bits(1 << 20, 0, -1, W.EMBEDDING, 0.02))
    assert abs(values.mean()) < 1e-4
    assert abs(values.std() - 0.02) < 2e-4
    assert np.abs(values).max() <= 0.02 * math.sqrt(3.0) * 2 + 1e-3  # Irwin-Hall(4) support
    # random access: a slice equals the same elements of the whole tensor
    whole = W.bf16_bits(5000, 7, 2, W.DOWN)
    assert np.array_equal(W.bf16_bits(100, 7, 2, W.DOWN, first=1234), whole[1234:1334])
    ones = W.f32(64, 0, 0, W.INPUT_NORM, 0.0, 1.0)
    assert np.all(ones == 1.0)


def _loop_reduction(probs, heads, T, qb, qe, spans, chunk, normalize):
    """Literal transcription of reduce_document_attention_kernel + the per-chunk call site:
    every chunk holds queries [c0, c1) and keys [0, c1); spans clip at key_count = c1."""
    total = [0.0] * len(spans)
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        for s, (b, e) in enumerate(spans):
            end = min(e, c1)
            for h in range(heads):
                for q in range(c0, c1):
                    if q < qb or q >= min(qe, T):
                        continue
                    value = sum(float(probs[h, q, k]) for k in range(b, end))
                    if normalize and end > b:
                        value /= end - b
                    total[s] += value
    return np.array(total)


@pytest.mark.parametrize("normalize", [False, True])
@pytest.mark.parametrize("query", [(13, 21), (-4, 21), (5, 40), (21, 13), (13, 13)])
def test_document_mass_matches_literal_reference_loop(normalize, query):
    """Ordinary and degenerate spans the reference accepts without an error: a query span that
    starts before token 0 or ends past the prompt, an empty or reversed query span, and empty or
    reversed document spans (their key loops run zero times)."""
    rng = np.random.default_rng(5)
    heads, T, chunk = 3, 23, 8
    scores = torch.from_numpy(rng.standard_normal((heads, T, T)).astype(np.float32))
    mask = torch.arange(T)[None, :] <= torch.arange(T)[:, None]
    probs = torch.softmax(scores.masked_fill(~mask[None], float("-inf")), dim=-1)
    spans = [(0, 5), (5, 11), (11, 16), (3, 9), (14, 40), (9, 3), (7, 7)]
    prompt = F.Prompt(tokens=np.zeros(T, np.int32), query_span=query, spans=spans)
    got = F.document_mass(probs, prompt, chunk, normalize)
    want = _loop_reduction(probs.numpy(), heads, T, query[0], query[1], spans, chunk, normalize)
    np.testing.assert_allclose(got, want, rtol=1e-12)
    assert got[5] == 0.0 and got[6] == 0.0


def _fixture(name):
    path = GOLDEN / name
    if not path.exists():
        pytest.skip(f"{name} not generated yet (tests/golden/make_reference_fixtures.py on a B200)")
    return json.loads(path.read_text())


def _shape(config):
    return F.Shape(hidden=config["hidden_size"], intermediate=config["intermediate_size"],
                   layers=config["num_hidden_layers"], heads=config["num_attention_heads"],
                   kv_heads=config["num_key_value_heads"], vocab=config["vocab_size"], eps=config["rms_norm_eps"],
                   theta=config["rope_theta"], window=config["sliding_window"], bias=config["attention_bias"])


def _prompt(entry):
    return F.Prompt(tokens=np.asarray(entry["tokens"], np.int32), query_span=tuple(entry["query_span"]),
                    spans=[tuple(s) for s in entry["spans"]])


@pytest.mark.parametrize("gemm_inputs,rel", [("fp16", 2e-4), (None, 1e-3)])
def test_oracle_matches_reference_cuda_build_small_model(gemm_inputs, rel):
    """fp16-emulating oracle ~ the reference's own numerics; the pure fp32 oracle within the mass tolerance."""
    data = _fixture("reference_small.json")
    model = F.OracleModel(_shape(data["config"]), seed=data["seed"], std=data["std"], gemm_inputs=gemm_inputs,
                          chunk=data["prefill_chunk_tokens"])
    prompts = [_prompt(p) for p in data["prompts"]]
    worst = 0.0
    for case in data["cases"]:
        prompt = prompts[case["prompt"]]
        if "measure_attention" in case:
            begin, end = case["measure_attention"]
            got = model.measure_attention(prompt, begin, end)
            want = np.asarray(case["attention"])
        else:
            rows, _ = model.probe([prompt], case["layer_begin"], case["layer_end"], case["normalize_by_length"])
            got, want = rows[0], np.asarray(case["rows"])
        worst = max(worst, float(np.max(np.abs(got - want) / np.maximum(np.abs(want), 1e-12))))
    assert worst <= rel, f"oracle vs reference build: max relative error {worst:.3e}"


def test_config1_tinyllama_single_layer_runs_on_cpu():
    """TinyLlama-1.1B-shaped single layer, fp32 weights, 256 ids from seed 0,
    16 query tokens over 5 document spans of 48 tokens."""
    shape = F.Shape(hidden=2048, intermediate=5632, layers=1, heads=32, kv_heads=4, vocab=32000, eps=1e-5,
                    theta=10000.0)
    rng = np.random.default_rng(0)
    tokens = rng.integers(0, 32000, size=256).astype(np.int32)
    prompt = F.Prompt(tokens=tokens, query_span=(240, 256), spans=[(48 * i, 48 * i + 48) for i in range(5)])
    rows, raw = F.OracleModel(shape, seed=0).probe([prompt])
    assert rows[0].shape == (1, 5)
    assert rows[0].sum() == pytest.approx(1.0, rel=1e-12)
    # every query row's softmax mass over the five spans (tokens 0..239) is below 1 and above 0
    assert 0.0 < raw[0].sum() < 1.0

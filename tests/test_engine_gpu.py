"""End-to-end parity of the B200 engine (C ABI, via the Python mirror of the reference API).

  * a small Llama/Qwen-shaped model against the fp32 CPU oracle (oracle/forward.py);
  * the Qwen2.5-7B architecture against the reference's own CUDA build (oracle/_ref) and the oracle;
  * the full layer scan against the reference's stock AttentionLayerScanner path.
Tolerances: per-prompt / per-layer mass rows rel 1e-3 (fp32 attention mass); selected layer and
slot order bit-exact.
"""
from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MASS_REL = 1e-3


def small_config(bias=True, layers=3):
    import attnrank as ar
    return ar.LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=layers, num_attention_heads=4,
                          num_key_value_heads=2, vocab_size=2000, max_position_embeddings=4096, rms_norm_eps=1e-6,
                          rope_theta=1e6, attention_bias=bias)


def oracle_shape(config):
    from oracle import forward as F
    return F.Shape(hidden=config.hidden_size, intermediate=config.intermediate_size, layers=config.num_hidden_layers,
                   heads=config.num_attention_heads, kv_heads=config.num_key_value_heads, vocab=config.vocab_size,
                   eps=config.rms_norm_eps, theta=config.rope_theta, window=config.sliding_window,
                   bias=config.attention_bias)


def oracle_prompt(prompt):
    from oracle import forward as F
    return F.Prompt(tokens=np.asarray(prompt.tokens), query_span=(prompt.query_span.begin, prompt.query_span.end),
                    spans=[(s.begin, s.end) for s in prompt.document_spans])


def small_prompts(count, vocab, seed=3):
    from attnrank import synthetic
    shape = synthetic.PromptShape(documents=5, document_min=20, document_max=90, question=12)
    return synthetic.prompts(count, vocab, shape, seed=seed)


def assert_rows_close(got, want, rel=MASS_REL):
    got, want = np.asarray(got), np.asarray(want)
    error = np.abs(got - want) / np.maximum(np.abs(want), 1e-12)
    assert error.max() <= rel, f"max relative error {error.max():.3e} > {rel}"


@pytest.mark.parametrize("bias,dtype,kernel", [(True, "fp16", "tcgen05"), (False, "fp16", "tcgen05"),
                                               (True, "bf16", "tcgen05"), (True, "fp16", "mma")])
def test_small_model_rows_match_oracle(cuda, bias, dtype, kernel):
    """tcgen05: attention with the mass fused into its softmax; mma: attention + the separate
    tcgen05 mass kernel."""
    import attnrank as ar
    from oracle import forward as F
    config = small_config(bias)
    engine = ar.Engine.synthetic(config, seed=0,
                                 options=ar.RuntimeOptions(activation_dtype=dtype, attention_kernel=kernel))
    prompts = small_prompts(4, config.vocab_size)
    rows, first = engine.probe_rows(prompts)
    assert first == 0 and rows.shape == (4, config.num_hidden_layers, 5)
    oracle = F.OracleModel(oracle_shape(config), seed=0)
    want, _ = oracle.probe([oracle_prompt(p) for p in prompts])
    for p in range(len(prompts)):
        np.testing.assert_allclose(rows[p].sum(axis=1), 1.0, rtol=1e-9)
        assert_rows_close(rows[p], want[p])


def test_small_model_layer_range_and_length_normalisation(cuda):
    import attnrank as ar
    from oracle import forward as F
    config = small_config(True, layers=4)
    engine = ar.Engine.synthetic(config, seed=5)
    prompts = small_prompts(2, config.vocab_size, seed=9)
    result = engine.measure_attention_by_layer(prompts[1], layer_begin=1, layer_end=3, normalize_by_length=True)
    assert result.layer_begin == 1 and len(result.attention_by_layer) == 2
    oracle = F.OracleModel(oracle_shape(config), seed=5)
    want, _ = oracle.probe([oracle_prompt(prompts[1])], 1, 3, normalize_by_length=True)
    assert_rows_close(result.attention_by_layer, want[0])
    # measure_attention: the layer-averaged single profile of model.cu:567-591
    got = engine.measure_attention(prompts[0], layer_span_begin=0, layer_span_end=4)
    assert_rows_close(got, oracle.measure_attention(oracle_prompt(prompts[0]), 0, 4))


@pytest.mark.parametrize("kernel", ["tcgen05", "mma"])
@pytest.mark.parametrize("normalize", [False, True])
def test_long_question_over_several_query_tiles(cuda, kernel, normalize):
    """A 300-token question starting mid-tile: the probe rows span three 128-row query tiles, so
    the fused mass writes several partials per head, and length normalisation crosses the
    reference's 512-token chunk boundary."""
    import attnrank as ar
    from attnrank import synthetic
    from oracle import forward as F
    config = small_config(True, layers=2)
    engine = ar.Engine.synthetic(config, seed=2, options=ar.RuntimeOptions(attention_kernel=kernel))
    shape = synthetic.PromptShape(documents=4, document_min=60, document_max=110, question=300)
    prompts = synthetic.prompts(3, config.vocab_size, shape, seed=21)
    rows, _ = engine.probe_rows(prompts, normalize_by_length=normalize)
    oracle = F.OracleModel(oracle_shape(config), seed=2)
    want, _ = oracle.probe([oracle_prompt(p) for p in prompts], normalize_by_length=normalize)
    for p in range(len(prompts)):
        assert_rows_close(rows[p], want[p])


def test_small_model_scan_matches_host_accumulation(cuda):
    """The device accumulator equals the sum of the per-prompt rows (attnrank.cpp:350-362)."""
    import attnrank as ar
    config = small_config(True)
    engine = ar.Engine.synthetic(config, seed=1)
    prompts = small_prompts(9, config.vocab_size, seed=4)
    rows, _ = engine.probe_rows(prompts)
    accumulated = engine.scan(prompts)
    np.testing.assert_allclose(accumulated, rows.sum(axis=0), rtol=1e-6)
    scan = ar.find_shallowest_attention_layer(engine=engine, samples=prompts,
                                              settings=ar.LayerScanSettings(min_edge_ratio=1.0))
    for layer, profile in enumerate(scan.profiles):
        mean = rows[:, layer, :].mean(axis=0)
        np.testing.assert_allclose(profile.attention, mean / mean.sum(), rtol=1e-6)


def test_engine_rejects_bad_requests(cuda):
    import attnrank as ar
    config = small_config(False, layers=2)
    engine = ar.Engine.synthetic(config, seed=0)
    good = small_prompts(1, config.vocab_size)[0]
    with pytest.raises(ar.AttnRankError):
        engine.measure_attention_by_layer(good, layer_begin=0, layer_end=5)
    bad_token = ar.StructuredPrompt(tokens=[1, 2, config.vocab_size], document_spans=[(0, 1), (1, 2), (2, 3)],
                                    query_span=(2, 3))
    with pytest.raises(ar.AttnRankError, match="vocabulary"):
        engine.measure_attention_by_layer(bad_token)
    # the engine stays usable after a reported error
    assert engine.measure_attention_by_layer(good).layer_begin == 0


@pytest.mark.parametrize("kernel", ["tcgen05", "mma"])
def test_degenerate_spans_follow_the_reference(cuda, kernel):
    """Spans the reference accepts without an error (DocumentAttentionProbe, model.cu:248-251;
    reduce_document_attention_kernel, kernels.cu:211-219): a query span starting before token 0
    covers every row from 0, an empty or reversed query span gives all-zero rows, and an empty or
    reversed document span holds no keys. A document span beginning before token 0 is rejected
    (the reference would read before the score row)."""
    import attnrank as ar
    from oracle import forward as F
    config = small_config(True, layers=2)
    engine = ar.Engine.synthetic(config, seed=4, options=ar.RuntimeOptions(attention_kernel=kernel))
    oracle = F.OracleModel(oracle_shape(config), seed=4)
    base = small_prompts(1, config.vocab_size, seed=11)[0]
    q0, q1 = base.query_span.begin, base.query_span.end
    spans = [(s.begin, s.end) for s in base.document_spans]
    reversed_doc = list(spans)
    reversed_doc[2] = (spans[2][1], spans[2][0])
    empty_doc = list(spans)
    empty_doc[2] = (spans[2][1], spans[2][1])

    def probe(query, document_spans):
        prompt = ar.StructuredPrompt(tokens=base.tokens, document_spans=document_spans, query_span=query)
        return np.asarray(engine.measure_attention_by_layer(prompt).attention_by_layer)

    def expected(query, document_spans):
        prompt = F.Prompt(tokens=np.asarray(base.tokens), query_span=query, spans=document_spans)
        return oracle.probe([prompt])[0][0]

    for query in [(-7, q1), (0, q1)]:
        assert_rows_close(probe(query, spans), expected(query, spans))
    np.testing.assert_array_equal(probe((-7, q1), spans), probe((0, q1), spans))
    for query in [(q1, q0), (q0, q0)]:
        assert not np.any(probe(query, spans))
    got = probe((q0, q1), reversed_doc)
    np.testing.assert_array_equal(got, probe((q0, q1), empty_doc))
    assert not np.any(got[:, 2])
    assert_rows_close(got, expected((q0, q1), reversed_doc))
    with pytest.raises(ar.AttnRankError, match="before token 0"):
        probe((q0, q1), [(-1, 5)] + spans[1:])
    assert engine.measure_attention_by_layer(base).layer_begin == 0  # still usable


# ---- 7B architecture against the reference's CUDA build ------------------------------------
@pytest.fixture(scope="module")
def qwen_pair(cuda, reference_lib):
    if reference_lib is None:
        pytest.skip("oracle/_ref not built")
    import attnrank as ar
    from attnrank import synthetic
    from oracle.reference import ReferenceModel
    config = synthetic.qwen2_7b()
    engine = ar.Engine.synthetic(config, seed=0, options=ar.RuntimeOptions(max_sequence_length=4096))
    reference = ReferenceModel(config, seed=0, max_sequence_length=2048)
    yield config, engine, reference
    reference.close()
    engine.close()


@pytest.mark.slow
def test_qwen7b_rows_match_reference(qwen_pair):
    from attnrank import synthetic
    config, engine, reference = qwen_pair
    prompts = synthetic.prompts(3, config.vocab_size)
    rows, _ = engine.probe_rows(prompts)
    for p, prompt in enumerate(prompts):
        want = reference.measure_attention_by_layer(prompt)
        assert_rows_close(rows[p], want)


def _slot_gap(rows):
    """Smallest relative gap between adjacent masses of any sorted row (an error below half of it
    cannot reorder the slots)."""
    gaps = [(a - b) / a for row in rows for a, b in zip(sorted(row)[::-1], sorted(row)[::-1][1:]) if a > 0]
    return min(gaps)


@pytest.mark.slow
def test_qwen7b_scan_matches_reference(qwen_pair):
    """BASELINE config 3 in full: the 400-prompt scan through find_shallowest_attention_layer
    against the reference's stock AttentionLayerScanner::scan (attnrank.cpp:364-375) on the same
    prompts: every layer's mass row (rel 1e-3) and slot order (exact), the pick at min_edge_ratio
    1.3, LayerScan.highest_ratio_layer (engine.py:304-306), and select_shallowest_basin_layer
    (attnrank.cpp:257-265) at thresholds that pick a layer: 0.9, 1.0 and 1.05, and the midpoints
    between adjacent edge ratios of the reference's profiles. A threshold is used only when its
    distance to every ratio exceeds 3x the largest relative mass error measured here (the
    ratio min(first, last) / mean(interior) moves by at most about twice that), so that no
    threshold sits where the measured error could flip a basin."""
    import attnrank as ar
    from attnrank import synthetic
    from oracle import reference as R
    config, engine, reference = qwen_pair
    prompts = synthetic.prompts(400, config.vocab_size)
    scan = ar.find_shallowest_attention_layer(engine=engine, samples=prompts,
                                              settings=ar.LayerScanSettings(min_edge_ratio=1.3))
    want = reference.scan(prompts, min_edge_ratio=1.3)
    gap = _slot_gap(want.attention)
    worst = max(float(np.max(np.abs(np.asarray(p.attention) - want.attention[i]) / np.abs(want.attention[i])))
                for i, p in enumerate(scan.profiles))
    assert scan.selected_layer == want.selected_layer
    for layer, profile in enumerate(scan.profiles):
        assert profile.layer_index == int(want.layer_index[layer])
        assert_rows_close(profile.attention, want.attention[layer])
        assert list(profile.position_order) == [int(v) for v in want.position_order[layer]], (
            f"layer {layer}: max rel mass error {worst:.2e}, smallest adjacent slot gap {gap:.2e}")
    ratios = [float(R.basin_statistics(row, 1.3)[3]) for row in want.attention]
    highest = int(want.layer_index[max(range(len(ratios)), key=lambda i: ratios[i])])
    assert scan.highest_ratio_layer() == highest
    distinct = sorted(set(ratios))
    candidates = [0.9, 1.0, 1.05] + [0.5 * (a + b) for a, b in zip(distinct, distinct[1:])]
    thresholds = [x for x in candidates if all(abs(x - r) > 3 * worst * r for r in ratios)]
    assert len(thresholds) >= 3, (ratios, worst)
    picked = set()
    for threshold in thresholds:
        mine = ar.select_shallowest_basin_layer(profiles=scan.profiles, min_edge_ratio=threshold)
        theirs = R.select_shallowest(want.attention, want.layer_index, threshold)
        assert mine == theirs, (threshold, mine, theirs)
        picked.add(mine)
    assert any(layer >= 0 for layer in picked), (ratios, thresholds)


# ---- Llama-3-8B long-context probe (4K-token prompts, 20 document spans) against the reference build
@pytest.mark.slow
def test_llama3_long_context_rows_match_reference(cuda, reference_lib):
    if reference_lib is None:
        pytest.skip("oracle/_ref not built")
    import attnrank as ar
    from attnrank import synthetic
    from oracle.reference import ReferenceModel
    config = synthetic.llama3_8b()
    prompts = synthetic.prompts(2, config.vocab_size, synthetic.LLAMA3_LONG_PROMPTS)
    assert all(len(p.document_spans) == 20 for p in prompts)
    longest = max(len(p.tokens) for p in prompts)
    engine = ar.Engine.synthetic(config, seed=0, options=ar.RuntimeOptions(max_sequence_length=8192))
    rows, _ = engine.probe_rows(prompts)
    engine.close()
    reference = ReferenceModel(config, seed=0, max_sequence_length=max(longest, 4096))
    try:
        for p, prompt in enumerate(prompts):
            assert_rows_close(rows[p], reference.measure_attention_by_layer(prompt))
    finally:
        reference.close()


def test_scheduler_scan_on_one_process_equals_the_api_scan(cuda):
    """ProbeScheduler (the multi-GPU scan, here with no process group) against
    find_shallowest_attention_layer on the same engine: same profiles and pick; negative layer
    bounds resolve like the reference (model.cpp:66-68)."""
    import attnrank as ar
    from attnrank.scheduler import ProbeScheduler
    config = small_config(True, layers=3)
    engine = ar.Engine.synthetic(config, seed=6)
    prompts = small_prompts(9, config.vocab_size, seed=17)
    settings = ar.LayerScanSettings(min_edge_ratio=1.0)
    want = ar.find_shallowest_attention_layer(engine=engine, samples=prompts, settings=settings)
    for scan_settings in [settings, ar.LayerScanSettings(layer_begin=-1, layer_end=-1, min_edge_ratio=1.0)]:
        got = ProbeScheduler(engine).find_shallowest_attention_layer(prompts, scan_settings)
        assert got.selected_layer == want.selected_layer
        assert [p.layer_index for p in got.profiles] == [p.layer_index for p in want.profiles]
        for mine, theirs in zip(got.profiles, want.profiles):
            np.testing.assert_allclose(mine.attention, theirs.attention, rtol=1e-6)
            assert mine.position_order == theirs.position_order

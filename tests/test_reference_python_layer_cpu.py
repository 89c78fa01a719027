"""The reference's own Python layer, unchanged, on top of this build's core.

The drop-in keeps the reference's `attnrank/engine.py` and replaces what sits under it
(`attnrank._core`). Here the reference's file is loaded from the reference checkout (the test is
skipped where there is none) with `attnrank._core` bound to this build's `attnrank.core`, and its
functions are checked against this build's own API on the same inputs: basin statistics, the basin
pick, LayerScan (statistics, highest_ratio_layer, profile_for, table, to_dict), the slot order and
the reranking; its find_shallowest_attention_layer runs over token-id prompts with the layer scan
supplied by the fp32 CPU oracle (this host has no GPU), so its validation, configuration and
selection steps all run on this build's types.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

import numpy as np
import pytest

from oracle import REFERENCE_ROOT as REFERENCE  # noqa: E402


@pytest.fixture(scope="module")
def reference_engine():
    path = REFERENCE / "attnrank" / "engine.py"
    if not path.exists():
        pytest.skip("the reference checkout is not on this host")
    from attnrank import core
    saved = sys.modules.get("attnrank._core")
    sys.modules["attnrank._core"] = core
    try:
        spec = importlib.util.spec_from_file_location("reference_attnrank_engine", path)
        module = importlib.util.module_from_spec(spec)
        sys.modules[spec.name] = module  # dataclasses look their module up while the class is built
        spec.loader.exec_module(module)
    finally:
        if saved is None:
            sys.modules.pop("attnrank._core", None)
        else:
            sys.modules["attnrank._core"] = saved
    assert module.core is core
    return module


def _profiles(rows):
    from attnrank import core
    return [core.AttentionProfile.from_accumulated("synthetic", layer, 7, list(row)) for layer, row in enumerate(rows)]


def _rows(seed, layers=6, slots=5):
    rng = np.random.default_rng(seed)
    rows = rng.uniform(0.5, 1.5, size=(layers, slots))
    rows[2] = [3.0, 1.0, 1.0, 1.0, 2.5]   # a basin at ratio 2.5
    rows[4] = [1.0, 1.0, 1.0, 1.0, 1.0]   # ties: the stable order keeps slot order
    return rows


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_host_functions_agree(reference_engine, seed):
    import attnrank as ar
    ref = reference_engine
    profiles = _profiles(_rows(seed))
    for ratio in (0.9, 1.3, 2.0, 3.0):
        for profile in profiles:
            mine = ar.basin_statistics(attention=profile.attention, min_edge_ratio=ratio)
            theirs = ref.basin_statistics(attention=profile.attention, min_edge_ratio=ratio)
            assert (mine.first, mine.last, mine.interior_mean, mine.edge_ratio, mine.is_basin) == (
                theirs.first, theirs.last, theirs.interior_mean, theirs.edge_ratio, theirs.is_basin)
        assert (ar.select_shallowest_basin_layer(profiles=profiles, min_edge_ratio=ratio) ==
                ref.select_shallowest_basin_layer(profiles=profiles, min_edge_ratio=ratio))
        mine = ar.LayerScan(selected_layer=2, min_edge_ratio=ratio, profiles=profiles)
        theirs = ref.LayerScan(selected_layer=2, min_edge_ratio=ratio, profiles=profiles)
        assert mine.highest_ratio_layer() == theirs.highest_ratio_layer()
        assert mine.table() == theirs.table()
        assert mine.to_dict() == theirs.to_dict()
        assert mine.profile_for(layer_index=3) is theirs.profile_for(layer_index=3)
        with pytest.raises(KeyError):
            mine.profile_for(layer_index=99)
        with pytest.raises(KeyError):
            theirs.profile_for(layer_index=99)
    documents = [f"doc{i}" for i in range(7)]
    for profile in profiles:
        for order in (profile.position_order, [4, 4, 0], [9, -1, 2, 1]):
            assert (ar.attention_slot_order(position_order=order, count=7) ==
                    ref.attention_slot_order(position_order=order, count=7))
            assert (ar.rerank_documents(documents_by_relevance=documents, position_order=order) ==
                    ref.rerank_documents(documents_by_relevance=documents, position_order=order))
        assert (ar.rerank_with_profile(documents_by_relevance=documents[:5], profile=profile) ==
                ref.rerank_with_profile(documents_by_relevance=documents[:5], profile=profile))


def test_reference_scan_entry_point_runs_on_token_id_prompts(reference_engine, monkeypatch):
    """The reference's find_shallowest_attention_layer (engine.py:337-355) over token-id prompts:
    its document-count check reads StructuredPrompt.documents, it builds this build's
    LayerScanConfig, and the core's scan -- here the fp32 oracle's rows of a 2-layer model, in
    place of the device scan this host cannot run -- feeds its basin pick."""
    import attnrank as ar
    from attnrank import core, synthetic
    from oracle import forward as F
    ref = reference_engine
    shape = synthetic.PromptShape(documents=5, document_min=10, document_max=30, question=6)
    prompts = synthetic.prompts(3, 500, shape, seed=4)
    oracle = F.OracleModel(F.Shape(hidden=128, intermediate=256, layers=2, heads=2, kv_heads=1, vocab=500,
                                   eps=1e-6, theta=1e6, bias=True), seed=0)
    rows, _ = oracle.probe([F.Prompt(tokens=p.tokens, query_span=tuple(p.query_span),
                                     spans=[tuple(s) for s in p.document_spans]) for p in prompts])
    seen = []

    def oracle_scan(engine, samples, config, progress=None):
        assert isinstance(config, core.LayerScanConfig)
        seen.append((config.model_id, config.layer_begin, config.layer_end, config.normalize_by_document_length))
        assert all(isinstance(s, core.StructuredPrompt) for s in samples)
        accumulated = np.sum(rows, axis=0)
        return [core.AttentionProfile.from_accumulated(config.model_id, layer, len(samples), list(accumulated[layer]))
                for layer in range(accumulated.shape[0])]

    monkeypatch.setattr(core, "scan_attention_layers", oracle_scan)

    class Engine:
        model_directory = "synthetic-2-layer"

    settings = ar.LayerScanSettings(min_edge_ratio=0.5, layer_end=None)
    theirs = ref.find_shallowest_attention_layer(engine=Engine(), samples=prompts, settings=settings)
    mine = ar.find_shallowest_attention_layer(engine=Engine(), samples=prompts, settings=settings)
    assert seen[0] == seen[1] == ("synthetic-2-layer", 0, -1, False)
    assert theirs.selected_layer == mine.selected_layer == 0
    assert theirs.to_dict() == mine.to_dict()
    with pytest.raises(ValueError):
        ref.find_shallowest_attention_layer(engine=Engine(), samples=[], settings=settings)
    short = core.StructuredPrompt(tokens=[1, 2, 3, 4], document_spans=[(0, 1), (1, 2)], query_span=(2, 4))
    with pytest.raises(ValueError):
        ref.find_shallowest_attention_layer(engine=Engine(), samples=[short], settings=settings)
    with pytest.raises(ValueError):
        ar.find_shallowest_attention_layer(engine=Engine(), samples=[short], settings=settings)

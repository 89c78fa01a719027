"""The Python surface keeps the reference's names and keyword arguments (drop-in for the profiling
path). No GPU: signatures and host-only behaviour.

REFERENCE_API lists the public functions of the reference's attnrank/engine.py with their
keyword-only parameters (every one of them is keyword-only there). Two documented differences:
measure_document_attention / measure_attention_by_layer take a token-id `prompt` in place of the
reference's text `question` + `documents` (text needs the reference's tokenizer), and
generate_from_prompt accepts an extra `decode` (token ids -> text) for stop strings.
"""
from __future__ import annotations

import inspect

import pytest

REFERENCE_API = {
    "set_log_level": ["level"],
    "is_model_directory": ["path"],
    "download_model": ["repo_id", "out_dir", "revision", "token", "max_workers"],
    "resolve_model_directory": ["model", "cache_dir", "revision", "token"],
    "model_config": ["model_dir"],
    "detect_chat_format": ["model_dir"],
    "chat_format_names": [],
    "reranker_names": [],
    "load_model": ["model_dir", "settings"],
    "from_pretrained": ["model", "settings", "cache_dir", "revision", "token"],
    "load_model_and_profile": ["model", "profile", "settings"],
    "make_document": ["item", "fallback_id"],
    "make_documents": ["items", "prefix"],
    "make_probe_sample": ["question", "documents", "sample_id"],
    "make_probe_samples": ["items"],
    "load_probe_samples": ["path", "limit"],
    "synthetic_probe_samples": ["settings"],
    "basin_statistics": ["attention", "min_edge_ratio"],
    "scan_attention_layers": ["engine", "samples", "settings", "progress"],
    "select_shallowest_basin_layer": ["profiles", "min_edge_ratio"],
    "find_shallowest_attention_layer": ["engine", "samples", "settings", "progress"],
    "extract_attention_profile": ["engine", "samples", "settings", "progress"],
    "save_attention_profile": ["profile", "path"],
    "load_attention_profile": ["path"],
    "profile_to_dict": ["profile"],
    "build_prompt": ["engine", "question", "documents"],
    "measure_document_attention": ["engine", "question", "documents", "layer_index", "layer_span",
                                   "average_all_layers", "normalize_by_length"],
    "measure_attention_by_layer": ["engine", "question", "documents", "layer_begin", "layer_end",
                                   "normalize_by_length"],
    "attention_slot_order": ["position_order", "count"],
    "rerank_documents": ["documents_by_relevance", "position_order"],
    "rerank_with_profile": ["documents_by_relevance", "profile"],
    "make_reranker": ["strategy", "position_order", "seed", "lim_start_first"],
    "rerank_baseline": ["documents_by_relevance", "strategy", "position_order", "seed", "lim_start_first"],
    "generate_answer": ["engine", "question", "documents", "settings"],
    "generate_from_prompt": ["engine", "prompt", "settings"],
}
TOKEN_PROMPT = {"measure_document_attention", "measure_attention_by_layer"}  # prompt replaces question + documents
EXTRA = {"generate_from_prompt": {"decode"}}


@pytest.mark.parametrize("name", sorted(REFERENCE_API))
def test_reference_function_is_present_with_its_keywords(name):
    import attnrank as ar
    function = getattr(ar, name)
    parameters = inspect.signature(function).parameters
    expected = list(REFERENCE_API[name])
    if name in TOKEN_PROMPT:
        expected = [p for p in expected if p not in ("question", "documents")] + ["prompt"]
    for keyword in expected:
        assert keyword in parameters, f"{name} lacks `{keyword}`"
        assert parameters[keyword].kind == inspect.Parameter.KEYWORD_ONLY, f"{name}: `{keyword}` is keyword-only"
    unexpected = set(parameters) - set(expected) - EXTRA.get(name, set())
    assert not unexpected, f"{name} has parameters the reference does not: {sorted(unexpected)}"


def test_engine_generate_keeps_the_binding_defaults():
    """Engine.generate (bindings.cpp:360-363): prompt_tokens, max_new_tokens=128, stop_sequences=[],
    temperature=0.0, top_p=0.9, top_k=0, seed=1234."""
    import attnrank as ar
    parameters = inspect.signature(ar.Engine.generate).parameters
    defaults = {name: p.default for name, p in parameters.items() if p.default is not inspect.Parameter.empty}
    assert list(parameters)[1] == "prompt_tokens"
    assert defaults["max_new_tokens"] == 128
    assert list(defaults["stop_sequences"]) == []
    assert (defaults["temperature"], defaults["top_p"], defaults["top_k"], defaults["seed"]) == (0.0, 0.9, 0, 1234)


def test_text_only_helpers_say_why_they_are_unavailable(tmp_path):
    import attnrank as ar
    for call in (lambda: ar.build_prompt(engine=None, question="q", documents=[]),
                 lambda: ar.make_documents(items=["a"]),
                 lambda: ar.generate_answer(engine=None, question="q", documents=[]),
                 lambda: ar.download_model(repo_id="org/model")):
        with pytest.raises(ar.AttnRankError, match="tokenizer|outside this build"):
            call()
    assert ar.chat_format_names() == [] and ar.detect_chat_format(model_dir=tmp_path) == ""
    (tmp_path / "config.json").write_text('{"hidden_size": 64}')
    assert ar.model_config(model_dir=tmp_path) == {"hidden_size": 64}
    with pytest.raises(FileNotFoundError):
        ar.resolve_model_directory(model=tmp_path)  # a config.json alone is not a checkpoint directory
    ar.set_log_level(level="debug")


# classes and functions the reference's pybind module registers (bindings.cpp:131-369)
REFERENCE_CORE = ["AttentionProfile", "AttnRankError", "BasinCriterion", "BasinStatistics", "Document",
                  "GenerationResult", "LayerProbeResult", "LayerScanConfig", "LlamaConfig", "ProbeSample",
                  "ProfilerConfig", "PromptTemplate", "RuntimeOptions", "ScoredDocument", "StructuredPrompt",
                  "SyntheticProbeConfig", "TokenSpan", "basin_statistics", "build_attention_profile",
                  "chat_format_names", "detect_chat_format", "load_probe_samples", "make_reranker", "reranker_names",
                  "resolve_position_order", "scan_attention_layers", "select_shallowest_basin_layer", "set_log_level",
                  "synthetic_probe_samples", "Engine"]


def test_core_module_names_match_the_reference_bindings():
    from attnrank import core
    missing = [name for name in REFERENCE_CORE if not hasattr(core, name)]
    assert not missing, missing
    template = core.PromptTemplate()
    assert template.document_index_placeholder == "{index}" and not template.include_titles
    with pytest.raises(core.AttnRankError, match="tokenizer"):
        core.synthetic_probe_samples(core.SyntheticProbeConfig())

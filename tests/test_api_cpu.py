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


def test_config_json_values_are_read_like_the_reference(tmp_path):
    """LlamaConfig::from_json (model.cpp:24-51) through Json::as_int64 / as_double / as_bool
    (core.cpp:412-428): numbers are used, bools count as 0 / 1, and anything else (null, a list
    such as Llama-3-Instruct's eos_token_id, a string) keeps the default."""
    import json

    import attnrank as ar
    (tmp_path / "config.json").write_text(json.dumps({
        "hidden_size": 4096, "intermediate_size": 14336, "num_hidden_layers": 32, "num_attention_heads": 32,
        "num_key_value_heads": 8, "vocab_size": 128256, "rms_norm_eps": 1e-5, "rope_theta": 500000.0,
        "bos_token_id": 128000, "eos_token_id": [128001, 128008, 128009], "max_position_embeddings": None,
        "tie_word_embeddings": False, "sliding_window": None, "model_type": "llama"}))
    config = ar.LlamaConfig.from_file(tmp_path / "config.json")
    assert (config.num_key_value_heads, config.vocab_size, config.bos_token_id) == (8, 128256, 128000)
    assert config.eos_token_id == 2 and config.max_position_embeddings == 4096  # the defaults
    assert config.rope_theta == 500000.0 and config.sliding_window == 0 and not config.tie_word_embeddings
    quirky = ar.LlamaConfig.from_dict({"hidden_size": 512, "num_attention_heads": 4, "vocab_size": "2000",
                                       "tie_word_embeddings": 1, "sliding_window": True})
    assert quirky.vocab_size == 32000 and quirky.tie_word_embeddings and quirky.sliding_window == 0
    assert quirky.num_key_value_heads == 4  # defaults to the attention heads
    with pytest.raises(ar.AttnRankError, match="key/value head"):
        ar.LlamaConfig.from_dict({"hidden_size": 512, "num_attention_heads": 4, "num_key_value_heads": 3})


# attnrank/__init__.py of the reference, less the text facade (AttnRank, PromptTemplate), the dataset
# sources (DatasetSpec, FieldMapping, load_rows) and the answer services (rerank_top_k,
# answer_with_top_k): those need a tokenizer or a dataset service, outside the profiling path
REFERENCE_TOP_LEVEL = [
    "AttentionProfile", "AttnRankError", "Document", "Engine", "EngineSettings", "GenerationSettings", "LayerScan",
    "LayerScanSettings", "ProbeSample", "ProfileSettings", "SyntheticProbeSettings", "attention_slot_order",
    "basin_statistics", "build_prompt", "chat_format_names", "core", "detect_chat_format", "download_model",
    "extract_attention_profile", "find_shallowest_attention_layer", "from_pretrained", "generate_answer",
    "generate_from_prompt", "is_model_directory", "load_attention_profile", "load_model", "load_model_and_profile",
    "load_probe_samples", "make_document", "make_documents", "make_probe_sample", "make_probe_samples",
    "make_reranker", "measure_attention_by_layer", "measure_document_attention", "model_config", "profile_to_dict",
    "rerank_baseline", "rerank_documents", "rerank_with_profile", "reranker_names", "resolve_model_directory",
    "save_attention_profile", "scan_attention_layers", "select_shallowest_basin_layer", "set_log_level",
    "synthetic_probe_samples"]


def test_package_exports_and_settings_keep_the_reference_fields():
    import dataclasses

    import attnrank as ar
    from attnrank.data import classes
    assert [name for name in REFERENCE_TOP_LEVEL if not hasattr(ar, name)] == []
    # data/classes.py:19-31 of the reference, in its order (positional construction agrees)
    engine_fields = ["device", "max_sequence", "chunk", "chat_format", "system_prompt", "instruction", "example",
                     "max_document_tokens", "include_titles", "document_separator", "document_label",
                     "extra_stop_sequences"]
    assert [f.name for f in dataclasses.fields(ar.EngineSettings)][:len(engine_fields)] == engine_fields
    settings = ar.EngineSettings(instruction="Answer briefly.", document_separator="\n\n")
    assert (settings.max_sequence, settings.chunk, settings.document_label) == (4096, 512, None)
    synthetic = ar.SyntheticProbeSettings()
    assert (synthetic.document_slots, synthetic.sample_count, synthetic.words_per_document, synthetic.seed) == \
        (5, 32, 60, 20250807)
    assert classes.STRATEGIES == ("random", "descending", "ascending", "lim", "attnrank")
    assert (classes.DEFAULT_MIN_EDGE_RATIO, classes.DEFAULT_PROBE_SAMPLES, classes.DEFAULT_SEED) == (1.3, 400, 1234)

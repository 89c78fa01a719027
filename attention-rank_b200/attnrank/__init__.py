"""attnrank (B200 build): the attention-profiling path of AttnRank on sm_100a.

Drop-in for the reference's Python API on the profiling path: ``from_pretrained``,
``find_shallowest_attention_layer``, ``scan_attention_layers``, ``rerank_with_profile`` and the
profile / basin helpers keep the reference's names and keyword arguments. Probe samples are
token-id prompts (``StructuredPrompt``). All probing runs in libattnrank_b200.so; importing this
package without the built library raises ImportError.
"""
from attnrank import core
from attnrank.core import (AttentionProfile, AttnRankError, BasinCriterion, BasinStatistics, Document, Engine,
                           GenerationResult, LayerProbeResult, LayerScanConfig, LlamaConfig, ProbeSample,
                           ProfilerConfig, RuntimeOptions, StructuredPrompt, TokenSampler, TokenSpan, make_sampler)
from attnrank.data.classes import (EngineSettings, GenerationSettings, LayerScanSettings, ProfileSettings,
                                   SyntheticProbeSettings)
from attnrank.engine import (LayerScan, attention_slot_order, basin_statistics, extract_attention_profile,
                             find_shallowest_attention_layer, from_pretrained, generate_from_prompt,
                             is_model_directory, set_log_level, model_config, resolve_model_directory,
                             download_model, load_model_and_profile, chat_format_names, detect_chat_format,
                             make_document, make_documents, make_probe_sample, make_probe_samples,
                             load_probe_samples, synthetic_probe_samples, build_prompt, generate_answer,
                             load_attention_profile, load_model, make_prompt, make_reranker,
                             measure_attention_by_layer, measure_document_attention, profile_to_dict,
                             rerank_baseline, rerank_documents, rerank_with_profile, reranker_names,
                             save_attention_profile, scan_attention_layers, select_shallowest_basin_layer,
                             synthetic_engine)

__version__ = "0.1.0"

__all__ = [
    "AttentionProfile", "AttnRankError", "BasinCriterion", "BasinStatistics", "Document", "Engine", "EngineSettings",
    "ProbeSample", "SyntheticProbeSettings",
    "GenerationResult", "GenerationSettings", "TokenSampler", "generate_from_prompt", "make_sampler",
    "LayerProbeResult", "LayerScan", "LayerScanConfig", "LayerScanSettings", "LlamaConfig", "ProfileSettings",
    "ProfilerConfig", "RuntimeOptions", "StructuredPrompt", "TokenSpan", "attention_slot_order", "basin_statistics",
    "core", "extract_attention_profile", "find_shallowest_attention_layer", "from_pretrained", "is_model_directory",
    "load_attention_profile", "load_model", "make_prompt", "make_reranker", "measure_attention_by_layer",
    "measure_document_attention", "profile_to_dict", "rerank_baseline", "rerank_documents", "rerank_with_profile",
    "reranker_names", "save_attention_profile", "scan_attention_layers", "select_shallowest_basin_layer",
    "synthetic_engine", "set_log_level", "model_config", "resolve_model_directory", "download_model",
    "load_model_and_profile", "chat_format_names", "detect_chat_format", "make_document", "make_documents",
    "make_probe_sample", "make_probe_samples", "load_probe_samples", "synthetic_probe_samples", "build_prompt",
    "generate_answer",
]

"""Keyword-only Python API of the profiling path (reference: attnrank/engine.py).

Same function names, arguments and return types as the reference for:
  from_pretrained (:168-182), load_model (:148-165), basin_statistics (:258-259),
  scan_attention_layers (:262-275), select_shallowest_basin_layer (:278-283), LayerScan (:286-334),
  find_shallowest_attention_layer (:337-355), extract_attention_profile (:358-375),
  save/load_attention_profile (:378-384), profile_to_dict (:387-388),
  measure_attention_by_layer (:417-433), attention_slot_order (:436-437),
  rerank_documents (:440-445), rerank_with_profile (:448-449), make_reranker (:452-471),
  rerank_baseline (:474-490).
Probe samples are token-id prompts (core.StructuredPrompt); the reference's text samples need its
tokenizer and prompt builder, which are outside this build: the text-only names (make_document,
build_prompt, generate_answer, ...) exist and raise AttnRankError saying so. Also here:
set_log_level, model_config, resolve_model_directory (local directories), load_model_and_profile,
generate_from_prompt (:504-514).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable, Sequence

import numpy as np

from attnrank import core
from attnrank.core import (AttentionProfile, AttnRankError, Engine, LlamaConfig, RuntimeOptions, StructuredPrompt,
                           TokenSpan)
from attnrank.data.classes import (DEFAULT_MIN_EDGE_RATIO, DEFAULT_SEED, EngineSettings, GenerationSettings,
                                   LayerScanSettings, ProfileSettings)

MODEL_CONFIG_FILE = "config.json"
WEIGHT_FILE_PATTERNS = ("*.safetensors", "pytorch_model*.bin")
MINIMUM_BASIN_SLOTS = 3

ProgressCallback = Callable[[int, int], None]


def is_model_directory(*, path: Path) -> bool:
    if not (path / MODEL_CONFIG_FILE).is_file():
        return False
    return any(any(path.glob(pattern)) for pattern in WEIGHT_FILE_PATTERNS)


def runtime_options(settings: EngineSettings) -> RuntimeOptions:
    return RuntimeOptions(device_index=settings.device, max_sequence_length=settings.max_sequence,
                          prefill_chunk_tokens=settings.chunk, max_batch_tokens=settings.max_batch_tokens,
                          max_batch_prompts=settings.max_batch_prompts, activation_dtype=settings.activation_dtype,
                          attention_kernel=settings.attention_kernel)


def load_model(*, model_dir: Path, settings: EngineSettings = EngineSettings()) -> Engine:
    return Engine(str(model_dir), runtime_options(settings), settings.chat_format, settings.system_prompt)


def from_pretrained(*, model: str | Path, settings: EngineSettings = EngineSettings(), cache_dir: Path | None = None,
                    revision: str | None = None, token: str | None = None) -> Engine:
    candidate = Path(model)
    if is_model_directory(path=candidate):
        return load_model(model_dir=candidate.resolve(), settings=settings)
    if candidate.exists():
        raise FileNotFoundError(f"{model} exists but holds no {MODEL_CONFIG_FILE} and weight shards")
    raise FileNotFoundError(f"{model} is not a local checkpoint directory (hub downloads are outside this build)")


def set_log_level(*, level: str = "info") -> None:
    """set_log_level (reference engine.py:75-76): the level of this package's logger."""
    import logging
    logging.getLogger("attnrank").setLevel(level.upper())


def model_config(*, model_dir: Path) -> dict[str, Any]:
    """model_config (reference engine.py:131-133): the checkpoint's config.json."""
    return json.loads((Path(model_dir) / MODEL_CONFIG_FILE).read_text())


def resolve_model_directory(*, model: str | Path, cache_dir: Path | None = None, revision: str | None = None,
                            token: str | None = None) -> Path:
    """resolve_model_directory (reference engine.py:108-128) for local checkpoint directories; hub
    downloads are outside this build."""
    candidate = Path(model)
    if is_model_directory(path=candidate):
        return candidate.resolve()
    raise FileNotFoundError(f"{model} is not a local checkpoint directory (hub downloads are outside this build)")


def download_model(*, repo_id: str, out_dir: Path | None = None, revision: str | None = None,
                   token: str | None = None, max_workers: int = 8) -> Path:
    """download_model (reference engine.py:85-105): hub downloads are outside this build."""
    raise AttnRankError(f"cannot download {repo_id}: hub downloads are outside this build; pass a local "
                        "checkpoint directory to from_pretrained")


def load_model_and_profile(*, model: str | Path, profile: Path,
                           settings: EngineSettings = EngineSettings()) -> tuple[Engine, AttentionProfile]:
    """load_model_and_profile (reference engine.py:185-193)."""
    return from_pretrained(model=model, settings=settings), load_attention_profile(path=profile)


def chat_format_names() -> list[str]:
    """chat_format_names (reference engine.py:140-141): chat formats belong to the reference's
    prompt builder, which this build does not carry."""
    return []


def detect_chat_format(*, model_dir: Path) -> str:
    """detect_chat_format (reference engine.py:136-137): no chat formats in this build."""
    return ""


def _needs_text(name: str) -> AttnRankError:
    return AttnRankError(f"{name} works on text, which needs the reference's tokenizer and prompt builder; this "
                         "build takes token-id prompts (attnrank.make_prompt / StructuredPrompt)")


def make_document(*, item: Any, fallback_id: str = "") -> Any:
    """make_document (reference engine.py:196-207): text documents are outside this build."""
    raise _needs_text("make_document")


def make_documents(*, items: Any, prefix: str = "doc") -> list[Any]:
    raise _needs_text("make_documents")


def make_probe_sample(*, question: str, documents: Any, sample_id: str = "sample") -> Any:
    raise _needs_text("make_probe_sample")


def make_probe_samples(*, items: Any) -> list[Any]:
    raise _needs_text("make_probe_samples")


def load_probe_samples(*, path: Path, limit: int = 0) -> list[Any]:
    raise _needs_text("load_probe_samples")


def synthetic_probe_samples(*, settings: Any = None) -> list[Any]:
    """synthetic_probe_samples (reference engine.py:249-255) builds text samples; the token-id
    equivalent is attnrank.synthetic.prompts."""
    raise _needs_text("synthetic_probe_samples")


def build_prompt(*, engine: Engine, question: str, documents: Any) -> Any:
    raise _needs_text("build_prompt")


def generate_answer(*, engine: Engine, question: str, documents: Any,
                    settings: GenerationSettings = GenerationSettings()) -> Any:
    """generate_answer (reference engine.py:493-501) formats text; generate_from_prompt or
    Engine.generate take the token ids."""
    raise _needs_text("generate_answer")


def synthetic_engine(*, config: LlamaConfig, seed: int = 0, std: float = 0.02,
                     settings: EngineSettings = EngineSettings()) -> Engine:
    """Additive: an engine on the seeded synthetic checkpoint of ``config``'s architecture."""
    return Engine.synthetic(config, seed=seed, std=std, options=runtime_options(settings))


def make_prompt(*, tokens: Sequence[int], document_spans: Sequence[tuple[int, int]],
                query_span: tuple[int, int]) -> StructuredPrompt:
    """Additive: a token-id probe prompt."""
    return StructuredPrompt(tokens=tokens, document_spans=[TokenSpan(*s) for s in document_spans],
                            query_span=TokenSpan(*query_span))


def basin_statistics(*, attention: Sequence[float], min_edge_ratio: float = DEFAULT_MIN_EDGE_RATIO) -> Any:
    """The basin test of one profile row (reference: engine.py:258-259, attnrank.cpp:236-255)."""
    return core.basin_statistics(attention, core.BasinCriterion(min_edge_ratio))


def _scan_config(settings: LayerScanSettings, engine: Engine) -> core.LayerScanConfig:
    """LayerScanSettings -> the core's LayerScanConfig (a missing layer_end means every layer)."""
    config = core.LayerScanConfig()
    config.model_id = settings.model_id if settings.model_id else engine.model_directory
    config.layer_begin = settings.layer_begin
    config.layer_end = settings.layer_end if settings.layer_end is not None else -1
    config.normalize_by_document_length = settings.normalize_by_length
    config.progress_interval = 0
    return config


def scan_attention_layers(*, engine: Engine, samples: Sequence[StructuredPrompt],
                          settings: LayerScanSettings = LayerScanSettings(),
                          progress: ProgressCallback | None = None) -> list[AttentionProfile]:
    """Profiles of every probed layer over the samples (reference: engine.py:262-275)."""
    return core.scan_attention_layers(engine, list(samples), _scan_config(settings, engine), progress)


def select_shallowest_basin_layer(*, profiles: Sequence[AttentionProfile],
                                  min_edge_ratio: float = DEFAULT_MIN_EDGE_RATIO) -> int:
    """The shallowest basin layer, -1 if none (reference: engine.py:278-283)."""
    return core.select_shallowest_basin_layer(profiles, core.BasinCriterion(min_edge_ratio))


# Columns of LayerScan.table(): header, width, and the row value (profile, statistics) -> text.
_SCAN_COLUMNS = (
    ("layer", 5, lambda profile, stats: f"{profile.layer_index:>5}"),
    ("first", 8, lambda profile, stats: f"{stats.first:>8.4f}"),
    ("interior", 9, lambda profile, stats: f"{stats.interior_mean:>9.4f}"),
    ("last", 8, lambda profile, stats: f"{stats.last:>8.4f}"),
    ("ratio", 7, lambda profile, stats: f"{stats.edge_ratio:>7.2f}"),
)


@dataclass
class LayerScan:
    """What find_shallowest_attention_layer returns: the pick and the profile of every probed
    layer. Fields, methods and the table / dict layouts are the reference's LayerScan
    (engine.py:286-334); its callers (the profile service, the facade) log table(), look a layer
    up with profile_for() and fall back to highest_ratio_layer() when no layer is a basin."""

    selected_layer: int
    min_edge_ratio: float
    profiles: list[AttentionProfile] = field(default_factory=list)

    def statistics(self) -> list[Any]:
        """Basin statistics of each profile, in scan order, at this scan's min_edge_ratio."""
        criterion = core.BasinCriterion(self.min_edge_ratio)
        return [core.basin_statistics(profile.attention, criterion) for profile in self.profiles]

    def profile_for(self, *, layer_index: int) -> AttentionProfile:
        found = next((profile for profile in self.profiles if profile.layer_index == layer_index), None)
        if found is None:
            raise KeyError(f"layer {layer_index} is not part of this scan")
        return found

    def highest_ratio_layer(self) -> int:
        """Layer with the largest edge ratio (the first of equal ones); ValueError on an empty scan."""
        ratios = np.array([stats.edge_ratio for stats in self.statistics()], dtype=np.float64)
        if ratios.size == 0:
            raise ValueError("highest_ratio_layer of a scan without profiles")
        return self.profiles[int(np.argmax(ratios))].layer_index

    def table(self) -> str:
        header = " ".join(f"{name:>{width}}" for name, width, _ in _SCAN_COLUMNS) + "  basin"
        rows = [header]
        for profile, stats in zip(self.profiles, self.statistics()):
            cells = " ".join(render(profile, stats) for _, _, render in _SCAN_COLUMNS)
            mark = ("yes" if stats.is_basin else "-") + ("  <- selected" if profile.layer_index == self.selected_layer
                                                        else "")
            rows.append(f"{cells}  {mark}")
        return "\n".join(rows)

    def to_dict(self) -> dict[str, Any]:
        layers = []
        for profile, stats in zip(self.profiles, self.statistics()):
            layers.append(dict(layer_index=profile.layer_index, attention=list(profile.attention),
                               position_order=list(profile.position_order), edge_ratio=stats.edge_ratio,
                               is_basin=stats.is_basin))
        return dict(selected_layer=self.selected_layer, min_edge_ratio=self.min_edge_ratio, profiles=layers)


def find_shallowest_attention_layer(*, engine: Engine, samples: Sequence[StructuredPrompt],
                                    settings: LayerScanSettings = LayerScanSettings(),
                                    progress: ProgressCallback | None = None) -> LayerScan:
    """Scan every probed layer and pick the shallowest attention basin (reference: engine.py:337-355;
    the same ValueErrors for an empty sample list and for fewer than three documents)."""
    if not samples:
        raise ValueError("at least one probe sample is required")
    slots = len(samples[0].document_spans)
    if slots < MINIMUM_BASIN_SLOTS:
        raise ValueError(f"attention-basin detection needs at least {MINIMUM_BASIN_SLOTS} documents per sample")
    profiles = scan_attention_layers(engine=engine, samples=samples, settings=settings, progress=progress)
    return LayerScan(selected_layer=select_shallowest_basin_layer(profiles=profiles,
                                                                  min_edge_ratio=settings.min_edge_ratio),
                     min_edge_ratio=settings.min_edge_ratio, profiles=profiles)


def extract_attention_profile(*, engine: Engine, samples: Sequence[StructuredPrompt], settings: ProfileSettings,
                              progress: ProgressCallback | None = None) -> AttentionProfile:
    if len(samples) == 0:
        raise ValueError("at least one probe sample is required")
    config = core.ProfilerConfig()
    config.model_id = settings.model_id or engine.model_directory
    config.layer_index = settings.layer_index
    config.average_all_layers = settings.average_all_layers
    if settings.layer_span is not None:
        config.layer_span_begin, config.layer_span_end = settings.layer_span[0], settings.layer_span[1] + 1
    config.normalize_by_document_length = settings.normalize_by_length
    config.progress_interval = 0
    return core.build_attention_profile(engine, list(samples), config, progress)


def save_attention_profile(*, profile: AttentionProfile, path: Path) -> None:
    path.parent.mkdir(parents=True, exist_ok=True)
    profile.save(str(path))


def load_attention_profile(*, path: Path) -> AttentionProfile:
    return AttentionProfile.load(str(path))


def profile_to_dict(*, profile: AttentionProfile) -> dict[str, Any]:
    return json.loads(profile.to_json_string())


def measure_attention_by_layer(*, engine: Engine, prompt: StructuredPrompt, layer_begin: int = 0,
                               layer_end: int | None = None, normalize_by_length: bool = False) -> list[list[float]]:
    result = engine.measure_attention_by_layer(prompt, layer_begin=layer_begin,
                                               layer_end=-1 if layer_end is None else layer_end,
                                               normalize_by_length=normalize_by_length)
    return [list(row) for row in result.attention_by_layer]


def measure_document_attention(*, engine: Engine, prompt: StructuredPrompt, layer_index: int = 0,
                               layer_span: tuple[int, int] | None = None, average_all_layers: bool = False,
                               normalize_by_length: bool = False) -> list[float]:
    span_begin, span_end = (-1, -1) if layer_span is None else (layer_span[0], layer_span[1] + 1)
    return engine.measure_attention(prompt, layer_index=layer_index, layer_span_begin=span_begin,
                                    layer_span_end=span_end, average_all_layers=average_all_layers,
                                    normalize_by_length=normalize_by_length)


def attention_slot_order(*, position_order: Sequence[int], count: int) -> list[int]:
    """The slot of every rank: the profile's order deduplicated and completed to 0..count-1
    (reference: engine.py:436-437, attnrank.cpp:377-392)."""
    return core.resolve_position_order(position_order, count)


def rerank_documents(*, documents_by_relevance: Sequence[Any], position_order: Sequence[int]) -> list[Any]:
    """Place the document of rank r at slot order[r] (reference: engine.py:440-445)."""
    slots = attention_slot_order(position_order=position_order, count=len(documents_by_relevance))
    at_slot = dict(zip(slots, documents_by_relevance))  # slots is a permutation of 0..n-1
    return [at_slot[slot] for slot in range(len(documents_by_relevance))]


def rerank_with_profile(*, documents_by_relevance: Sequence[Any], profile: AttentionProfile) -> list[Any]:
    """rerank_documents with the profile's position order (reference: engine.py:448-449)."""
    return rerank_documents(documents_by_relevance=documents_by_relevance, position_order=profile.position_order)


def generate_from_prompt(*, engine: Engine, prompt: Any, settings: GenerationSettings = GenerationSettings(),
                         decode: Callable[[list[int]], str] | None = None) -> core.GenerationResult:
    """generate_from_prompt (reference engine.py:504-514) on a StructuredPrompt or token ids.

    The reference adds its prompt builder's stop strings; this library has no tokenizer or chat
    formatter, so only ``settings.extra_stop_sequences`` apply, and they need ``decode``."""
    tokens = prompt.tokens if hasattr(prompt, "tokens") else prompt
    return engine.generate(tokens, max_new_tokens=settings.max_new_tokens,
                           stop_sequences=list(settings.extra_stop_sequences), temperature=settings.temperature,
                           top_p=settings.top_p, top_k=settings.top_k, seed=settings.seed, decode=decode)


def make_reranker(*, strategy: str, position_order: Sequence[int] | None = None, seed: int = DEFAULT_SEED,
                  lim_start_first: bool = False) -> Any:
    if strategy == "attnrank":
        if not position_order:
            raise ValueError("strategy 'attnrank' needs a position_order")
        return core.AttentionReranker(list(position_order))
    if strategy == "descending":
        return core.DescendingReranker()
    if strategy == "ascending":
        return core.AscendingReranker()
    if strategy == "random":
        return core.RandomReranker(seed)
    if strategy == "lim":
        return core.LostInTheMiddleReranker(lim_start_first)
    raise ValueError(f"unknown strategy '{strategy}'")


def rerank_baseline(*, documents_by_relevance: Sequence[Any], strategy: str, position_order: Sequence[int] | None = None,
                    seed: int = DEFAULT_SEED, lim_start_first: bool = False) -> list[Any]:
    reranker = make_reranker(strategy=strategy, position_order=position_order, seed=seed,
                             lim_start_first=lim_start_first)
    count = len(documents_by_relevance)
    ranked = [core.ScoredDocument(index, float(count - index)) for index in range(count)]
    return [documents_by_relevance[scored.index] for scored in reranker.rerank(ranked)]


def reranker_names() -> list[str]:
    return core.reranker_names()

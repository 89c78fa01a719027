"""Frozen settings of the Python API (reference: attnrank/data/classes.py:9-80, profiling fields)."""
from __future__ import annotations

from dataclasses import dataclass

DEFAULT_MAX_SEQUENCE = 4096
DEFAULT_PREFILL_CHUNK = 512
DEFAULT_MIN_EDGE_RATIO = 1.3
DEFAULT_PROBE_SAMPLES = 400
DEFAULT_SEED = 1234
DEFAULT_SYNTHETIC_SEED = 20250807
STRATEGIES = ("random", "descending", "ascending", "lim", "attnrank")
DEFAULT_MAX_BATCH_TOKENS = 16384
DEFAULT_MAX_BATCH_PROMPTS = 256


@dataclass(frozen=True, slots=True)
class EngineSettings:
    """The reference's fields in its order (classes.py:19-31), then this build's additions. The
    prompt-builder fields (instruction .. extra_stop_sequences) are kept for callers that set them;
    this build takes token-id prompts, so nothing reads them."""

    device: int = -1
    max_sequence: int = DEFAULT_MAX_SEQUENCE
    chunk: int = DEFAULT_PREFILL_CHUNK
    chat_format: str = ""
    system_prompt: str = ""
    instruction: str | None = None
    example: str | None = None
    max_document_tokens: int = 0
    include_titles: bool = False
    document_separator: str = "\n"
    document_label: str | None = None
    extra_stop_sequences: tuple[str, ...] = ()
    max_batch_tokens: int = DEFAULT_MAX_BATCH_TOKENS      # additive: packed tokens per forward
    max_batch_prompts: int = DEFAULT_MAX_BATCH_PROMPTS    # additive
    activation_dtype: str = "fp16"                        # additive: "fp16" (reference GEMM type) or "bf16"
    #                                                       (bf16 is outside the rel 1e-3 mass bar at 7B)
    attention_kernel: str = "tcgen05"                     # additive: "tcgen05" or "mma"


@dataclass(frozen=True, slots=True)
class SyntheticProbeSettings:
    """SyntheticProbeSettings (classes.py:34-39 of the reference): settings of its text-sample
    generator, which needs a tokenizer; attnrank.synthetic.prompts makes token-id samples."""

    document_slots: int = 5
    sample_count: int = 32
    words_per_document: int = 60
    seed: int = DEFAULT_SYNTHETIC_SEED


@dataclass(frozen=True, slots=True)
class GenerationSettings:
    """GenerationSettings (attnrank/data/classes.py:61-67 of the reference)."""

    max_new_tokens: int = 128
    temperature: float = 0.0
    top_p: float = 0.9
    top_k: int = 0
    seed: int = DEFAULT_SEED
    extra_stop_sequences: tuple[str, ...] = ()


@dataclass(frozen=True, slots=True)
class LayerScanSettings:
    layer_begin: int = 0
    layer_end: int | None = None
    min_edge_ratio: float = DEFAULT_MIN_EDGE_RATIO
    normalize_by_length: bool = False
    model_id: str | None = None


@dataclass(frozen=True, slots=True)
class ProfileSettings:
    layer_index: int
    layer_span: tuple[int, int] | None = None
    average_all_layers: bool = False
    normalize_by_length: bool = False
    model_id: str | None = None

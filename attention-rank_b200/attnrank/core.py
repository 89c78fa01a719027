"""Classes and functions of the reference's ``attnrank._core`` module, backed by libattnrank_b200.so.

Names, fields, defaults and error behaviour follow attnrank/src/bindings.cpp:131-369 for the
parts of the module on the profiling path. Additions are marked "additive": the reference's
``StructuredPrompt`` has no Python constructor (bindings.cpp:173-177), so token-id prompts need
one; ``Engine.synthetic`` builds an engine on the seeded synthetic checkpoint; ``Engine.scan``
exposes the batched device scan.
"""
from __future__ import annotations

import ctypes
import json
import threading
from dataclasses import dataclass, field
from pathlib import Path
from typing import Callable, Sequence

import numpy as np

from attnrank import _native
from attnrank._native import AttnRankError, check, lib

ProgressCallback = Callable[[int, int], None]


# ---------------------------------------------------------------------------------------------
# Plain value types
# ---------------------------------------------------------------------------------------------
@dataclass
class TokenSpan:
    """Half-open token range (include/attnrank/core.hpp:54-60)."""

    begin: int = 0
    end: int = 0

    def length(self) -> int:
        return self.end - self.begin

    def __iter__(self):
        yield self.begin
        yield self.end

    def __repr__(self) -> str:
        return f"TokenSpan({self.begin}, {self.end})"


def _span(value) -> TokenSpan:
    if isinstance(value, TokenSpan):
        return value
    begin, end = value
    return TokenSpan(int(begin), int(end))


@dataclass
class StructuredPrompt:
    """Tokens plus document and query spans (include/attnrank/prompt.hpp:12-17).

    Additive: constructible from token ids, so probes can be fed without the text prompt builder.
    """

    tokens: Sequence[int]
    document_spans: Sequence[TokenSpan]
    query_span: TokenSpan
    text: str = ""

    def __post_init__(self) -> None:
        self.tokens = np.ascontiguousarray(np.asarray(self.tokens, dtype=np.int32))
        self.document_spans = [_span(s) for s in self.document_spans]
        self.query_span = _span(self.query_span)

    @property
    def documents(self) -> list[TokenSpan]:
        """The document spans, under the name a ProbeSample gives its documents: the reference's
        Python layer checks `len(samples[0].documents)` before a scan (engine.py:343-346), so
        token-id prompts pass through it unchanged."""
        return self.document_spans


@dataclass
class LlamaConfig:
    """Model dimensions (include/attnrank/model.hpp:16-38; parsed like model.cpp:24-51)."""

    hidden_size: int = 4096
    intermediate_size: int = 11008
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 32
    vocab_size: int = 32000
    max_position_embeddings: int = 4096
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    bos_token_id: int = 1
    eos_token_id: int = 2
    sliding_window: int = 0
    tie_word_embeddings: bool = False
    attention_bias: bool = False

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_attention_heads

    @classmethod
    def from_dict(cls, root: dict) -> "LlamaConfig":
        def read(key, fallback):
            # Json::as_int64 / as_double (core.cpp:418-428): a number, a bool as 0 / 1, anything
            # else (absent, null, a list such as Llama-3's eos_token_id, a string) the fallback
            value = root.get(key)
            if isinstance(value, bool):
                return int(value)
            return value if isinstance(value, (int, float)) else fallback

        config = cls()
        config.hidden_size = int(read("hidden_size", config.hidden_size))
        config.intermediate_size = int(read("intermediate_size", config.intermediate_size))
        config.num_hidden_layers = int(read("num_hidden_layers", config.num_hidden_layers))
        config.num_attention_heads = int(read("num_attention_heads", config.num_attention_heads))
        config.num_key_value_heads = int(read("num_key_value_heads", config.num_attention_heads))
        config.vocab_size = int(read("vocab_size", config.vocab_size))
        config.max_position_embeddings = int(read("max_position_embeddings", config.max_position_embeddings))
        config.rms_norm_eps = float(read("rms_norm_eps", config.rms_norm_eps))
        config.rope_theta = float(read("rope_theta", config.rope_theta))
        config.bos_token_id = int(read("bos_token_id", config.bos_token_id))
        config.eos_token_id = int(read("eos_token_id", config.eos_token_id))
        window = root.get("sliding_window")
        if isinstance(window, (int, float)) and not isinstance(window, bool):
            config.sliding_window = int(window)
        tied = root.get("tie_word_embeddings")  # Json::as_bool(false), core.cpp:412-416
        config.tie_word_embeddings = bool(tied) if isinstance(tied, (bool, int, float)) else False
        model_type = str(root.get("model_type", ""))
        config.attention_bias = bool(root.get("attention_bias", model_type.startswith("qwen2")))
        if config.num_attention_heads <= 0 or config.hidden_size % config.num_attention_heads != 0:
            raise AttnRankError("invalid attention head configuration")
        if config.num_key_value_heads <= 0 or config.num_attention_heads % config.num_key_value_heads != 0:
            raise AttnRankError("invalid key/value head configuration")
        return config

    @classmethod
    def from_file(cls, path: str | Path) -> "LlamaConfig":
        with open(path, encoding="utf-8") as handle:
            return cls.from_dict(json.load(handle))

    def to_struct(self) -> _native.LlamaConfigStruct:
        return _native.LlamaConfigStruct(
            self.hidden_size, self.intermediate_size, self.num_hidden_layers, self.num_attention_heads,
            self.num_key_value_heads, self.vocab_size, self.max_position_embeddings, self.rms_norm_eps,
            self.rope_theta, self.sliding_window, 1 if self.attention_bias else 0,
            1 if self.tie_word_embeddings else 0)


@dataclass
class RuntimeOptions:
    """LlamaRuntimeOptions (model.hpp:138-142; defaults of bindings.cpp:179-191) + batching limits."""

    device_index: int = -1
    max_sequence_length: int = 2048
    prefill_chunk_tokens: int = 512
    max_batch_tokens: int = 16384
    max_batch_prompts: int = 256
    # Additive: the 16-bit type of weights, GEMM operands and activations ("fp16", the reference's
    # GEMM operand type, or "bf16"), and the attention kernel ("tcgen05" or "mma"). Only "fp16"
    # is held to the rel 1e-3 attention-mass bar against the reference at the 7B shape: rounding
    # the GEMM inputs to bf16 alone moves the mass rows by up to 1.0e-3 from fp32, and a bf16
    # engine measured rel 1.7e-3 against the reference's build. "bf16" is outside that budget.
    activation_dtype: str = "fp16"
    attention_kernel: str = "tcgen05"

    def to_struct(self) -> _native.RuntimeOptionsStruct:
        dtypes = {"fp16": _native.DTYPE_F16, "bf16": _native.DTYPE_BF16}
        kernels = {"tcgen05": 0, "mma": 1}
        if self.activation_dtype not in dtypes:
            raise AttnRankError(f"activation_dtype must be one of {sorted(dtypes)}")
        if self.attention_kernel not in kernels:
            raise AttnRankError(f"attention_kernel must be one of {sorted(kernels)}")
        return _native.RuntimeOptionsStruct(self.device_index, self.max_sequence_length, self.prefill_chunk_tokens,
                                            self.max_batch_tokens, self.max_batch_prompts,
                                            dtypes[self.activation_dtype], kernels[self.attention_kernel])

    @property
    def dtype_code(self) -> int:
        return {"fp16": _native.DTYPE_F16, "bf16": _native.DTYPE_BF16}[self.activation_dtype]


@dataclass
class GenerationResult:
    """GenerationResult (model.hpp:124-129; Python fields of bindings.cpp:286-291)."""

    generated_tokens: list[int]
    text: str = ""
    prompt_token_count: int = 0
    hit_stop_sequence: bool = False

    @property
    def raw_bytes(self) -> bytes:
        return self.text.encode("utf-8", "surrogateescape")


class TokenSampler:
    """GreedySampler (temperature <= 0) or NucleusSampler (model.hpp:88-116, model.cpp:70-127),
    the library's host implementation: the same logits and seed give the reference's token ids."""

    def __init__(self, temperature: float = 0.0, top_p: float = 0.9, top_k: int = 0, seed: int = 1234):
        self.config = _native.SamplerConfigStruct(float(temperature), float(top_p), int(top_k), int(seed))
        handle = ctypes.c_void_p()
        check(lib.ar_sampler_create(ctypes.byref(self.config), ctypes.byref(handle)))
        self._handle = handle

    @property
    def greedy(self) -> bool:
        return self.config.temperature <= 0.0

    def select(self, logits) -> int:
        values = np.ascontiguousarray(logits, dtype=np.float32)
        token = ctypes.c_int32(0)
        check(lib.ar_sampler_select(self._handle, values.ctypes.data, values.size, ctypes.byref(token)))
        return int(token.value)

    def __del__(self, _destroy=lib.ar_sampler_destroy):  # bound now: module globals may be gone at exit
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            _destroy(handle)
            self._handle = None


def make_sampler(temperature: float = 0.0, top_p: float = 0.9, top_k: int = 0, seed: int = 1234) -> TokenSampler:
    """make_sampler (model.cpp:124-127)."""
    return TokenSampler(temperature, top_p, top_k, seed)


def _apply_stop_sequence(decoded: str, stops: Sequence[str]) -> tuple[bool, str]:
    """apply_stop_sequence (model.cu:490-501): the first stop string (in list order) found
    anywhere in the text cuts it at its first occurrence."""
    for stop in stops:
        if not stop:
            continue
        found = decoded.find(stop)
        if found >= 0:
            return True, decoded[:found]
    return False, decoded


@dataclass
class LayerProbeResult:
    """AttentionLayerProbeResult (model.hpp:74-77)."""

    layer_begin: int
    attention_by_layer: list[list[float]]


@dataclass
class LayerScanConfig:
    """LayerScanConfig (attnrank.hpp:170-178)."""

    model_id: str = ""
    layer_begin: int = 0
    layer_end: int = -1
    normalize_by_document_length: bool = False
    progress_interval: int = 25


@dataclass
class ProfilerConfig:
    """AttentionProfilerConfig (attnrank.hpp:144-154)."""

    model_id: str = ""
    layer_index: int = 5
    average_all_layers: bool = False
    layer_span_begin: int = -1
    layer_span_end: int = -1
    normalize_by_document_length: bool = False
    progress_interval: int = 25

    def resolve_layers(self, num_hidden_layers: int) -> tuple[int, int]:
        """AttentionProbeRequest::resolve_layers (model.cpp:57-62)."""
        if self.layer_span_begin >= 0 and self.layer_span_end > self.layer_span_begin:
            return self.layer_span_begin, self.layer_span_end
        if self.average_all_layers:
            return 0, num_hidden_layers
        return self.layer_index, self.layer_index + 1


@dataclass
class BasinCriterion:
    min_edge_ratio: float = 1.5


@dataclass
class BasinStatistics:
    first: float = 0.0
    last: float = 0.0
    interior_mean: float = 0.0
    edge_ratio: float = 0.0
    is_basin: bool = False

    def __repr__(self) -> str:
        return (f"BasinStatistics(first={self.first:.6f}, interior_mean={self.interior_mean:.6f}, "
                f"last={self.last:.6f}, edge_ratio={self.edge_ratio:.6f}, is_basin={self.is_basin})")


def _f64(values: Sequence[float]) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(values, dtype=np.float64))


@dataclass
class AttentionProfile:
    """AttentionProfile (attnrank.hpp:64-81): attention per slot and the slot order it implies."""

    model_id: str = ""
    layer_index: int = 0
    sample_count: int = 0
    attention: list[float] = field(default_factory=list)
    position_order: list[int] = field(default_factory=list)

    def recompute_position_order(self) -> None:
        values = _f64(self.attention)
        order = np.zeros(len(values), dtype=np.int32)
        check(lib.ar_position_order(values.ctypes.data, len(values), order.ctypes.data))
        self.position_order = [int(v) for v in order]

    @classmethod
    def from_accumulated(cls, model_id: str, layer_index: int, sample_count: int,
                         accumulated: Sequence[float]) -> "AttentionProfile":
        values = _f64(accumulated)
        attention = np.zeros(len(values), dtype=np.float64)
        order = np.zeros(len(values), dtype=np.int32)
        check(lib.ar_profile_from_accumulated(values.ctypes.data, len(values), int(sample_count),
                                              attention.ctypes.data, order.ctypes.data))
        return cls(model_id, layer_index, int(sample_count), [float(v) for v in attention], [int(v) for v in order])

    def to_dict(self) -> dict:
        return {
            "model_id": self.model_id,
            "layer_index": self.layer_index,
            "sample_count": self.sample_count,
            "document_slots": len(self.attention),
            "attention": list(self.attention),
            "position_order": list(self.position_order),
        }

    def to_json_string(self) -> str:
        return json.dumps(self.to_dict(), indent=2)

    def save(self, path: str | Path) -> None:
        try:
            Path(path).write_text(self.to_json_string() + "\n", encoding="utf-8")
        except OSError as error:
            raise AttnRankError(f"cannot write attention profile to '{path}'") from error

    @classmethod
    def from_json(cls, root: dict) -> "AttentionProfile":
        profile = cls(model_id=str(root.get("model_id", "")), layer_index=int(root["layer_index"]),
                      sample_count=int(root["sample_count"]),
                      attention=[float(v) for v in root["attention"]])
        order = root.get("position_order")
        if order is not None and len(order) == len(profile.attention):
            profile.position_order = [int(v) for v in order]
        else:
            profile.recompute_position_order()
        return profile

    @staticmethod
    def load(path: str | Path) -> "AttentionProfile":
        with open(path, encoding="utf-8") as handle:
            return AttentionProfile.from_json(json.load(handle))

    def __repr__(self) -> str:
        return self.to_json_string()


def basin_statistics(attention: Sequence[float], criterion: BasinCriterion) -> BasinStatistics:
    values = _f64(attention)
    out = _native.BasinStatsStruct()
    check(lib.ar_basin_statistics(values.ctypes.data, len(values), float(criterion.min_edge_ratio), ctypes.byref(out)))
    return BasinStatistics(out.first, out.last, out.interior_mean, out.edge_ratio, bool(out.is_basin))


def select_shallowest_basin_layer(profiles: Sequence[AttentionProfile], criterion: BasinCriterion) -> int:
    if not profiles:
        return -1
    slots = len(profiles[0].attention)
    if any(len(p.attention) != slots for p in profiles):
        raise AttnRankError("profiles must share the slot count")
    matrix = np.ascontiguousarray(np.array([p.attention for p in profiles], dtype=np.float64).reshape(-1))
    layers = np.ascontiguousarray(np.array([p.layer_index for p in profiles], dtype=np.int32))
    selected = ctypes.c_int(-1)
    check(lib.ar_select_shallowest_basin_layer(matrix.ctypes.data, layers.ctypes.data, len(profiles), slots,
                                               float(criterion.min_edge_ratio), ctypes.byref(selected)))
    return selected.value


def resolve_position_order(preferred: Sequence[int], count: int) -> list[int]:
    pref = np.ascontiguousarray(np.asarray(list(preferred), dtype=np.int32))
    out = np.zeros(max(count, 0), dtype=np.int32)
    check(lib.ar_resolve_position_order(pref.ctypes.data if pref.size else None, pref.size, int(count),
                                        out.ctypes.data if out.size else None))
    return [int(v) for v in out]


# ---------------------------------------------------------------------------------------------
# Rerankers (attnrank.hpp:197-269) -- host-only placement strategies around the profile
# ---------------------------------------------------------------------------------------------
@dataclass
class ScoredDocument:
    index: int
    score: float = 0.0


class Reranker:
    name = ""

    def rerank(self, ranked: Sequence[ScoredDocument]) -> list[ScoredDocument]:
        raise NotImplementedError


class DescendingReranker(Reranker):
    name = "descending"

    def rerank(self, ranked):
        return list(ranked)


class AscendingReranker(Reranker):
    name = "ascending"

    def rerank(self, ranked):
        return list(reversed(list(ranked)))


class RandomReranker(Reranker):
    """xorshift64 Fisher-Yates shuffle (attnrank.cpp:400-410)."""

    name = "random"
    _golden = 0x9E3779B97F4A7C15

    def __init__(self, seed: int = 1234):
        self._state = (seed if seed != 0 else self._golden) & 0xFFFFFFFFFFFFFFFF

    def rerank(self, ranked):
        result = list(ranked)
        mask = 0xFFFFFFFFFFFFFFFF
        for index in range(len(result), 1, -1):
            self._state ^= (self._state << 13) & mask
            self._state ^= self._state >> 7
            self._state ^= (self._state << 17) & mask
            j = self._state % index
            result[index - 1], result[j] = result[j], result[index - 1]
        return result


class PositionPriorityReranker(Reranker):
    def priority(self, count: int) -> list[int]:
        raise NotImplementedError

    def rerank(self, ranked):
        ranked = list(ranked)
        order = resolve_position_order(self.priority(len(ranked)), len(ranked))
        result: list = [None] * len(ranked)
        for rank, document in enumerate(ranked):
            result[order[rank]] = document
        return result


class LostInTheMiddleReranker(PositionPriorityReranker):
    name = "lim"

    def __init__(self, start_first: bool = False):
        self.start_first = start_first

    def priority(self, count):
        order, front, back, take_front = [], 0, count - 1, self.start_first
        while front <= back:
            if take_front:
                order.append(front)
                front += 1
            else:
                order.append(back)
                back -= 1
            take_front = not take_front
        return order


class AttentionReranker(PositionPriorityReranker):
    name = "attnrank"

    def __init__(self, position_order: Sequence[int]):
        if not position_order:
            raise AttnRankError("AttentionReranker requires a position order")
        self.position_order = list(position_order)

    def priority(self, count):
        return list(self.position_order)


def reranker_names() -> list[str]:
    return ["random", "descending", "ascending", "lim", "attnrank"]


def make_reranker(name: str, profile: AttentionProfile | None = None, seed: int = 1234,
                  lim_start_first: bool = False) -> Reranker:
    if name == "descending":
        return DescendingReranker()
    if name == "ascending":
        return AscendingReranker()
    if name == "random":
        return RandomReranker(seed)
    if name == "lim":
        return LostInTheMiddleReranker(lim_start_first)
    if name == "attnrank":
        if profile is None:
            raise AttnRankError("strategy 'attnrank' needs an attention profile")
        return AttentionReranker(profile.position_order)
    raise AttnRankError(f"unknown reranking strategy '{name}'")


# ---------------------------------------------------------------------------------------------
# Engine
# ---------------------------------------------------------------------------------------------
class _PackedPrompts:
    """Prompts laid out for the C ABI: one int32 token buffer, one span buffer, an ar_prompt array."""

    def __init__(self, prompts: Sequence[StructuredPrompt]):
        if len(prompts) == 0:
            raise AttnRankError("attention probe requires at least one prompt")
        self.span_count = len(prompts[0].document_spans)
        if self.span_count == 0:
            raise AttnRankError("attention probe requires document spans")
        for index, prompt in enumerate(prompts):
            if len(prompt.document_spans) != self.span_count:
                raise AttnRankError(f"probe sample {index} has {len(prompt.document_spans)} documents but the "
                                    f"first sample has {self.span_count}")
        lengths = np.array([len(p.tokens) for p in prompts], dtype=np.int64)
        offsets = np.concatenate([[0], np.cumsum(lengths)])
        self.tokens = np.empty(int(offsets[-1]), dtype=np.int32)
        for prompt, start in zip(prompts, offsets[:-1]):
            self.tokens[start:start + len(prompt.tokens)] = prompt.tokens
        self.spans = np.ascontiguousarray(
            np.array([[(s.begin, s.end) for s in p.document_spans] for p in prompts], dtype=np.int32).reshape(-1))
        self.array = (_native.PromptStruct * len(prompts))()
        base_tokens = self.tokens.ctypes.data
        base_spans = self.spans.ctypes.data
        for i, prompt in enumerate(prompts):
            entry = self.array[i]
            entry.tokens = base_tokens + int(offsets[i]) * 4
            entry.token_count = int(lengths[i])
            entry.query_begin = prompt.query_span.begin
            entry.query_end = prompt.query_span.end
            entry.spans = base_spans + i * self.span_count * 8
        self.count = len(prompts)
        self.token_total = int(offsets[-1])


class Engine:
    """The model resident on one B200 (reference: _core.Engine over CudaLlamaModel).

    Construct with a Hugging Face checkpoint directory (config.json + *.safetensors), or use
    ``Engine.synthetic`` for the seeded random-init checkpoint. Not reentrant: one host thread
    per engine, like the reference (its forward pass keeps a shared workspace).
    """

    def __init__(self, model_directory: str | Path | None = None, options: RuntimeOptions | None = None,
                 chat_format: str = "", system_prompt: str = "", prompt_template=None, *,
                 config: LlamaConfig | None = None):
        self._handle = None
        self._lock = threading.Lock()
        self.options = options or RuntimeOptions()
        self.model_directory = "" if model_directory is None else str(model_directory)
        self.chat_format = chat_format
        if config is None:
            if model_directory is None:
                raise AttnRankError("Engine needs a model directory or a config")
            config = LlamaConfig.from_file(Path(model_directory) / "config.json")
            # q/k/v biases are used when the checkpoint holds them (model.cu:160-162)
            from attnrank.checkpoint import has_attention_bias
            config.attention_bias = has_attention_bias(Path(model_directory))
        self.config = config
        handle = ctypes.c_void_p()
        options_struct = self.options.to_struct()
        config_struct = config.to_struct()
        check(lib.ar_engine_create(ctypes.byref(config_struct), ctypes.byref(options_struct), ctypes.byref(handle)))
        self._handle = handle
        if model_directory is not None:
            from attnrank.checkpoint import load_directory
            load_directory(self, Path(model_directory))

    @classmethod
    def synthetic(cls, config: LlamaConfig, seed: int = 0, std: float = 0.02,
                  options: RuntimeOptions | None = None, model_id: str = "synthetic") -> "Engine":
        """Additive: an engine on the seeded synthetic checkpoint (csrc/synthetic.h)."""
        engine = cls(None, options, config=config)
        engine.model_directory = model_id
        check(lib.ar_engine_init_synthetic(engine._handle, int(seed), float(std)))
        return engine

    def __del__(self, _destroy=lib.ar_engine_destroy):  # bound now: module globals may be gone at exit
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            _destroy(handle)
            self._handle = None

    def close(self) -> None:
        self.__del__()

    @property
    def num_layers(self) -> int:
        return self.config.num_hidden_layers

    @property
    def device(self) -> int:
        return int(lib.ar_engine_device(self._handle))

    @property
    def stream(self) -> int:
        return int(lib.ar_engine_stream(self._handle) or 0)

    def synchronize(self) -> None:
        """Wait for the engine's stream; raises AttnRankError on a device-reported error."""
        check(lib.ar_engine_synchronize(self._handle))

    def set_kernel_timing(self, enabled: bool) -> None:
        """Additive: bracket every engine launch with CUDA events (see kernel_timing)."""
        check(lib.ar_engine_set_kernel_timing(self._handle, 1 if enabled else 0))

    def kernel_timing(self) -> dict[str, dict]:
        """Per kernel class since the last call: {name: {ms, work, launches, tensor}} (then cleared).

        `work` is algorithmic FLOPs for tensor classes and HBM bytes for the others."""
        count = _native.KERNEL_CLASS_COUNT
        ms = (ctypes.c_double * count)()
        work = (ctypes.c_double * count)()
        launches = (ctypes.c_int64 * count)()
        check(lib.ar_engine_kernel_timing(self._handle, ms, work, launches))
        result = {}
        for k in range(count):
            name = lib.ar_kernel_class_name(k).decode()
            result[name] = {"ms": ms[k], "work": work[k], "launches": int(launches[k]),
                            "tensor": bool(lib.ar_kernel_class_is_tensor(k))}
        return result

    # -- generation ----------------------------------------------------------------------------
    def generate(self, prompt_tokens: Sequence[int], max_new_tokens: int = 128, stop_sequences: Sequence[str] = (),
                 temperature: float = 0.0, top_p: float = 0.9, top_k: int = 0, seed: int = 1234, *,
                 decode: Callable[[list[int]], str] | None = None) -> GenerationResult:
        """Engine.generate (bindings.cpp:360-363 -> CudaLlamaModel::generate, model.cu:532-565).

        Stops at the config's eos_token_id (not returned), max_new_tokens or the end of the context
        (RuntimeOptions.max_sequence_length). Text needs a tokenizer, which this library does not
        carry: pass ``decode`` (token ids -> str) to get ``text`` and to use ``stop_sequences``.
        Without stop strings the whole loop runs in the library (greedy selection on the device);
        with them the loop runs here, one library step per token, testing the decoded text after
        every token as the reference does."""
        tokens = np.ascontiguousarray(np.asarray(prompt_tokens, dtype=np.int32).ravel())
        stops = [stop for stop in stop_sequences if stop]
        if stops and decode is None:
            raise AttnRankError("stop_sequences need a decode function (token ids -> text)")
        eos = int(self.config.eos_token_id)
        if not stops:
            config = _native.SamplerConfigStruct(float(temperature), float(top_p), int(top_k), int(seed))
            out = np.zeros(max(int(max_new_tokens), 1), dtype=np.int32)
            count = ctypes.c_int(0)
            with self._lock:
                check(lib.ar_engine_generate(self._handle, tokens.ctypes.data, tokens.size, int(max_new_tokens), eos,
                                             ctypes.byref(config), out.ctypes.data, ctypes.byref(count)))
            generated = [int(t) for t in out[:count.value]]
            text = decode(generated) if decode is not None and generated else ""
            return GenerationResult(generated, text, int(tokens.size), False)

        sampler = make_sampler(temperature, top_p, top_k, seed)
        logits = np.empty(self.config.vocab_size, dtype=np.float32)
        generated: list[int] = []
        decoded, hit = "", False
        with self._lock:
            check(lib.ar_engine_generation_begin(self._handle, tokens.ctypes.data, tokens.size, logits.ctypes.data))
            limit = min(int(max_new_tokens), self.options.max_sequence_length - int(tokens.size))
            for step in range(limit):
                token = sampler.select(logits)
                if token == eos:
                    break
                generated.append(token)
                decoded = decode(generated)
                hit, text = _apply_stop_sequence(decoded, stops)
                if hit:
                    return GenerationResult(generated, text, int(tokens.size), True)
                if step + 1 >= limit:
                    break
                check(lib.ar_engine_generation_step(self._handle, token, logits.ctypes.data))
        return GenerationResult(generated, decoded, int(tokens.size), False)

    def generation_begin(self, prompt_tokens: Sequence[int]) -> np.ndarray:
        """Additive: prefill a prompt into the KV cache; returns the next-token logits (fp32 [vocab])."""
        tokens = np.ascontiguousarray(np.asarray(prompt_tokens, dtype=np.int32).ravel())
        logits = np.empty(self.config.vocab_size, dtype=np.float32)
        with self._lock:
            check(lib.ar_engine_generation_begin(self._handle, tokens.ctypes.data, tokens.size, logits.ctypes.data))
        return logits

    def generation_step(self, token: int) -> np.ndarray:
        """Additive: feed one token at the next position; returns the next-token logits."""
        logits = np.empty(self.config.vocab_size, dtype=np.float32)
        with self._lock:
            check(lib.ar_engine_generation_step(self._handle, int(token), logits.ctypes.data))
        return logits

    @property
    def generation_position(self) -> int:
        return int(lib.ar_engine_generation_position(self._handle))

    @property
    def decode_mode(self) -> str:
        """Additive: how decode steps run ("persistent", "programmatic", "serialised", or "" before
        the first generation)."""
        return {2: "persistent", 1: "programmatic", 0: "serialised"}.get(int(lib.ar_engine_decode_mode(self._handle)), "")

    def prepare_scan(self, prompts: Sequence[StructuredPrompt], layer_begin: int = 0, layer_end: int = -1,
                     normalize_by_length: bool = False) -> "PreparedScan":
        return PreparedScan(self, prompts, layer_begin, layer_end, normalize_by_length)

    def load_tensor(self, name: str, array: np.ndarray, dtype_code: int) -> None:
        array = np.ascontiguousarray(array)
        shape = (ctypes.c_int64 * array.ndim)(*array.shape)
        check(lib.ar_engine_load_tensor(self._handle, name.encode(), dtype_code, shape, array.ndim, array.ctypes.data))

    # -- probes ------------------------------------------------------------------------------
    def measure_attention_by_layer(self, prompt: StructuredPrompt, layer_begin: int = 0, layer_end: int = -1,
                                   normalize_by_length: bool = False) -> LayerProbeResult:
        rows, first = self.probe_rows([prompt], layer_begin, layer_end, normalize_by_length)
        return LayerProbeResult(first, rows[0].tolist())

    def probe_rows(self, prompts: Sequence[StructuredPrompt], layer_begin: int = 0, layer_end: int = -1,
                   normalize_by_length: bool = False) -> tuple[np.ndarray, int]:
        """Additive, batched measure_attention_by_layer: ([prompts, layers, spans] fp64, first layer)."""
        packed = _PackedPrompts(prompts)
        begin = 0 if layer_begin < 0 else layer_begin
        end = self.num_layers if layer_end < 0 else layer_end
        layers = max(end - begin, 0)
        rows = np.zeros((packed.count, max(layers, 1), packed.span_count), dtype=np.float64)
        first, count = ctypes.c_int(0), ctypes.c_int(0)
        with self._lock:
            check(lib.ar_engine_measure_attention_by_layer(self._handle, packed.array, packed.count, packed.span_count,
                                                           int(layer_begin), int(layer_end), int(normalize_by_length),
                                                           rows.ctypes.data, ctypes.byref(first), ctypes.byref(count)))
        return rows[:, :count.value, :], first.value

    def measure_attention(self, prompt: StructuredPrompt, layer_index: int = 0, layer_span_begin: int = -1,
                          layer_span_end: int = -1, average_all_layers: bool = False,
                          normalize_by_length: bool = False) -> list[float]:
        config = ProfilerConfig(layer_index=layer_index, average_all_layers=average_all_layers,
                                layer_span_begin=layer_span_begin, layer_span_end=layer_span_end)
        begin, end = config.resolve_layers(self.num_layers)
        packed = _PackedPrompts([prompt])
        out = np.zeros(packed.span_count, dtype=np.float64)
        with self._lock:
            check(lib.ar_engine_measure_attention(self._handle, packed.array, packed.span_count, begin, end,
                                                  int(normalize_by_length), out.ctypes.data))
        return [float(v) for v in out]

    def scan(self, prompts: Sequence[StructuredPrompt], layer_begin: int = 0, layer_end: int = -1,
             normalize_by_length: bool = False, accumulator=None) -> np.ndarray:
        """Additive: the device scan. Adds the per-prompt unit-sum rows of every prompt into
        ``accumulator`` (a torch fp32 CUDA tensor [layers * spans] on this engine's device; created
        zero-filled when omitted) and returns its value as fp64 [layers, spans]."""
        import torch

        packed = _PackedPrompts(prompts)
        begin = 0 if layer_begin < 0 else layer_begin
        end = self.num_layers if layer_end < 0 else layer_end
        layers = end - begin
        if accumulator is None:
            accumulator = torch.zeros(layers * packed.span_count, dtype=torch.float32, device=f"cuda:{self.device}")
            torch.cuda.synchronize(self.device)
        if accumulator.numel() != layers * packed.span_count or accumulator.dtype != torch.float32:
            raise AttnRankError("accumulator must be fp32 with layers * spans elements")
        host = np.zeros(layers * packed.span_count, dtype=np.float64)
        with self._lock:
            check(lib.ar_engine_scan(self._handle, packed.array, packed.count, packed.span_count, int(layer_begin),
                                     int(layer_end), int(normalize_by_length), accumulator.data_ptr(),
                                     host.ctypes.data))
        return host.reshape(layers, packed.span_count)


class PreparedScan:
    """Additive: a scan whose inputs are resident in HBM (ar_engine_prepare_scan).

    ``run`` enqueues every batch on the engine's stream; with ``synchronize=False`` it returns
    immediately, so several runs (or an NCCL all-reduce on the same stream) can be queued.
    """

    def __init__(self, engine: "Engine", prompts: Sequence[StructuredPrompt], layer_begin: int = 0,
                 layer_end: int = -1, normalize_by_length: bool = False):
        packed = _PackedPrompts(prompts)
        self.engine = engine
        self.span_count = packed.span_count
        self.prompt_count = packed.count
        self.token_count = packed.token_total
        begin = 0 if layer_begin < 0 else layer_begin
        end = engine.num_layers if layer_end < 0 else layer_end
        self.layer_begin = begin
        self.layers = end - begin
        handle = ctypes.c_void_p()
        check(lib.ar_engine_prepare_scan(engine._handle, packed.array, packed.count, packed.span_count,
                                         int(layer_begin), int(layer_end), int(normalize_by_length),
                                         ctypes.byref(handle)))
        self._handle = handle
        self.device_bytes = int(lib.ar_prepared_scan_bytes(handle))

    def run(self, accumulator, synchronize: bool = True) -> None:
        check(lib.ar_engine_run_prepared_scan(self.engine._handle, self._handle, accumulator.data_ptr(),
                                              1 if synchronize else 0))

    def __del__(self, _destroy=lib.ar_prepared_scan_destroy):  # bound now: module globals may be gone at exit
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            _destroy(handle)
            self._handle = None


# ---- text-side records of the reference's _core (bindings.cpp:136-244), kept for API compatibility.
# This build probes token-id prompts; these records carry text, which needs the reference's
# tokenizer and prompt builder, so scans given them raise AttnRankError (see _as_prompts).
@dataclass
class Document:
    """Document (core.hpp:43-47; bindings.cpp:136-149)."""

    id: str = ""
    title: str = ""
    text: str = ""


@dataclass
class ProbeSample:
    """ProbeSample (bindings.cpp:151-162): a question with its documents."""

    question: str = ""
    documents: list[Document] = field(default_factory=list)


@dataclass
class PromptTemplate:
    """DocumentPromptTemplate (prompt.hpp:78-92; bindings.cpp:207-219), the reference prompt
    builder's layout and defaults."""

    instruction: str = ("Write a high-quality answer for the given question using only the provided search "
                        "results (some of which might be irrelevant).")
    example: str = ""
    documents_header: str = ""
    document_label: str = "Document [{index}] "
    document_index_placeholder: str = "{index}"
    document_separator: str = "\n"
    question_prefix: str = "Question: "
    answer_prefix: str = "Answer:"
    max_document_tokens: int = 0
    include_titles: bool = False
    extra_stop_sequences: list[str] = field(default_factory=list)


@dataclass
class SyntheticProbeConfig:
    """SyntheticProbeConfig (attnrank.hpp:43-48): the reference's synthetic TEXT samples. The
    token-id workloads of this build come from attnrank.synthetic.prompts."""

    document_slots: int = 10
    sample_count: int = 400
    words_per_document: int = 60
    seed: int = 20250807


def _text_unavailable(name: str) -> AttnRankError:
    return AttnRankError(f"{name} builds text samples, which need the reference's tokenizer and prompt "
                         "builder; this build takes token-id prompts (StructuredPrompt)")


def load_probe_samples(jsonl_path) -> list[ProbeSample]:
    """load_probe_samples (bindings.cpp:331): text samples are outside this build."""
    raise _text_unavailable("load_probe_samples")


def synthetic_probe_samples(config: SyntheticProbeConfig) -> list[ProbeSample]:
    """synthetic_probe_samples (bindings.cpp:332): text samples are outside this build."""
    raise _text_unavailable("synthetic_probe_samples")


def chat_format_names() -> list[str]:
    """chat_format_names (bindings.cpp:333): no chat formats in this build."""
    return []


def detect_chat_format(model_directory) -> str:
    """detect_chat_format (bindings.cpp:334): no chat formats in this build."""
    return ""


def set_log_level(level: str) -> None:
    """set_log_level (bindings.cpp:335): the level of this package's logger."""
    import logging
    logging.getLogger("attnrank").setLevel(str(level).upper())


def _as_prompts(samples: Sequence) -> list[StructuredPrompt]:
    prompts = []
    for index, sample in enumerate(samples):
        if isinstance(sample, StructuredPrompt):
            prompts.append(sample)
        else:
            raise AttnRankError(
                f"probe sample {index} is a {type(sample).__name__}; this build probes token-id prompts "
                "(StructuredPrompt); text samples need the reference's tokenizer and prompt builder")
    return prompts


def scan_attention_layers(engine: Engine, samples: Sequence, config: LayerScanConfig,
                          progress: ProgressCallback | None = None) -> list[AttentionProfile]:
    """AttentionLayerScanner::scan (attnrank.cpp:364-375) on the device: per-layer profiles."""
    prompts = _as_prompts(samples)
    if not prompts:
        raise AttnRankError("probe needs at least one sample")
    if progress is None:
        accumulated = engine.scan(prompts, config.layer_begin, config.layer_end, config.normalize_by_document_length)
    else:
        accumulated = None
        step = max(1, engine.options.max_batch_prompts)
        for start in range(0, len(prompts), step):
            part = engine.scan(prompts[start:start + step], config.layer_begin, config.layer_end,
                               config.normalize_by_document_length)
            accumulated = part if accumulated is None else accumulated + part
            progress(min(start + step, len(prompts)), len(prompts))
    first = 0 if config.layer_begin < 0 else config.layer_begin
    model_id = config.model_id or engine.model_directory
    return [AttentionProfile.from_accumulated(model_id, first + layer, len(prompts), accumulated[layer])
            for layer in range(accumulated.shape[0])]


def build_attention_profile(engine: Engine, samples: Sequence, config: ProfilerConfig,
                            progress: ProgressCallback | None = None) -> AttentionProfile:
    """AttentionProfiler::build_profile (attnrank.cpp:331-335): one profile from measure_attention."""
    prompts = _as_prompts(samples)
    if not prompts:
        raise AttnRankError("probe needs at least one sample")
    slots = len(prompts[0].document_spans)
    accumulated = np.zeros(slots, dtype=np.float64)
    for index, prompt in enumerate(prompts):
        if len(prompt.document_spans) != slots:
            raise AttnRankError(f"probe sample {index} produced {len(prompt.document_spans)} spans, expected {slots}")
        accumulated += np.asarray(engine.measure_attention(
            prompt, layer_index=config.layer_index, layer_span_begin=config.layer_span_begin,
            layer_span_end=config.layer_span_end, average_all_layers=config.average_all_layers,
            normalize_by_length=config.normalize_by_document_length))
        if progress is not None:
            progress(index + 1, len(prompts))
    return AttentionProfile.from_accumulated(config.model_id or engine.model_directory, config.layer_index,
                                             len(prompts), accumulated)

"""Seeded synthetic probe prompts and model shapes of the benchmark configurations, as API types.

The generator itself is `probe_workloads` (numpy only, beside this package), so that code which
must not load this library -- the benchmark's reference arm -- draws the same prompts. Prompt i of
seed s is a pure function of (s, i).
"""
from __future__ import annotations

from dataclasses import asdict

from attnrank.core import LlamaConfig, StructuredPrompt, TokenSpan
from probe_workloads import (LLAMA3_8B, LLAMA3_LONG_PROMPTS, QWEN2_7B, QWEN_PROMPTS, ModelShape,  # noqa: F401
                             PromptShape, token_prompt)


def config_of(shape: ModelShape) -> LlamaConfig:
    return LlamaConfig(**asdict(shape))


def qwen2_7b() -> LlamaConfig:
    """Qwen2.5-7B architecture (28 layers, hidden 3584, 28 Q / 4 KV heads, q/k/v biases)."""
    return config_of(QWEN2_7B)


def llama3_8b() -> LlamaConfig:
    """Llama-3-8B architecture (32 layers, hidden 4096, 32 Q / 8 KV heads)."""
    return config_of(LLAMA3_8B)


def prompt(index: int, vocab: int, shape: PromptShape = QWEN_PROMPTS, seed: int = 1) -> StructuredPrompt:
    drawn = token_prompt(index, vocab, shape, seed)
    return StructuredPrompt(tokens=drawn.tokens,
                            document_spans=[TokenSpan(s.begin, s.end) for s in drawn.document_spans],
                            query_span=TokenSpan(drawn.query_span.begin, drawn.query_span.end))


def prompts(count: int, vocab: int, shape: PromptShape = QWEN_PROMPTS, seed: int = 1,
            first: int = 0) -> list[StructuredPrompt]:
    return [prompt(first + i, vocab, shape, seed) for i in range(count)]

"""Seeded synthetic probe prompts and the model shapes of the benchmark configurations.

numpy only: importing this module loads no native library, so the benchmark's reference arm (the
reference's own build) and the B200 arm draw the very same prompts without the reference arm
mapping this build's library. `attnrank.synthetic` wraps these into the API's types.

The reference profiles with real probe datasets (HotpotQA JSONL) or its text-level
SyntheticProbeSampleSource (attnrank/src/attnrank.cpp:96-125), both of which go through a
tokenizer. The benchmarks feed token ids directly: each prompt is k documents of uniformly random
token ids followed by a question, laid out in the reference's span order
(attnrank/src/prompt.cpp:152-171: documents, then the query span), with no instruction head or
answer tail.

Prompt i of seed s draws from numpy's PCG64 seeded with SeedSequence([s, i]), so any prompt can
be regenerated on its own and every rank of a sharded scan sees the same set.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class PromptShape:
    documents: int
    document_min: int   # inclusive
    document_max: int   # inclusive
    question: int


# 5 documents of U[120, 240] + a 40-token question (Qwen-7B scans),
# 20 documents of U[150, 250] + a 64-token question (Llama-3-8B long-context scan).
QWEN_PROMPTS = PromptShape(documents=5, document_min=120, document_max=240, question=40)
LLAMA3_LONG_PROMPTS = PromptShape(documents=20, document_min=150, document_max=250, question=64)


@dataclass(frozen=True)
class Span:
    begin: int
    end: int


@dataclass(frozen=True)
class TokenPrompt:
    """Token ids (int32) with half-open document spans and the query span."""

    tokens: np.ndarray
    document_spans: tuple
    query_span: Span


@dataclass(frozen=True)
class ModelShape:
    """The fields of a LlamaConfig that fix an architecture (include/attnrank/model.hpp:16-38)."""

    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    vocab_size: int
    max_position_embeddings: int
    rms_norm_eps: float
    rope_theta: float
    attention_bias: bool = False
    sliding_window: int = 0


# Qwen2.5-7B architecture (28 layers, hidden 3584, 28 Q / 4 KV heads, q/k/v biases)
QWEN2_7B = ModelShape(hidden_size=3584, intermediate_size=18944, num_hidden_layers=28, num_attention_heads=28,
                      num_key_value_heads=4, vocab_size=152064, max_position_embeddings=32768, rms_norm_eps=1e-6,
                      rope_theta=1e6, attention_bias=True)
# Llama-3-8B architecture (32 layers, hidden 4096, 32 Q / 8 KV heads)
LLAMA3_8B = ModelShape(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
                       num_key_value_heads=8, vocab_size=128256, max_position_embeddings=8192, rms_norm_eps=1e-5,
                       rope_theta=5e5)


def token_prompt(index: int, vocab: int, shape: PromptShape = QWEN_PROMPTS, seed: int = 1) -> TokenPrompt:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, index])))
    lengths = rng.integers(shape.document_min, shape.document_max + 1, size=shape.documents)
    total = int(lengths.sum()) + shape.question
    tokens = rng.integers(0, vocab, size=total, dtype=np.int64).astype(np.int32)
    ends = np.cumsum(lengths)
    spans = tuple(Span(int(end - length), int(end)) for end, length in zip(ends, lengths))
    return TokenPrompt(tokens=tokens, document_spans=spans, query_span=Span(int(ends[-1]), total))


def token_prompts(count: int, vocab: int, shape: PromptShape = QWEN_PROMPTS, seed: int = 1,
                  first: int = 0) -> list[TokenPrompt]:
    return [token_prompt(first + i, vocab, shape, seed) for i in range(count)]

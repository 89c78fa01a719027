"""Seeded synthetic probe prompts and model shapes of the benchmark configurations.

The reference profiles with real probe datasets (HotpotQA JSONL) or its text-level
SyntheticProbeSampleSource (attnrank.cpp:96-125), both of which go through a tokenizer. The B200
benchmarks feed token ids directly: each prompt is k documents of uniformly random token ids
followed by a question, laid out in the reference's span order (prompt.cpp:152-171: documents,
then the query span), with no instruction head or answer tail.

Prompt i of seed s draws from numpy's PCG64 seeded with SeedSequence([s, i]), so any prompt can
be regenerated on its own and every rank of a sharded scan sees the same set.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from attnrank.core import LlamaConfig, StructuredPrompt, TokenSpan


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


def qwen2_7b() -> LlamaConfig:
    """Qwen2.5-7B architecture (28 layers, hidden 3584, 28 Q / 4 KV heads, q/k/v biases)."""
    return LlamaConfig(hidden_size=3584, intermediate_size=18944, num_hidden_layers=28, num_attention_heads=28,
                       num_key_value_heads=4, vocab_size=152064, max_position_embeddings=32768, rms_norm_eps=1e-6,
                       rope_theta=1e6, attention_bias=True)


def llama3_8b() -> LlamaConfig:
    """Llama-3-8B architecture (32 layers, hidden 4096, 32 Q / 8 KV heads)."""
    return LlamaConfig(hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
                       num_key_value_heads=8, vocab_size=128256, max_position_embeddings=8192, rms_norm_eps=1e-5,
                       rope_theta=5e5)


def prompt(index: int, vocab: int, shape: PromptShape = QWEN_PROMPTS, seed: int = 1) -> StructuredPrompt:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([seed, index])))
    lengths = rng.integers(shape.document_min, shape.document_max + 1, size=shape.documents)
    total = int(lengths.sum()) + shape.question
    tokens = rng.integers(0, vocab, size=total, dtype=np.int64).astype(np.int32)
    spans, cursor = [], 0
    for length in lengths:
        spans.append(TokenSpan(cursor, cursor + int(length)))
        cursor += int(length)
    return StructuredPrompt(tokens=tokens, document_spans=spans, query_span=TokenSpan(cursor, total))


def prompts(count: int, vocab: int, shape: PromptShape = QWEN_PROMPTS, seed: int = 1,
            first: int = 0) -> list[StructuredPrompt]:
    return [prompt(first + i, vocab, shape, seed) for i in range(count)]

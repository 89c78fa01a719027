"""Generate tests/golden/reference_*.json by running the reference's own CUDA build on a B200.

The reference (attnrank/src/model.cu, kernels.cu, attnrank.cpp, compiled unmodified by
oracle/Makefile into oracle/_ref/libattnrank_ref.so) is driven through oracle/ref_harness.cpp on
the seeded synthetic checkpoint. Recorded per case: model shape, prompts (token ids and spans),
request, and the reference's measure_attention_by_layer rows / measure_attention vector.

    python tests/golden/make_reference_fixtures.py        # needs a GPU and the built oracle/_ref

Cases:
  small:  a 3-layer Qwen-shaped model (hidden 512, 4 Q / 2 KV heads, q/k/v bias), ragged prompts
          including ones longer than the 512-token prefill chunk, both normalize_by_length modes,
          a layer sub-range and the layer-averaged measure_attention;
  qwen7b: the Qwen2.5-7B architecture, two synthetic prompts of the benchmark shape.
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT / "attention-rank_b200"), str(ROOT)]

from attnrank import synthetic  # noqa: E402
from attnrank.core import LlamaConfig, StructuredPrompt, TokenSpan  # noqa: E402
from oracle import reference  # noqa: E402

OUT = Path(__file__).resolve().parent


def small_config() -> LlamaConfig:
    return LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=4,
                       num_key_value_heads=2, vocab_size=2000, max_position_embeddings=4096, rms_norm_eps=1e-6,
                       rope_theta=1e6, attention_bias=True)


def small_prompts() -> list[StructuredPrompt]:
    shapes = [synthetic.PromptShape(5, 20, 90, 12), synthetic.PromptShape(5, 120, 200, 40),
              synthetic.PromptShape(6, 150, 220, 30)]
    prompts = [synthetic.prompt(i, 2000, shapes[i % 3], seed=21) for i in range(6)]
    # a prompt whose query span is not at the end and whose last span runs past the prompt
    tokens = synthetic.prompt(99, 2000, shapes[1], seed=21).tokens
    T = len(tokens)
    prompts.append(StructuredPrompt(tokens=tokens, document_spans=[(0, 100), (100, 300), (300, 500), (500, 620),
                                                                    (620, T + 50)],
                                    query_span=TokenSpan(T - 90, T - 40)))
    return prompts


def encode(prompt: StructuredPrompt) -> dict:
    return {"tokens": [int(t) for t in prompt.tokens], "spans": [[s.begin, s.end] for s in prompt.document_spans],
            "query_span": [prompt.query_span.begin, prompt.query_span.end]}


def config_dict(config: LlamaConfig) -> dict:
    return {k: getattr(config, k) for k in ["hidden_size", "intermediate_size", "num_hidden_layers",
                                            "num_attention_heads", "num_key_value_heads", "vocab_size", "rms_norm_eps",
                                            "rope_theta", "sliding_window", "attention_bias"]}


def main() -> None:
    if reference.load_or_none() is None:
        raise SystemExit("build the reference first: make -C oracle reference")
    config = small_config()
    model = reference.ReferenceModel(config, seed=0, max_sequence_length=2048)
    cases = []
    for index, prompt in enumerate(small_prompts()):
        for normalize in (False, True):
            rows = model.measure_attention_by_layer(prompt, 0, -1, normalize)
            cases.append({"prompt": index, "layer_begin": 0, "layer_end": -1, "normalize_by_length": normalize,
                          "rows": rows.tolist()})
        rows = model.measure_attention_by_layer(prompt, 1, 3, False)
        cases.append({"prompt": index, "layer_begin": 1, "layer_end": 3, "normalize_by_length": False,
                      "rows": rows.tolist()})
        averaged = model.measure_attention(prompt, 0, 3, False)
        cases.append({"prompt": index, "measure_attention": [0, 3], "attention": averaged.tolist()})
    model.close()
    (OUT / "reference_small.json").write_text(json.dumps(
        {"seed": 0, "std": 0.02, "prefill_chunk_tokens": 512, "config": config_dict(config),
         "prompts": [encode(p) for p in small_prompts()], "cases": cases}) + "\n")

    config = synthetic.qwen2_7b()
    prompts = synthetic.prompts(2, config.vocab_size)
    model = reference.ReferenceModel(config, seed=0, max_sequence_length=2048)
    rows = [model.measure_attention_by_layer(p).tolist() for p in prompts]
    model.close()
    (OUT / "reference_qwen7b.json").write_text(json.dumps(
        {"seed": 0, "std": 0.02, "prefill_chunk_tokens": 512, "config": config_dict(config),
         "prompts": [encode(p) for p in prompts], "rows": rows}) + "\n")
    print("wrote", OUT / "reference_small.json", OUT / "reference_qwen7b.json")


if __name__ == "__main__":
    main()

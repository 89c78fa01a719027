"""The numpy-only workload generator that both benchmark arms draw from.

The reference arm must not load this build's library, so it takes its prompts and model shapes
from `probe_workloads`; the B200 arm takes them through `attnrank.synthetic`. Both must describe
the same workload, prompt for prompt, and the module must load no native library.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]


def test_both_arms_draw_the_same_prompts_and_shapes():
    import probe_workloads as PW
    from attnrank import synthetic
    for shape, count in [(PW.QWEN_PROMPTS, 25), (PW.LLAMA3_LONG_PROMPTS, 5)]:
        plain = PW.token_prompts(count, 152064, shape)
        typed = synthetic.prompts(count, 152064, shape)
        for a, b in zip(plain, typed):
            np.testing.assert_array_equal(a.tokens, b.tokens)
            assert [(s.begin, s.end) for s in a.document_spans] == [(s.begin, s.end) for s in b.document_spans]
            assert (a.query_span.begin, a.query_span.end) == (b.query_span.begin, b.query_span.end)
            assert a.query_span.begin == a.document_spans[-1].end and a.query_span.end == len(a.tokens)
            assert len(a.tokens) - a.query_span.begin == shape.question
            lengths = [s.end - s.begin for s in a.document_spans]
            assert all(shape.document_min <= n <= shape.document_max for n in lengths)
    assert synthetic.qwen2_7b().hidden_size == PW.QWEN2_7B.hidden_size == 3584
    assert synthetic.llama3_8b().num_key_value_heads == PW.LLAMA3_8B.num_key_value_heads == 8


def test_a_prompt_depends_only_on_seed_and_index():
    import probe_workloads as PW
    batch = PW.token_prompts(6, 1000, PW.QWEN_PROMPTS, seed=4)
    alone = PW.token_prompt(3, 1000, PW.QWEN_PROMPTS, seed=4)
    np.testing.assert_array_equal(batch[3].tokens, alone.tokens)
    np.testing.assert_array_equal(PW.token_prompts(2, 1000, PW.QWEN_PROMPTS, seed=4, first=3)[0].tokens, alone.tokens)
    assert not np.array_equal(PW.token_prompt(3, 1000, PW.QWEN_PROMPTS, seed=5).tokens[:40], alone.tokens[:40])


def test_the_generator_loads_no_library_of_this_build():
    probe = ("import sys; sys.path.insert(0, %r); import probe_workloads as PW; PW.token_prompts(3, 100); "
             "print('attnrank' in sys.modules, any('attnrank_b200' in str(m) for m in open('/proc/self/maps')))"
             % str(ROOT / "attention-rank_b200"))
    out = subprocess.run([sys.executable, "-c", probe], capture_output=True, text=True, check=True).stdout.split()
    assert out == ["False", "False"], out

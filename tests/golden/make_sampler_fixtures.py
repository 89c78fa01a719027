"""Generate tests/golden/sampler_fixtures.json from the reference's own samplers.

The reference's GreedySampler / NucleusSampler / make_sampler (attnrank/src/model.cpp:70-127,
compiled unmodified by oracle/Makefile into oracle/_ref/libattnrank_ref.so) run here, without a
GPU, through oracle/ref_harness.cpp:ref_sample. Each case records the sampler config, seeded
logits rows (float32, base64) and the token ids one sampler returns over the rows in order (its
generator advances between draws).

    python tests/golden/make_sampler_fixtures.py      # needs the built oracle/_ref

`ties` marks cases whose logits repeat values: there the reference's std::partial_sort order of
equal logits decides tokens, which the library reproduces (same call) and the oracle's stable
order need not.
"""
from __future__ import annotations

import base64
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path[:0] = [str(ROOT)]

from oracle import reference  # noqa: E402

OUT = Path(__file__).resolve().parent / "sampler_fixtures.json"


def rows(seed: int, count: int, vocab: int, scale: float = 1.0, quantum: float = 0.0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    values = rng.normal(0.0, scale, size=(count, vocab))
    if quantum > 0.0:
        values = np.round(values / quantum) * quantum
    return values.astype(np.float32)


def main() -> None:
    cases = []
    specs = [
        # name, temperature, top_p, top_k, seed, logits
        ("greedy", 0.0, 0.9, 0, 1234, rows(1, 4, 129)),
        ("greedy_ties", 0.0, 0.9, 0, 1234, rows(2, 4, 128, quantum=0.5)),
        ("reference_default", 0.7, 0.9, 0, 1234, rows(3, 6, 192)),
        ("no_cut", 1.0, 1.0, 0, 99, rows(4, 6, 160)),
        ("top_k_40", 0.5, 0.5, 40, 7, rows(5, 6, 192)),
        ("top_k_1", 0.8, 0.9, 1, 3, rows(6, 4, 96)),
        ("narrow_nucleus", 1.3, 0.01, 0, 11, rows(7, 4, 128)),
        ("peaked", 0.2, 0.95, 0, 2024, rows(8, 6, 160, scale=4.0)),
        ("flat", 5.0, 0.99, 0, 5, rows(9, 6, 128, scale=0.01)),
        ("many_ties", 1.0, 0.95, 0, 77, rows(10, 6, 128, quantum=0.25)),
    ]
    for name, temperature, top_p, top_k, seed, logits in specs:
        tokens = reference.sample(logits, temperature, top_p, top_k, seed)
        ties = bool(any(len(np.unique(r)) < r.size for r in logits))
        cases.append({
            "name": name, "temperature": temperature, "top_p": top_p, "top_k": top_k, "seed": seed,
            "rows": int(logits.shape[0]), "vocab": int(logits.shape[1]), "ties": ties,
            "logits_f32_b64": base64.b64encode(logits.tobytes()).decode(),
            "tokens": tokens,
        })
    OUT.write_text(json.dumps({"source": "reference model.cpp:70-127 via oracle/ref_harness.cpp:ref_sample",
                               "cases": cases}, indent=1) + "\n")
    print(f"wrote {OUT} ({len(cases)} cases)")


if __name__ == "__main__":
    main()

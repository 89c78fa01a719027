"""Generate tests/golden/host_fixtures.json from the reference's own compiled host code.

Runs the reference's AttentionProfile::from_accumulated, basin_statistics,
select_shallowest_basin_layer and resolve_position_order (attnrank/src/attnrank.cpp) through
oracle/_ref/libattnrank_ref.so (build: make -C oracle reference) on seeded random inputs and the
edge cases the reference's semantics define, and records inputs and outputs.

    python tests/golden/make_host_fixtures.py
"""
from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import reference  # noqa: E402

OUT = Path(__file__).resolve().parent / "host_fixtures.json"


def main() -> None:
    if reference.load_or_none() is None:
        raise SystemExit("build the reference first: make -C oracle reference")
    rng = np.random.default_rng(20251201)
    fixtures: dict[str, list] = {"from_accumulated": [], "basin_statistics": [], "select_shallowest": [],
                                 "resolve_position_order": []}
    for slots in [1, 2, 3, 5, 10, 20]:
        for _ in range(4):
            accumulated = rng.random(slots) * rng.integers(1, 400)
            if rng.random() < 0.3:  # ties
                accumulated[rng.integers(0, slots)] = accumulated[0]
            count = int(rng.integers(1, 400))
            attention, order = reference.from_accumulated(accumulated, count)
            fixtures["from_accumulated"].append({"accumulated": accumulated.tolist(), "sample_count": count,
                                                 "attention": attention.tolist(), "position_order": order.tolist()})
    fixtures["from_accumulated"].append({"accumulated": [0.0, 0.0, 0.0], "sample_count": 3,
                                         "attention": reference.from_accumulated([0.0] * 3, 3)[0].tolist(),
                                         "position_order": reference.from_accumulated([0.0] * 3, 3)[1].tolist()})
    edge_cases = [[0.3, 0.1, 0.1, 0.1, 0.4], [0.5, 0.5], [0.5, 0.0, 0.5], [0.0, 0.0, 0.0], [0.2, 0.2, 0.2, 0.2, 0.2]]
    for attention in edge_cases + [list(rng.dirichlet(np.ones(int(s)))) for s in rng.integers(3, 21, 30)]:
        for ratio in [1.0, 1.3, 1.5]:
            stats = reference.basin_statistics(attention, ratio)
            fixtures["basin_statistics"].append({
                "attention": list(map(float, attention)), "min_edge_ratio": ratio,
                "statistics": [float(v) if not math.isinf(v) else "inf" for v in stats]})
    for _ in range(30):
        layers = int(rng.integers(1, 33))
        slots = int(rng.integers(3, 21))
        attention = rng.dirichlet(np.ones(slots) * rng.choice([0.5, 5.0, 50.0]), size=layers)
        indices = rng.permutation(layers) + int(rng.integers(0, 4))
        ratio = float(rng.choice([1.0, 1.1, 1.3, 1.5]))
        selected = reference.select_shallowest(attention, indices, ratio)
        fixtures["select_shallowest"].append({"attention": attention.tolist(), "layers": indices.tolist(),
                                              "min_edge_ratio": ratio, "selected": int(selected)})
    for _ in range(30):
        count = int(rng.integers(0, 21))
        preferred = rng.integers(-2, count + 3, size=int(rng.integers(0, 25))).tolist()
        fixtures["resolve_position_order"].append({"preferred": preferred, "count": count,
                                                   "order": reference.resolve_position_order(preferred, count)})
    OUT.write_text(json.dumps(fixtures, indent=1) + "\n")
    print(f"wrote {OUT} ({sum(len(v) for v in fixtures.values())} cases)")


if __name__ == "__main__":
    main()

"""Restatement of the reference's host-side profile, basin and placement logic. Test infrastructure.

  from_accumulated         AttentionProfile::from_accumulated   attnrank/src/attnrank.cpp:151-169
  position_order           recompute_position_order             attnrank/src/attnrank.cpp:171-177
  basin_statistics         basin_statistics                     attnrank/src/attnrank.cpp:236-255
  select_shallowest        select_shallowest_basin_layer        attnrank/src/attnrank.cpp:257-265
  resolve_position_order   resolve_position_order               attnrank/src/attnrank.cpp:377-392
  rerank_documents         rerank_documents                     attnrank/engine.py:440-445
  lim_priority             LostInTheMiddleReranker::priority    attnrank/src/attnrank.cpp:420-431
  accumulate_rows          AttentionLayerScanner::observe       attnrank/src/attnrank.cpp:350-362
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

MINIMUM_BASIN_SLOTS = 3


def position_order(attention: Sequence[float]) -> list[int]:
    # std::stable_sort by attention descending == Python's stable sort on the negated key
    return sorted(range(len(attention)), key=lambda slot: -attention[slot])


def from_accumulated(accumulated: Sequence[float], sample_count: int) -> tuple[list[float], list[int]]:
    attention = [value / float(sample_count) for value in accumulated]
    total = 0.0
    for value in attention:
        total += value
    if total > 0.0:
        attention = [value / total for value in attention]
    return attention, position_order(attention)


@dataclass
class BasinStatistics:
    first: float = 0.0
    last: float = 0.0
    interior_mean: float = 0.0
    edge_ratio: float = 0.0
    is_basin: bool = False


def basin_statistics(attention: Sequence[float], min_edge_ratio: float) -> BasinStatistics:
    stats = BasinStatistics()
    if len(attention) < MINIMUM_BASIN_SLOTS:
        return stats
    stats.first = attention[0]
    stats.last = attention[-1]
    interior = 0.0
    for value in attention[1:-1]:
        interior += value
    stats.interior_mean = interior / float(len(attention) - 2)
    weakest = min(stats.first, stats.last)
    if stats.interior_mean > 0.0:
        stats.edge_ratio = weakest / stats.interior_mean
    else:
        stats.edge_ratio = math.inf if weakest > 0.0 else 0.0
    stats.is_basin = stats.edge_ratio >= min_edge_ratio
    return stats


def select_shallowest(profiles: Sequence[tuple[int, Sequence[float]]], min_edge_ratio: float) -> int:
    """profiles: (layer_index, attention) pairs."""
    selected = -1
    for layer, attention in profiles:
        if not basin_statistics(attention, min_edge_ratio).is_basin:
            continue
        if selected < 0 or layer < selected:
            selected = layer
    return selected


def resolve_position_order(preferred: Sequence[int], count: int) -> list[int]:
    order: list[int] = []
    taken = [False] * count
    for slot in preferred:
        if slot < 0 or slot >= count or taken[slot]:
            continue
        taken[slot] = True
        order.append(slot)
    order.extend(slot for slot in range(count) if not taken[slot])
    return order


def rerank_documents(documents_by_relevance: Sequence, position_order_: Sequence[int]) -> list:
    slots = resolve_position_order(position_order_, len(documents_by_relevance))
    placed = [None] * len(documents_by_relevance)
    for rank, document in enumerate(documents_by_relevance):
        placed[slots[rank]] = document
    return placed


def lim_priority(count: int, start_first: bool = False) -> list[int]:
    order, front, back, take_front = [], 0, count - 1, start_first
    while front <= back:
        if take_front:
            order.append(front)
            front += 1
        else:
            order.append(back)
            back -= 1
        take_front = not take_front
    return order


def accumulate_rows(rows_per_prompt: Sequence[Sequence[Sequence[float]]]) -> list[list[float]]:
    """Sum of per-prompt [layers][slots] rows, prompt by prompt, in fp64."""
    layers = len(rows_per_prompt[0])
    slots = len(rows_per_prompt[0][0])
    total = [[0.0] * slots for _ in range(layers)]
    for rows in rows_per_prompt:
        for layer in range(layers):
            for slot in range(slots):
                total[layer][slot] += rows[layer][slot]
    return total

"""Multi-GPU probe scheduler: shard prompts across ranks, one all-reduce of the mass accumulator.

The reference profiles on one GPU (README.md:17); multi-GPU use means separate processes on
dataset shards run by hand (README.md:149). Here one process per GPU holds a full weight replica,
prompts are sharded by length (longest-processing-time first, so ranks finish together), every
rank adds the unit-sum rows of its prompts into an fp32 [layers x slots] accumulator on its GPU,
and a single all-reduce (NCCL over NVLink on GPUs; gloo in the CPU tests) joins them. The sum of
per-prompt rows is order independent, so the profile equals the single-GPU scan up to fp32
rounding; profiles, the basin pick and the slot order are then computed identically on every rank.

Failure handling. Every failure surfaces on every rank as AttnRankError, the error type of the
reference's bindings (attnrank/src/bindings.cpp:134):
  * input errors (span counts, layer range) are checked on every rank before any collective, so
    all ranks reject the same input themselves;
  * before the all-reduce the ranks exchange a small header (accumulator length, layer range,
    slots, prompt count); a rank whose accumulator does not match the others' makes every rank
    raise instead of reducing buffers of different lengths;
  * each collective runs asynchronously under a host deadline (`deadline_s`): a rank that raised
    before the collective, stalls past the deadline or died leaves the others waiting at most
    that long; they then abort the process group's communicators where the backend supports it
    (NCCL) and raise.
"""
from __future__ import annotations

import datetime
import heapq
from typing import Sequence

from attnrank import core
from attnrank.data.classes import LayerScanSettings


def shard_by_length(lengths: Sequence[int], world_size: int) -> list[list[int]]:
    """Longest-processing-time assignment: prompts by descending length to the least-loaded rank
    (ties to the lowest rank). Each shard keeps ascending prompt order."""
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    heap = [(0, rank) for rank in range(world_size)]
    shards: list[list[int]] = [[] for _ in range(world_size)]
    for index in sorted(range(len(lengths)), key=lambda i: (-lengths[i], i)):
        load, rank = heapq.heappop(heap)
        shards[rank].append(index)
        heapq.heappush(heap, (load + int(lengths[index]), rank))
    return [sorted(shard) for shard in shards]


def layer_range(settings: LayerScanSettings, num_layers: int) -> tuple[int, int]:
    """The scanned layers [begin, end): a negative begin means 0 and a negative (or absent) end
    means every layer, as AttentionLayerProbeRequest::resolve_layers (attnrank/src/model.cpp:66-68)."""
    begin = 0 if settings.layer_begin < 0 else settings.layer_begin
    end = num_layers if settings.layer_end is None or settings.layer_end < 0 else settings.layer_end
    if begin >= end or end > num_layers:
        raise core.AttnRankError(f"layer range [{begin}, {end}) is outside the model's {num_layers} layers")
    return begin, end


def _dist():
    import torch.distributed as dist
    return dist if dist.is_available() and dist.is_initialized() else None


DEFAULT_DEADLINE_S = 120.0  # host deadline of one collective of a scan


class ProbeScheduler:
    """Runs one layer scan over all ranks of the default (or given) process group."""

    def __init__(self, engine, group=None, deadline_s: float = DEFAULT_DEADLINE_S):
        self.engine = engine
        self.group = group
        self.deadline_s = float(deadline_s)
        dist = _dist()
        self.rank = dist.get_rank(group) if dist else 0
        self.world_size = dist.get_world_size(group) if dist else 1

    def _bounded(self, dist, work, what: str) -> None:
        """Wait for an asynchronous collective until the deadline; on expiry or error abort the
        group's communicators (where the backend can) and raise AttnRankError."""
        try:
            work.wait(datetime.timedelta(seconds=self.deadline_s))
            if not work.is_completed():
                raise TimeoutError("not completed")
        except Exception as error:  # noqa: BLE001 - every backend failure becomes AttnRankError
            group = self.group if self.group is not None else dist.group.WORLD
            try:
                group.abort()
            except Exception:  # noqa: BLE001 - a backend without abort (gloo) just drops the collective
                pass
            raise core.AttnRankError(f"rank {self.rank}: {what} failed or missed its {self.deadline_s:g} s "
                                     f"deadline ({type(error).__name__}: {str(error)[:200]})") from error

    def _reduce(self, accumulator, header: list[int]) -> None:
        """Header check, then the one all-reduce of the accumulator, both under the deadline."""
        import torch
        dist = _dist()
        if dist is None or self.world_size <= 1:
            return
        mine = torch.tensor(header, dtype=torch.int64, device=accumulator.device)
        gathered = [torch.empty_like(mine) for _ in range(self.world_size)]
        self._bounded(dist, dist.all_gather(gathered, mine, group=self.group, async_op=True), "the scan header exchange")
        rows = [[int(v) for v in g.cpu()] for g in gathered]
        if any(row != rows[0] for row in rows):
            raise core.AttnRankError("ranks disagree on the scan (accumulator length, layer begin, layer end, slots, "
                                     f"prompts): {rows}")
        self._bounded(dist, dist.all_reduce(accumulator, op=dist.ReduceOp.SUM, group=self.group, async_op=True),
                      "the accumulator all-reduce")

    def accumulator_device(self) -> str:
        device = getattr(self.engine, "accumulator_device", None)
        return device if device is not None else f"cuda:{self.engine.device}"

    def shard(self, samples: Sequence[core.StructuredPrompt]) -> list[int]:
        return shard_by_length([len(s.tokens) for s in samples], self.world_size)[self.rank]

    def accumulate(self, samples: Sequence[core.StructuredPrompt], settings: LayerScanSettings = LayerScanSettings()):
        """Sum over all prompts of their unit-sum rows, reduced over ranks: fp64 [layers, slots]."""
        import torch

        if len(samples) == 0:
            raise core.AttnRankError("probe needs at least one sample")
        begin, end = layer_range(settings, self.engine.num_layers)
        slots = len(samples[0].document_spans)
        for index, sample in enumerate(samples):  # every rank checks every sample, before any collective
            if len(sample.document_spans) != slots:
                raise core.AttnRankError(f"probe sample {index} produced {len(sample.document_spans)} spans, "
                                         f"expected {slots}")
        accumulator = torch.zeros((end - begin) * slots, dtype=torch.float32, device=self.accumulator_device())
        if accumulator.is_cuda:
            torch.cuda.synchronize(accumulator.device)
        mine = [samples[i] for i in self.shard(samples)]
        if mine:
            self.engine.scan(mine, begin, end, settings.normalize_by_length, accumulator=accumulator)
        self._reduce(accumulator, [accumulator.numel(), begin, end, slots, len(samples)])
        return accumulator.double().cpu().numpy().reshape(end - begin, slots)

    def find_shallowest_attention_layer(self, samples: Sequence[core.StructuredPrompt],
                                        settings: LayerScanSettings = LayerScanSettings()):
        from attnrank.engine import LayerScan, MINIMUM_BASIN_SLOTS
        if len(samples) == 0:
            raise ValueError("at least one probe sample is required")
        if len(samples[0].document_spans) < MINIMUM_BASIN_SLOTS:
            raise ValueError(f"attention-basin detection needs at least {MINIMUM_BASIN_SLOTS} documents per sample")
        accumulated = self.accumulate(samples, settings)
        model_id = settings.model_id or getattr(self.engine, "model_directory", "")
        begin, _ = layer_range(settings, self.engine.num_layers)
        profiles = [core.AttentionProfile.from_accumulated(model_id, begin + layer, len(samples),
                                                           accumulated[layer])
                    for layer in range(accumulated.shape[0])]
        selected = core.select_shallowest_basin_layer(profiles, core.BasinCriterion(settings.min_edge_ratio))
        return LayerScan(selected_layer=selected, min_edge_ratio=settings.min_edge_ratio, profiles=profiles)


def find_shallowest_attention_layer_sharded(*, engine, samples: Sequence[core.StructuredPrompt],
                                            settings: LayerScanSettings = LayerScanSettings(), group=None,
                                            deadline_s: float = DEFAULT_DEADLINE_S):
    """find_shallowest_attention_layer over every rank of the process group (same result on all)."""
    return ProbeScheduler(engine, group, deadline_s).find_shallowest_attention_layer(samples, settings)

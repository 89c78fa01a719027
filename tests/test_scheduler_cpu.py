"""Multi-rank probe scheduler on CPU (gloo, world_size 2) with a host-side fake engine.

Checks the host logic of the N>1 path: length-balanced sharding, one all-reduce of the
[layers x slots] accumulator, identical profiles / basin pick on every rank, equality with the
single-process scan, and failure propagation (a rank that raises before the all-reduce makes
the others fail with an error instead of hanging).
"""
from __future__ import annotations

import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from attnrank.scheduler import ProbeScheduler, shard_by_length


class FakeEngine:
    """Deterministic stand-in for the device engine: each prompt contributes a unit-sum row per
    layer that depends on its tokens and spans."""

    accumulator_device = "cpu"
    model_directory = "fake"

    def __init__(self, layers=4, fail=False, stall_s=0.0):
        self.num_layers = layers
        self.fail = fail
        self.stall_s = stall_s

    @staticmethod
    def rows(prompt, layers):
        lengths = np.array([s.end - s.begin for s in prompt.document_spans], dtype=np.float64)
        out = []
        for layer in range(layers):
            weights = lengths * (1.0 + 0.1 * layer * np.cos(np.arange(len(lengths)) + prompt.tokens[0] % 7))
            out.append(weights / weights.sum())
        return np.array(out)

    def scan(self, prompts, layer_begin, layer_end, normalize_by_length, accumulator=None):
        if self.fail:
            raise RuntimeError("injected rank failure")
        if self.stall_s:
            __import__("time").sleep(self.stall_s)
        begin = 0 if layer_begin < 0 else layer_begin  # the engine's own range resolution
        end = self.num_layers if layer_end < 0 else layer_end
        total = sum(self.rows(p, self.num_layers)[begin:end] for p in prompts)
        accumulator += __import__("torch").from_numpy(total.reshape(-1).astype(np.float32))
        return total


def _prompts():
    from attnrank import synthetic
    shape = synthetic.PromptShape(documents=5, document_min=10, document_max=60, question=8)
    return synthetic.prompts(37, 1000, shape, seed=2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, queue, bad_spans=False, prompt_count=None, stall_rank=-1, stall_s=0.0,
            deadline_s=60.0, short_rank=-1):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "attention-rank_b200"), str(root)]
    import torch.distributed as dist

    import attnrank as ar
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        engine = FakeEngine(layers=3 if rank == short_rank else 4, fail=(rank == fail_rank),
                            stall_s=stall_s if rank == stall_rank else 0.0)
        prompts = list(_prompts())[:prompt_count]
        if bad_spans:  # one sample with a span fewer than the rest
            odd = prompts[-1]
            prompts[-1] = ar.StructuredPrompt(tokens=odd.tokens, document_spans=list(odd.document_spans)[:4],
                                              query_span=odd.query_span)
        import time
        start = time.monotonic()
        try:
            scan = ProbeScheduler(engine, deadline_s=deadline_s).find_shallowest_attention_layer(
                prompts, ar.LayerScanSettings(min_edge_ratio=0.9))
        except Exception as error:  # noqa: BLE001 - reported to the parent with the time it took
            queue.put((rank, "error", type(error).__name__, str(error)[:300], time.monotonic() - start))
            return
        queue.put((rank, "ok", scan.selected_layer, [p.attention for p in scan.profiles],
                   [p.position_order for p in scan.profiles]))
    except Exception as error:  # noqa: BLE001 - reported to the parent
        queue.put((rank, "error", type(error).__name__, str(error)[:300], None))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1, bad_spans=False, prompt_count=None, **options):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, queue, bad_spans, prompt_count),
                         kwargs=options)
             for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_shard_by_length_balances_and_covers():
    lengths = [900, 100, 500, 500, 300, 800, 50]
    shards = shard_by_length(lengths, 3)
    assert sorted(i for s in shards for i in s) == list(range(len(lengths)))
    loads = [sum(lengths[i] for i in s) for s in shards]
    assert max(loads) - min(loads) <= max(lengths)
    assert shard_by_length(lengths, 1) == [list(range(len(lengths)))]


def test_two_rank_scan_equals_single_process():
    import attnrank as ar
    single = ProbeScheduler(FakeEngine()).find_shallowest_attention_layer(_prompts(), ar.LayerScanSettings(min_edge_ratio=0.9))
    results = _run(2)
    assert all(r[1] == "ok" for r in results), results
    for _, _, selected, attention, order in results:
        assert selected == single.selected_layer
        for layer, profile in enumerate(single.profiles):
            np.testing.assert_allclose(attention[layer], profile.attention, rtol=1e-6)
            assert order[layer] == profile.position_order


def test_rank_failure_propagates_without_hanging():
    results = _run(2, fail_rank=1)
    assert results[1][1] == "error" and "injected" in results[1][3]
    assert results[0][1] == "error"  # the surviving rank's all-reduce fails instead of hanging


def test_layer_range_follows_the_reference_resolution():
    """A negative begin means layer 0 and a negative or absent end means every layer
    (model.cpp:66-68); the profiles carry the resolved layer indices."""
    import attnrank as ar
    from attnrank.scheduler import layer_range
    prompts = _prompts()
    everything = ProbeScheduler(FakeEngine()).find_shallowest_attention_layer(prompts, ar.LayerScanSettings())
    for begin, end in [(-1, None), (0, -1), (-5, -2)]:
        scan = ProbeScheduler(FakeEngine()).find_shallowest_attention_layer(
            prompts, ar.LayerScanSettings(layer_begin=begin, layer_end=end))
        assert [p.layer_index for p in scan.profiles] == [0, 1, 2, 3]
        for mine, full in zip(scan.profiles, everything.profiles):
            np.testing.assert_allclose(mine.attention, full.attention, rtol=1e-6)
    window = ProbeScheduler(FakeEngine()).find_shallowest_attention_layer(
        prompts, ar.LayerScanSettings(layer_begin=1, layer_end=3))
    assert [p.layer_index for p in window.profiles] == [1, 2]
    np.testing.assert_allclose(window.profiles[0].attention, everything.profiles[1].attention, rtol=1e-6)
    for bad in [(2, 2), (0, 9), (3, 1)]:
        with pytest.raises(ar.AttnRankError):
            layer_range(ar.LayerScanSettings(layer_begin=bad[0], layer_end=bad[1]), 4)


def test_mixed_span_counts_fail_on_every_rank_before_the_all_reduce():
    """AttentionProbeRun::run (attnrank.cpp:283-307) rejects a sample whose span count differs from
    the first one; the sharded scan checks all samples on every rank, so no rank reaches the
    collective with a mismatched accumulator."""
    import attnrank as ar
    from attnrank import core
    prompts = list(_prompts())
    odd = prompts[5]
    prompts[5] = core.StructuredPrompt(tokens=odd.tokens, document_spans=list(odd.document_spans)[:4],
                                       query_span=odd.query_span)
    with pytest.raises(ar.AttnRankError, match="probe sample 5 produced 4 spans, expected 5"):
        ProbeScheduler(FakeEngine()).find_shallowest_attention_layer(prompts, ar.LayerScanSettings())


def test_bad_input_fails_on_every_rank_before_the_collective():
    """Two gloo ranks, one sample with a missing span: both ranks raise the reference's error
    themselves (none is left waiting in the all-reduce for its peer's timeout)."""
    results = _run(2, bad_spans=True)
    for _, status, kind, message, _ in results:
        assert status == "error" and kind == "AttnRankError", results
        assert "produced 4 spans, expected 5" in message


def test_a_rank_with_no_prompts_still_joins_the_all_reduce():
    """One prompt over two ranks: rank 1's shard is empty, it adds nothing and still takes part in
    the all-reduce, so both ranks return the single-process result."""
    import attnrank as ar
    prompts = list(_prompts())[:1]
    single = ProbeScheduler(FakeEngine()).find_shallowest_attention_layer(prompts, ar.LayerScanSettings(min_edge_ratio=0.9))
    results = _run(2, prompt_count=1)
    assert all(r[1] == "ok" for r in results), results
    for _, _, selected, attention, order in results:
        assert selected == single.selected_layer
        for layer, profile in enumerate(single.profiles):
            np.testing.assert_allclose(attention[layer], profile.attention, rtol=1e-6)
            assert order[layer] == profile.position_order


def test_a_stalled_rank_makes_the_others_raise_at_the_deadline():
    """Rank 1 stalls 12 s inside its scan; rank 0 waits for it in the header exchange for its 2 s
    deadline only, then raises AttnRankError (the reference's error type, bindings.cpp:134)
    instead of waiting for the process group's 20 s timeout. Rank 1, arriving late to a group
    its peer has left, fails with an error too."""
    results = _run(2, stall_rank=1, stall_s=12.0, deadline_s=2.0)
    rank0 = results[0]
    assert rank0[1] == "error" and rank0[2] == "AttnRankError", results
    assert "deadline" in rank0[3] and rank0[4] < 10.0, rank0
    assert results[1][1] == "error", results


def test_a_rank_with_a_wrong_length_accumulator_fails_every_rank():
    """Rank 1's engine reports 3 layers instead of 4, so its accumulator is shorter: the header
    exchange before the all-reduce shows the mismatch and both ranks raise AttnRankError instead
    of reducing buffers of different lengths."""
    results = _run(2, short_rank=1)
    for _, status, kind, message, _ in results:
        assert status == "error" and kind == "AttnRankError", results
        assert "ranks disagree" in message and "[20, 0, 4, 5, 37]" in message and "[15, 0, 3, 5, 37]" in message

"""The sharded scan on two GPUs over NCCL (skipped on a box with fewer than two).

Two processes, one per GPU, each with its own engine on the same seeded synthetic checkpoint,
shard the prompts by length, scan their shards and join the [layers x slots] accumulators with one
NCCL all-reduce (attnrank.scheduler). Both ranks must return the single-GPU scan: the same pick
and slot orders, and mass rows equal up to the fp32 summation order of the accumulator (rel 1e-5).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _config():
    import attnrank as ar
    return ar.LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=4,
                          num_key_value_heads=2, vocab_size=2000, max_position_embeddings=4096, rms_norm_eps=1e-6,
                          rope_theta=1e6, attention_bias=True)


def _prompts():
    from attnrank import synthetic
    shape = synthetic.PromptShape(documents=5, document_min=20, document_max=120, question=12)
    return synthetic.prompts(29, 2000, shape, seed=13)


def _worker(rank, world, port, queue):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    sys.path[:0] = [str(root / "attention-rank_b200"), str(root)]
    import torch
    import torch.distributed as dist

    import attnrank as ar
    from attnrank.scheduler import ProbeScheduler
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(f"cuda:{rank}"))
    try:
        engine = ar.Engine.synthetic(_config(), seed=3, options=ar.RuntimeOptions(device_index=rank))
        scan = ProbeScheduler(engine, deadline_s=60).find_shallowest_attention_layer(
            _prompts(), ar.LayerScanSettings(min_edge_ratio=1.0))
        queue.put((rank, scan.selected_layer, [list(p.attention) for p in scan.profiles],
                   [list(p.position_order) for p in scan.profiles]))
        engine.close()
    except Exception as error:  # noqa: BLE001 - reported to the parent
        queue.put((rank, "error", repr(error)[:300], None))
    finally:
        dist.destroy_process_group()


def test_two_gpu_sharded_scan_equals_the_single_gpu_scan(cuda):
    import multiprocessing as mp

    import torch

    import attnrank as ar
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    engine = ar.Engine.synthetic(_config(), seed=3, options=ar.RuntimeOptions(device_index=0))
    single = ar.find_shallowest_attention_layer(engine=engine, samples=_prompts(),
                                                settings=ar.LayerScanSettings(min_edge_ratio=1.0))
    engine.close()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted((queue.get(timeout=300) for _ in procs), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for rank, selected, attention, order in results:
        assert selected != "error", attention
        assert selected == single.selected_layer
        for layer, profile in enumerate(single.profiles):
            np.testing.assert_allclose(attention[layer], profile.attention, rtol=1e-5)
            assert order[layer] == list(profile.position_order)

#!/usr/bin/env python
"""Layer-scan throughput of the attention-profiling path on B200 (prompts/s).

Workload: the Qwen2.5-7B architecture with seeded random-init weights
(bf16 values, held as fp16 -- the reference's GEMM operand type -- unless --dtype bf16), 400 seeded synthetic prompts (5 documents of U[120, 240] random token ids + a 40-token
question), a full layer scan (prefill with per-layer query->document mass capture, cross-prompt
accumulation, all-reduce, basin pick with min_edge_ratio 1.3). One step = the whole 400-prompt
scan, sharded across N GPUs (strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

`value` is device-timed (CUDA events on the engine stream, max over ranks) with every input
resident in HBM; `e2e` is the same scan through the public Python API with host prompts (H2D of
tokens and batch metadata and D2H of the accumulator inside the timed region, wall clock, max over
ranks). Inputs are larger than L2 (15 GB of weights stream through every batch), so no L2 flush
is needed between steps.

`--impl reference` times the reference's own scan (its unmodified sources compiled into
oracle/_ref: CudaLlamaModel + AttentionLayerScanner + select_shallowest_basin_layer) on the same
prompts, one GPU, and leaves its per-layer profiles in a result file; the B200 arm, run after it on
the same box, compares its own profiles, slot orders and pick against that file
(`reference_parity`). The reference arm imports nothing from this build's package.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "attention-rank_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "profiled prompts/s (7B arch, 1/2/4/8 B200); fused-kernel HBM GB/s vs peak"
MIN_EDGE_RATIO = 1.3
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# The scan workloads: BASELINE config 3 (the default bench line) and config 4.
WORKLOADS = {
    "qwen-scan": {"model": "QWEN2_7B", "shape": "QWEN_PROMPTS", "prompts": 400, "max_sequence": 4096,
                  "text": "layer scan, Qwen2.5-7B architecture, {n} prompts x (5 docs U[120,240] + 40-token question), "
                          "min_edge_ratio 1.3"},
    "llama3-long": {"model": "LLAMA3_8B", "shape": "LLAMA3_LONG_PROMPTS", "prompts": 256, "max_sequence": 8192,
                    "text": "long-context layer scan, Llama-3-8B architecture, {n} prompts x (20 docs U[150,250] + "
                            "64-token question), min_edge_ratio 1.3"},
}


def workload(args):
    """(LlamaConfig, prompts, spec) of the chosen workload, as the library's API types."""
    from attnrank import synthetic
    spec = WORKLOADS[args.config]
    config = synthetic.config_of(getattr(synthetic, spec["model"]))
    count = args.prompts if args.prompts is not None else spec["prompts"]
    prompts = synthetic.prompts(count, config.vocab_size, getattr(synthetic, spec["shape"]))
    return config, prompts, spec


def plain_workload(args):
    """The same workload from the numpy-only generator (loads no library of this build)."""
    import probe_workloads as PW
    spec = WORKLOADS[args.config]
    shape = getattr(PW, spec["model"])
    count = args.prompts if args.prompts is not None else spec["prompts"]
    return shape, PW.token_prompts(count, shape.vocab_size, getattr(PW, spec["shape"])), spec


def reference_result_path(config_name: str, prompt_count: int) -> Path:
    """Where the reference arm leaves its scan result for the B200 arm run after it on the same box."""
    import tempfile
    return Path(tempfile.gettempdir()) / f"attnrank_bench_reference_{config_name}_{prompt_count}.json"


def slot_gap(attention_rows) -> float:
    """Smallest relative gap between adjacent masses of any layer's sorted row: a mass error below
    half of it cannot reorder the slots."""
    gaps = []
    for row in attention_rows:
        ordered = sorted(row, reverse=True)
        for a, b in zip(ordered, ordered[1:]):
            gaps.append((a - b) / a if a > 0 else 0.0)
    return min(gaps) if gaps else 0.0


def parse_args():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=3)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--config", choices=sorted(WORKLOADS), default="qwen-scan",
                        help="qwen-scan: BASELINE config 3 (the bench line); llama3-long: config 4")
    parser.add_argument("--prompts", type=int, default=None, help="prompts per scan (default: the workload's)")
    parser.add_argument("--batch-tokens", type=int, default=32768,
                        help="packed tokens per batch (engine max_batch_tokens)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-kernels", action="store_true", help="skip the per-kernel roofline timing")
    parser.add_argument("--kernels-only", action="store_true",
                        help="only the per-kernel roofline timing (about 3 GB of device memory; for ncu captures)")
    parser.add_argument("--kernel-tokens", type=int, default=16384)
    parser.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16",
                        help="16-bit type of weights, GEMM operands and activations")
    parser.add_argument("--attention", choices=["tcgen05", "mma"], default="tcgen05")
    parser.add_argument("--decode", action="store_true",
                        help="decode tokens/s of greedy generation after one config-3 prompt (a separate line)")
    parser.add_argument("--decode-tokens", type=int, default=256)
    parser.add_argument("--decode-layers", type=int, default=None,
                        help="decode on the first N layers only (a small case for ncu captures; not a bench line)")
    parser.add_argument("--sweep", action="store_true",
                        help="only the fused-kernel bandwidth sweep of BASELINE config 5 (one GPU)")
    parser.add_argument("--no-sweep", action="store_true",
                        help="leave the config-5 sweep out of the N=1 bench line")
    parser.add_argument("--attention-compare", action="store_true",
                        help="only the tcgen05 attention beside torch's cuDNN and flash attention (one GPU)")
    parser.add_argument("--copy-under-cap", action="store_true",
                        help="only a plain device copy timed alone and between power-capping GEMMs (one GPU)")
    return parser.parse_args()


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.process = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.process = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.process.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.process is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.process.terminate()
        try:
            self.process.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.process.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        sm, sm_max, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(sm_max) if sm_max else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def scan_flops(config, prompts) -> float:
    """Algorithmic FLOPs of one full scan: per layer the q|k|v GEMM, causal attention and mass
    scoring (Q K^T of the query rows over the document-span keys); o_proj and the MLP on every
    layer but the last (whose outputs no probe reads)."""
    H, I, L = config.hidden_size, config.intermediate_size, config.num_hidden_layers
    Hq, Hkv, D = config.num_attention_heads, config.num_key_value_heads, config.head_dim
    qkv_per_token = 2 * H * (Hq + 2 * Hkv) * D
    rest_per_token = 2 * (Hq * D * H + 3 * H * I)
    total = 0.0
    for p in prompts:
        T = len(p.tokens)
        Tq = p.query_span.end - p.query_span.begin
        span_keys = sum(d.end - d.begin for d in p.document_spans)
        attention = 2 * Hq * D * T * (T + 1)          # QK^T and PV over the causal half
        mass = 2 * Hq * Tq * span_keys * D
        total += L * (qkv_per_token * T + attention + mass) + (L - 1) * rest_per_token * T
    return total


def init_distributed(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    torch.cuda.set_device(local_rank)
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        # NCCL's own log lines (its version banner included) go to stderr: stdout carries the JSON line
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device(f"cuda:{local_rank}"))
    return rank, world, local_rank


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_over_ranks(values: list[float], world: int) -> list[list[float]]:
    """Every rank's list of floats, in rank order (one all-gather)."""
    if world == 1:
        return [list(values)]
    import torch
    import torch.distributed as dist
    mine = torch.tensor(values, dtype=torch.float64, device="cuda")
    gathered = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(gathered, mine)
    return [[float(v) for v in g.cpu()] for g in gathered]


def barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ---------------------------------------------------------------------------------------------
# per-kernel roofline timing (live, CUDA events, on the engine's kernels through the C ABI)
# ---------------------------------------------------------------------------------------------
def kernel_rooflines(config, hbm_peak, tensor_peak, tokens: int = 16384, repeats: int = 20,
                     dtype: str = "fp16") -> dict:
    """Each kernel timed alone (CUDA events over `repeats` back-to-back launches, 3 warm-up
    launches) on a 16K-token batch; work per launch is the algorithmic HBM bytes or FLOPs."""
    import ctypes

    import torch
    from attnrank import _native

    half = torch.float16 if dtype == "fp16" else torch.bfloat16
    code = _native.DTYPE_F16 if dtype == "fp16" else _native.DTYPE_BF16

    lib = _native.lib
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream()
    s = ctypes.c_void_p(stream.cuda_stream)
    H, I, Hq, Hkv, D, V = (config.hidden_size, config.intermediate_size, config.num_attention_heads,
                           config.num_key_value_heads, config.head_dim, config.vocab_size)
    W = (Hq + 2 * Hkv) * D
    gen = torch.Generator(device=dev).manual_seed(0)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    results = {}

    def timed(name, launch, bytes_moved=None, flops=None):
        for _ in range(3):
            launch()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(repeats):
            launch()
        stop.record(stream)
        stop.synchronize()
        seconds = start.elapsed_time(stop) / 1000 / repeats
        entry = {"us_per_launch": round(seconds * 1e6, 2)}
        if bytes_moved is not None:
            achieved = bytes_moved / seconds / 1e9
            entry.update({"bound": "hbm", "algorithmic_bytes": int(bytes_moved), "achieved": round(achieved, 1),
                          "unit": "GB/s", "frac": round(achieved / hbm_peak, 4)})
        if flops is not None:
            achieved = flops / seconds / 1e12
            entry.update({"bound": "tensor", "algorithmic_flops": int(flops), "achieved": round(achieved, 1),
                          "unit": "TFLOP/s", "frac": round(achieved / tensor_peak, 4)})
        results[name] = entry

    residual = torch.randn(tokens, H, device=dev, generator=gen)
    delta = torch.randn(tokens, H, device=dev, generator=gen).to(half)
    gamma = torch.ones(H, device=dev)
    normed = torch.empty(tokens, H, device=dev, dtype=half)
    timed("rms_norm_residual", lambda: _native.check(lib.ar_rms_norm_residual(
        P(residual), P(delta), P(gamma), tokens, H, 1e-6, P(normed), code, s)), bytes_moved=12 * tokens * H + 4 * H)

    table = (torch.randn(V, H, device=dev, generator=gen) * 0.02).to(half)
    ids = torch.randint(0, V, (tokens,), device=dev, dtype=torch.int32, generator=gen)
    timed("embedding_rms_norm", lambda: _native.check(lib.ar_embedding_rms_norm(
        P(ids), tokens, P(table), V, H, P(gamma), 1e-6, P(residual), P(normed), None, code, s)),
        bytes_moved=tokens * (2 * H + 4 * H + 2 * H + 4))
    del table

    qkv = torch.randn(tokens, W, device=dev, generator=gen).to(half)
    bias = torch.zeros(W, device=dev)
    cos = torch.empty(8192, D // 2, device=dev)
    sin = torch.empty_like(cos)
    _native.check(lib.ar_rope_table(P(cos), P(sin), 8192, D, config.rope_theta, s))
    positions = (torch.arange(tokens, device=dev, dtype=torch.int32) % 940).contiguous()
    timed("rotary_bias", lambda: _native.check(lib.ar_rotary_embedding(
        P(qkv), P(bias), P(positions), tokens, Hq, Hkv, D, P(cos), P(sin), 8192, None, code, s)),
        bytes_moved=4 * tokens * W)

    gate_up = torch.randn(tokens, 2 * I, device=dev, generator=gen).to(half)
    act = torch.empty(tokens, I, device=dev, dtype=half)
    timed("silu_multiply", lambda: _native.check(lib.ar_silu_multiply(
        P(gate_up), ctypes.c_void_p(gate_up.data_ptr() + 2 * I), 2 * I, P(act), I, tokens, I, code, s)),
        bytes_moved=6 * tokens * I)
    del gate_up, act

    # attention + mass on 17 prompts of 940 tokens (a 16K-token batch of the scan)
    from attnrank import synthetic
    prompts = synthetic.prompts(17, V)
    lengths = [len(p.tokens) for p in prompts]
    import numpy as np
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    total = int(offsets[-1])
    qkv2 = (torch.randn(total, W, device=dev, generator=gen)).to(half)
    out = torch.empty(total, Hq * D, device=dev, dtype=half)
    lse = torch.empty(total, Hq, device=dev)
    offsets_d = torch.from_numpy(offsets).to(dev)
    attention_flops = sum(2 * Hq * D * T * (T + 1) for T in lengths)
    timed("causal_attention_mma (incl. host tile list + sync)", lambda: _native.check(lib.ar_causal_attention_mma(
        P(qkv2), P(out), P(lse), offsets.ctypes.data, P(offsets_d), len(lengths), Hq, Hkv, D, 0, code, s)),
        flops=attention_flops)
    timed("causal_attention (incl. host tile list + sync)", lambda: _native.check(lib.ar_causal_attention(
        P(qkv2), P(out), P(lse), offsets.ctypes.data, P(offsets_d), len(lengths), Hq, Hkv, D, 0, code, s)),
        flops=attention_flops)
    qs = np.ascontiguousarray(np.array([(p.query_span.begin, p.query_span.end) for p in prompts], np.int32).reshape(-1))
    sp = np.ascontiguousarray(np.array([[(d.begin, d.end) for d in p.document_spans] for p in prompts],
                                       np.int32).reshape(-1))
    mass = np.zeros((len(prompts), 5))
    mass_flops = sum(2 * Hq * (p.query_span.end - p.query_span.begin) * p.document_spans[-1].end * D for p in prompts)
    timed("document_mass (incl. host planning + sync)", lambda: _native.check(lib.ar_document_attention_mass(
        P(qkv2), total, P(lse), offsets.ctypes.data, len(prompts), qs.ctypes.data, sp.ctypes.data, 5, Hq, Hkv, D, 0,
        512, 0, mass.ctypes.data, code, s)), flops=mass_flops)
    # 4.6 GFLOP is a few µs of tensor work: this synchronous call (host planning, metadata upload,
    # the mass kernel and its finaliser, read-back of the doubles) is latency, not a roofline
    entry = results["document_mass (incl. host planning + sync)"]
    entry.update({"bound": "latency: one synchronous C-ABI call", "frac": None})
    torch.cuda.synchronize()
    return results


def attention_comparison(tensor_peak: float, dtype: str = "fp16", repeats: int = 20) -> list[dict]:
    """This build's tcgen05 attention beside the attention kernels shipped with torch (cuDNN's and
    the flash backend of scaled_dot_product_attention) on equal-length causal batches of the scan's
    two shapes: 17 prompts of 940 tokens with 28/4 heads (config 3) and 4 of 4096 with 32/8 heads
    (config 4). Same inputs for all; FLOPs count the causal triangle, 2·Hq·D·T(T+1) per prompt. The
    build's figure goes through the C ABI (host tile list and a sync inside every call); the
    libraries' are back-to-back launches. Output difference against cuDNN is reported beside it."""
    import ctypes

    import numpy as np
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from attnrank import _native

    half = torch.float16 if dtype == "fp16" else torch.bfloat16
    code = _native.DTYPE_F16 if dtype == "fp16" else _native.DTYPE_BF16
    lib = _native.lib
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream()
    s = ctypes.c_void_p(stream.cuda_stream)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    gen = torch.Generator(device=dev).manual_seed(1)

    def time_it(launch) -> float:
        for _ in range(3):
            launch()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(repeats):
            launch()
        stop.record(stream)
        stop.synchronize()
        return start.elapsed_time(stop) / 1000 / repeats

    rows = []
    for name, B, T, Hq, Hkv in [("config 3 shape", 17, 940, 28, 4), ("config 4 shape", 4, 4096, 32, 8)]:
        D = 128
        W = (Hq + 2 * Hkv) * D
        flops = B * 2 * Hq * D * T * (T + 1)
        qkv = torch.randn(B * T, W, device=dev, generator=gen).to(half)
        out = torch.empty(B * T, Hq * D, device=dev, dtype=half)
        lse = torch.empty(B * T, Hq, device=dev)
        offsets = (np.arange(B + 1) * T).astype(np.int32)
        offsets_d = torch.from_numpy(offsets).to(dev)
        entry = {"case": name, "prompts": B, "tokens_per_prompt": T, "heads": f"{Hq}/{Hkv}",
                 "gflop": round(flops / 1e9, 1)}

        def ours():
            _native.check(lib.ar_causal_attention(P(qkv), P(out), P(lse), offsets.ctypes.data, P(offsets_d), B, Hq,
                                                  Hkv, D, 0, code, s))
        seconds = time_it(ours)
        entry["this_build_tcgen05"] = {"us": round(seconds * 1e6, 1), "tflops": round(flops / seconds / 1e12, 1),
                                       "frac": round(flops / seconds / 1e12 / tensor_peak, 4)}
        view = qkv.view(B, T, Hq + 2 * Hkv, D)
        q = view[:, :, :Hq].transpose(1, 2)
        k = view[:, :, Hq:Hq + Hkv].transpose(1, 2).repeat_interleave(Hq // Hkv, dim=1)
        v = view[:, :, Hq + Hkv:].transpose(1, 2).repeat_interleave(Hq // Hkv, dim=1)
        mine = out.view(B, T, Hq, D).transpose(1, 2).float()
        for label, backend in [("torch_sdpa_cudnn", SDPBackend.CUDNN_ATTENTION),
                               ("torch_sdpa_flash", SDPBackend.FLASH_ATTENTION)]:
            try:
                with sdpa_kernel([backend]):
                    seconds = time_it(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
                    reference = F.scaled_dot_product_attention(q, k, v, is_causal=True)
                torch.cuda.synchronize()
                entry[label] = {"us": round(seconds * 1e6, 1), "tflops": round(flops / seconds / 1e12, 1),
                                "frac": round(flops / seconds / 1e12 / tensor_peak, 4),
                                "max_abs_diff_vs_this_build": float((reference.float() - mine).abs().max())}
                del reference
            except Exception as error:  # noqa: BLE001 - a backend this torch build lacks is reported
                entry[label] = {"unavailable": repr(error)[:200]}
        rows.append(entry)
        del qkv, out, lse, q, k, v, view, mine
        torch.cuda.empty_cache()
    return rows


def copy_under_power_cap(local_rank: int) -> dict:
    """A plain 1 GiB device copy (torch, CUDA events) timed alone, then between bursts of 8192^3
    bf16 GEMMs that hold the GPU at its power-capped clock, as the scan's GEMMs do: how much of
    the HBM-bound kernels' in-scan slowdown the memory path itself shows at that clock."""
    import torch

    stream = torch.cuda.current_stream()
    a = torch.randn(1 << 29, device="cuda", dtype=torch.bfloat16)
    b = torch.empty_like(a)
    x = torch.randn(8192, 8192, device="cuda", dtype=torch.bfloat16)
    y = torch.randn(8192, 8192, device="cuda", dtype=torch.bfloat16)
    z = torch.empty_like(x)

    def copy_gbs(repeats: int) -> float:
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(repeats):
            b.copy_(a)
        stop.record(stream)
        stop.synchronize()
        return 2 * a.numel() * a.element_size() * repeats / (start.elapsed_time(stop) / 1000) / 1e9

    for _ in range(3):
        copy_gbs(3)
    sampler = ClockSampler(local_rank)
    sampler.start()
    alone = [copy_gbs(10) for _ in range(60)]  # about 0.2 s: long enough for a clock sample
    clocks_alone = sampler.stop()
    for _ in range(200):  # about 3 s of GEMMs: the power limiter settles
        torch.matmul(x, y, out=z)
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.start()
    capped = []
    for _ in range(10):
        for _ in range(20):
            torch.matmul(x, y, out=z)
        capped.append(copy_gbs(2))
    clocks_capped = sampler.stop()
    return {"copy_alone_gbs": round(statistics.median(alone), 1), "clocks_alone": clocks_alone,
            "copy_between_gemms_gbs": round(statistics.median(capped), 1), "clocks_between_gemms": clocks_capped,
            "ratio": round(statistics.median(capped) / statistics.median(alone), 3)}


SWEEP_TOKENS = (1, 64, 1024, 8192, 32768)
SWEEP_HIDDEN = (2048, 3584, 4096, 8192)
SWEEP_KV_HEADS = {2048: 4, 3584: 4, 4096: 8, 8192: 8}


def bandwidth_sweep(hbm_peak: float, dtype: str = "fp16", repeats: int = 20) -> list[dict]:
    """the fused elementwise kernels over tokens x hidden (head_dim 128,
    intermediate 3.5 x hidden, vocab 152064), N(0,1) activations, N(0,0.02) table, each timed alone
    with CUDA events (3 warm-up + `repeats` launches) against its algorithmic HBM bytes. Small
    sizes fit in L2 and are launch-bound; the large ones measure HBM."""
    import ctypes

    import torch
    from attnrank import _native

    lib = _native.lib
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream()
    s = ctypes.c_void_p(stream.cuda_stream)
    half = torch.float16 if dtype == "fp16" else torch.bfloat16
    code = _native.DTYPE_F16 if dtype == "fp16" else _native.DTYPE_BF16
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    gen = torch.Generator(device=dev).manual_seed(5)
    vocab, D = 152064, 128
    rows = []

    def timed(kernel, tokens, hidden, launch, bytes_moved):
        for _ in range(3):
            launch()
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(repeats):
            launch()
        stop.record(stream)
        stop.synchronize()
        seconds = start.elapsed_time(stop) / 1000 / repeats
        achieved = bytes_moved / seconds / 1e9
        rows.append({"kernel": kernel, "tokens": tokens, "hidden": hidden, "us": round(seconds * 1e6, 2),
                     "bytes": int(bytes_moved), "gbs": round(achieved, 1), "frac": round(achieved / hbm_peak, 4)})

    cos = torch.empty(32768, D // 2, device=dev)
    sin = torch.empty_like(cos)
    _native.check(lib.ar_rope_table(P(cos), P(sin), 32768, D, 1e6, s))
    for hidden in SWEEP_HIDDEN:
        intermediate = int(hidden * 3.5)
        heads, kv_heads = hidden // D, SWEEP_KV_HEADS[hidden]
        width = (heads + 2 * kv_heads) * D
        gamma = torch.ones(hidden, device=dev)
        table = (torch.randn(vocab, hidden, device=dev, generator=gen) * 0.02).to(half)
        bias = (torch.randn(width, device=dev, generator=gen) * 0.02)
        for tokens in SWEEP_TOKENS:
            residual = torch.randn(tokens, hidden, device=dev, generator=gen)
            delta = torch.randn(tokens, hidden, device=dev, generator=gen).to(half)
            normed = torch.empty(tokens, hidden, device=dev, dtype=half)
            timed("rms_norm_residual", tokens, hidden, lambda: _native.check(lib.ar_rms_norm_residual(
                P(residual), P(delta), P(gamma), tokens, hidden, 1e-6, P(normed), code, s)),
                12 * tokens * hidden + 4 * hidden)
            ids = torch.randint(0, vocab, (tokens,), device=dev, dtype=torch.int32, generator=gen)
            timed("embedding_rms_norm", tokens, hidden, lambda: _native.check(lib.ar_embedding_rms_norm(
                P(ids), tokens, P(table), vocab, hidden, P(gamma), 1e-6, P(residual), P(normed), None, code, s)),
                tokens * (8 * hidden + 4))
            del residual, delta, normed, ids
            qkv = torch.randn(tokens, width, device=dev, generator=gen).to(half)
            positions = (torch.arange(tokens, device=dev, dtype=torch.int32) % 32768).contiguous()
            timed("rotary_bias", tokens, hidden, lambda: _native.check(lib.ar_rotary_embedding(
                P(qkv), P(bias), P(positions), tokens, heads, kv_heads, D, P(cos), P(sin), 32768, None, code, s)),
                4 * tokens * width)
            del qkv, positions
            gate_up = torch.randn(tokens, 2 * intermediate, device=dev, generator=gen).to(half)
            act = torch.empty(tokens, intermediate, device=dev, dtype=half)
            timed("silu_multiply", tokens, hidden, lambda: _native.check(lib.ar_silu_multiply(
                P(gate_up), ctypes.c_void_p(gate_up.data_ptr() + 2 * intermediate), 2 * intermediate, P(act),
                intermediate, tokens, intermediate, code, s)), 6 * tokens * intermediate)
            del gate_up, act
        del table
        torch.cuda.empty_cache()
    return rows


def cpu_baseline(config, prompt, layers: int = 4) -> dict:
    """The oracle port (fp32 torch on the host cores) on a bounded sample: one prompt through the
    first `layers` layers, scaled to the full depth."""
    import torch
    from oracle import forward as F
    from oracle import weights as W
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    W.set_threads(cores)
    shape = F.Shape(hidden=config.hidden_size, intermediate=config.intermediate_size, layers=layers,
                    heads=config.num_attention_heads, kv_heads=config.num_key_value_heads, vocab=config.vocab_size,
                    eps=config.rms_norm_eps, theta=config.rope_theta, bias=config.attention_bias)
    model = F.OracleModel(shape, seed=0)
    sample = F.Prompt(tokens=prompt.tokens, query_span=(prompt.query_span.begin, prompt.query_span.end),
                      spans=[(s.begin, s.end) for s in prompt.document_spans])
    model.prepare([sample])  # weights and embedding rows are generated before the clock starts
    start = time.perf_counter()
    model.probe([sample])
    seconds = (time.perf_counter() - start) * config.num_hidden_layers / layers
    # BASELINE config 1 in full: a TinyLlama-1.1B-shaped single layer, 256 tokens, 16 query
    # tokens over 5 document spans of 48 tokens
    tiny = F.Shape(hidden=2048, intermediate=5632, layers=1, heads=32, kv_heads=4, vocab=32000, eps=1e-5,
                   theta=1e4)
    import numpy as np
    tokens = np.random.default_rng(0).integers(0, 32000, 256).astype(np.int32)
    c1 = F.Prompt(tokens=tokens, query_span=(240, 256), spans=[(48 * i, 48 * i + 48) for i in range(5)])
    tiny_model = F.OracleModel(tiny, seed=0)
    tiny_model.prepare([c1])
    start = time.perf_counter()
    tiny_model.probe([c1])
    c1_seconds = time.perf_counter() - start
    return {"value": round(1.0 / seconds, 5), "unit": "prompts/s", "cores": cores, "kind": "port",
            "sample": f"1 prompt ({len(prompt.tokens)} tokens) x {layers} of {config.num_hidden_layers} layers, "
                      f"fp32 torch-CPU oracle, forward pass only (weights generated before the clock), "
                      f"scaled to all layers",
            "config1_seconds": round(c1_seconds, 4),
            "config1": "TinyLlama-1.1B-shaped single layer, 256 tokens, mass of 16 query tokens over 5 spans "
                       "of 48 (forward pass only)"}


# ---------------------------------------------------------------------------------------------
def run_b200(args, rank, world, local_rank):
    import numpy as np
    import torch

    import attnrank as ar
    from attnrank import synthetic
    from attnrank.scheduler import ProbeScheduler, shard_by_length

    config, prompts, spec = workload(args)
    prompt_count = len(prompts)
    options = ar.RuntimeOptions(device_index=local_rank, max_sequence_length=spec["max_sequence"],
                                max_batch_tokens=args.batch_tokens,
                                activation_dtype=args.dtype, attention_kernel=args.attention)
    engine = ar.Engine.synthetic(config, seed=0, options=options)
    shard = shard_by_length([len(p.tokens) for p in prompts], world)[rank]
    mine = [prompts[i] for i in shard]
    slots = len(prompts[0].document_spans)
    L = config.num_hidden_layers
    prepared = engine.prepare_scan(mine)
    accumulator = torch.zeros(L * slots, dtype=torch.float32, device=f"cuda:{local_rank}")
    torch.cuda.synchronize()
    engine_stream = torch.cuda.ExternalStream(engine.stream, device=f"cuda:{local_rank}")

    marks = []  # per timed step: events before the scan, after it and after the all-reduce

    def step(record=False):
        with torch.cuda.stream(engine_stream):
            events = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if record else None
            accumulator.zero_()
            if record:
                events[0].record(engine_stream)
            prepared.run(accumulator, synchronize=False)
            if record:
                events[1].record(engine_stream)
            if world > 1:
                import torch.distributed as dist
                dist.all_reduce(accumulator)
            if record:
                events[2].record(engine_stream)
                marks.append(events)

    for _ in range(args.warmup):
        step()
    engine.synchronize()
    barrier(world)
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.3)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(engine_stream)
    for _ in range(args.steps):
        step(record=True)
    stop.record(engine_stream)
    stop.synchronize()
    clocks = sampler.stop()
    engine.synchronize()  # raises on any device-reported error
    elapsed_ms = max_over_ranks(start.elapsed_time(stop), world)
    ms_per_step = elapsed_ms / args.steps
    value = prompt_count / (ms_per_step / 1000.0)
    # per rank: mean scan time and all-reduce time of the timed steps; min / max over ranks
    scan_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in marks)
    reduce_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in marks)
    per_rank = gather_over_ranks([scan_ms, reduce_ms, float(sum(len(p.tokens) for p in mine)), float(len(mine))],
                                 world)

    # one more (untimed) step with every engine launch bracketed by CUDA events: per-kernel
    # device time and algorithmic work inside the real scan, and the count of our own launches
    engine.set_kernel_timing(True)
    step()
    timing = engine.kernel_timing()
    engine.set_kernel_timing(False)

    # the scan result of the timed steps: accumulator of the last step -> profiles, basin pick
    accumulated = accumulator.double().cpu().numpy().reshape(L, slots)
    profiles = [ar.AttentionProfile.from_accumulated("synthetic", l, prompt_count, accumulated[l]) for l in range(L)]
    selected = ar.select_shallowest_basin_layer(profiles=profiles, min_edge_ratio=MIN_EDGE_RATIO)
    ratios = [ar.basin_statistics(attention=p.attention, min_edge_ratio=MIN_EDGE_RATIO).edge_ratio for p in profiles]
    highest = profiles[max(range(L), key=lambda i: ratios[i])].layer_index
    profile_record = {"layer_index": [p.layer_index for p in profiles],
                      "attention": [[float(v) for v in p.attention] for p in profiles],
                      "position_order": [[int(v) for v in p.position_order] for p in profiles],
                      "edge_ratio": [float(r) for r in ratios]}
    parity = reference_parity(args.config, prompt_count, profile_record, selected, highest)

    # end to end through the public API (host prompts in, H2D + D2H inside the timed region)
    scheduler = ProbeScheduler(engine)
    settings = ar.LayerScanSettings(min_edge_ratio=MIN_EDGE_RATIO)
    scheduler.find_shallowest_attention_layer(prompts, settings)  # warm-up
    e2e_seconds = []
    for _ in range(max(1, args.steps)):
        barrier(world)
        t0 = time.perf_counter()
        scan = scheduler.find_shallowest_attention_layer(prompts, settings)
        e2e_seconds.append(time.perf_counter() - t0)
    e2e_step = max_over_ranks(statistics.median(e2e_seconds), world)
    tokens_mine = sum(len(p.tokens) for p in mine)
    h2d = 4 * (tokens_mine + 6 * len(mine) + 2 * slots * len(mine)) + 8 * sum(
        (len(p.tokens) + 127) // 128 for p in mine)
    d2h = 4 * L * slots + 4

    peak, peak_kind = peaks()
    flops = scan_flops(config, prompts)
    achieved_tflops = flops / (ms_per_step / 1000.0) / 1e12
    tensor_peak = peak.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    job_peak = tensor_peak * world  # the whole job's FLOPs against the peak of all its GPUs
    hbm_peak = peak.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    timed_ms = sum(entry["ms"] for entry in timing.values()) or 1.0
    kernels = {}
    for name, entry in timing.items():
        if entry["launches"] == 0:
            continue
        seconds = entry["ms"] / 1000.0
        library = name.startswith("gemm_")
        record = {"launches_per_step": entry["launches"],
                  "us_per_launch": round(entry["ms"] * 1000.0 / entry["launches"], 2),
                  "share_of_step": round(entry["ms"] / timed_ms, 4), "library": library}
        if entry["tensor"]:
            achieved = entry["work"] / seconds / 1e12 if seconds > 0 else 0.0
            record.update({"bound": "tensor", "achieved": round(achieved, 1), "unit": "TFLOP/s",
                           "frac": round(achieved / tensor_peak, 4)})
        else:
            achieved = entry["work"] / seconds / 1e9 if seconds > 0 else 0.0
            record.update({"bound": "hbm", "achieved": round(achieved, 1), "unit": "GB/s",
                           "frac": round(achieved / hbm_peak, 4)})
        kernels[name] = record
    own_launches_per_step = sum(entry["launches"] for name, entry in timing.items() if not name.startswith("gemm_"))
    gpu_launches = args.steps * own_launches_per_step
    dominant = max((n for n in kernels), key=lambda n: kernels[n]["share_of_step"])
    result = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "prompts/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": args.dtype,
        "data": "synthetic (seeded random-init weights: bf16 values, stored in the compute dtype; seeded random "
                "token-id prompts)",
        "config": {"workload": spec["text"].format(n=prompt_count), "global_batch": prompt_count,
                   "seq_len": round(sum(len(p.tokens) for p in prompts) / len(prompts), 1),
                   "parallelism": f"dp{world} (prompt shards, one NCCL all-reduce)",
                   "batch_tokens": args.batch_tokens,
                   "l2": "inputs larger than L2 (15-16 GB of weights streamed per batch); no flush"},
        "selected_layer": selected,
        "slot_order_selected": profiles[selected].position_order if selected >= 0 else None,
        "highest_ratio_layer": highest,
        "profiles": profile_record,
        "reference_parity": parity,
        "e2e": {"value": round(prompt_count / e2e_step, 3), "unit": "prompts/s", "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "selected_layer": scan.selected_layer,
                "api": "attnrank.scheduler.ProbeScheduler.find_shallowest_attention_layer"},
        "roofline": {"bound": "tensor", "kernel": "whole scan step (cuBLASLt GEMMs + attention + mass)",
                     "dominant_kernel": dominant,
                     "achieved": round(achieved_tflops, 1), "peak": round(job_peak, 1), "unit": "TFLOP/s",
                     "frac": round(achieved_tflops / job_peak, 4), "traffic": None,
                     "peak_source": f"{peak_kind} bf16_tflops_sustained x {world} GPU(s)",
                     "algorithmic_flops_per_step": flops},
        "clocks": clocks,
        "ranks": {"scan_ms": {"min": round(min(r[0] for r in per_rank), 3), "max": round(max(r[0] for r in per_rank), 3)},
                  "allreduce_ms": {"min": round(min(r[1] for r in per_rank), 4),
                                   "max": round(max(r[1] for r in per_rank), 4)},
                  "tokens": [int(r[2]) for r in per_rank], "prompts": [int(r[3]) for r in per_rank],
                  "note": "per rank: mean over the timed steps of the scan and of the all-reduce (CUDA events "
                          "on the engine stream)"},
        "gpu_launches": gpu_launches,
        "attention_kernel": args.attention,
        "kernels": kernels,
        "kernels_peak_source": f"{peak_kind}: hbm_gbs for HBM-bound, bf16_tflops_sustained for tensor-bound; "
                               "CUDA events around every launch on the engine stream during one extra step",
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_baseline(config, prompts[0])
    if rank == 0 and not args.no_kernels:
        # The scan holds the GPU at its power-capped clock (about 1.3 GHz) and the power limiter
        # takes a while to release it; "alone" means at the clock these kernels set by themselves,
        # so the GPU idles first (the CPU baseline above already gave it that time at N=1), and
        # the SM clock seen during the timing is reported beside the figures.
        torch.cuda.synchronize()
        time.sleep(0 if "cpu_baseline" in result else 3)
        isolated_clock = ClockSampler(local_rank)
        isolated_clock.start()
        result["kernels_isolated"] = kernel_rooflines(config, hbm_peak, peak.get("bf16_tflops",
                                                                                 FALLBACK_PEAKS["bf16_tflops"]),
                                                      dtype=args.dtype)
        result["kernels_isolated_peak_source"] = f"{peak_kind} hbm_gbs / bf16_tflops (burst)"
        result["kernels_isolated_clocks"] = isolated_clock.stop()
    del prepared
    engine.close()
    if rank == 0 and world == 1 and not args.no_sweep:
        torch.cuda.empty_cache()
        result["sweep"] = {"rows": bandwidth_sweep(hbm_peak, dtype=args.dtype), "peak_source": f"{peak_kind} hbm_gbs",
                           "config": "BASELINE config 5: tokens {1,64,1024,8192,32768} x hidden {2048,3584,4096,8192}, "
                                     "head_dim 128, intermediate 3.5 x hidden, vocab 152064; each kernel timed alone "
                                     "(CUDA events, 3 warm-up + 20 launches)"}
    return result


def reference_parity(config_name: str, prompt_count: int, profiles: dict, selected: int, highest: int) -> dict:
    """This arm's scan result against the reference arm's, when the reference arm ran before this one
    on the same box with the same workload (its result file): the largest relative mass error, slot
    orders of every layer, the basin pick, the highest-ratio layer, and the smallest relative gap
    between adjacent masses (an error below half of it cannot flip an order)."""
    path = reference_result_path(config_name, prompt_count)
    if not path.exists():
        return {"available": False, "reason": f"no reference result for this workload ({path.name}); run "
                                              "bench.py --impl reference first on this box"}
    want = json.loads(path.read_text())
    theirs = want["profiles"]
    if want.get("prompts") != prompt_count or theirs["layer_index"] != profiles["layer_index"]:
        return {"available": False, "reason": "the reference result covers another workload"}
    worst = 0.0
    for mine, ref in zip(profiles["attention"], theirs["attention"]):
        for a, b in zip(mine, ref):
            worst = max(worst, abs(a - b) / max(abs(b), 1e-12))
    orders_equal = [a == b for a, b in zip(profiles["position_order"], theirs["position_order"])]
    return {"available": True, "prompts": prompt_count, "layers": len(orders_equal),
            "max_rel_err_vs_reference": worst, "mass_tolerance": 1e-3,
            "slot_orders_equal": all(orders_equal), "layers_with_equal_order": sum(orders_equal),
            "selected_layer_equal": selected == want["selected_layer"], "reference_selected_layer":
                want["selected_layer"],
            "highest_ratio_layer_equal": highest == want["highest_ratio_layer"],
            "min_adjacent_slot_gap_rel": slot_gap(theirs["attention"])}


def run_reference(args, rank, world, local_rank):
    """The reference's own scan (CudaLlamaModel + AttentionLayerScanner + select_shallowest_basin_layer,
    compiled from its unmodified sources into oracle/_ref) on the same prompts as the B200 arm. It
    imports nothing from this build's package: the prompts come from the numpy-only generator."""
    from oracle import reference

    if reference.load_or_none() is None:
        return {"impl": "reference", "unavailable": "oracle/_ref/libattnrank_ref.so was not built (make -C oracle reference)"}
    shape, prompts, spec = plain_workload(args)
    count = len(prompts)
    longest = max(len(p.tokens) for p in prompts)
    model = reference.ReferenceModel(shape, seed=0, max_sequence_length=max(2048, longest), device=local_rank)
    for _ in range(args.warmup):  # warm-up on a slice: the reference's first calls set up cuBLAS
        model.scan(prompts[:8], min_edge_ratio=MIN_EDGE_RATIO)
    seconds = []
    result = None
    sampler = ClockSampler(local_rank)
    sampler.start()
    for _ in range(args.steps):
        result = model.scan(prompts, min_edge_ratio=MIN_EDGE_RATIO)
        seconds.append(result.seconds)
    clocks = sampler.stop()
    model.close()
    step_seconds = sum(seconds) / len(seconds)
    value = count / step_seconds
    attention = [[float(v) for v in row] for row in result.attention]
    ratios = [float(reference.basin_statistics(row, MIN_EDGE_RATIO)[3]) for row in result.attention]
    highest = int(result.layer_index[max(range(len(ratios)), key=lambda i: ratios[i])])
    profiles = {"layer_index": [int(v) for v in result.layer_index], "attention": attention,
                "position_order": [[int(v) for v in row] for row in result.position_order],
                "edge_ratio": ratios}
    reference_result_path(args.config, count).write_text(json.dumps({
        "config": args.config, "prompts": count, "min_edge_ratio": MIN_EDGE_RATIO,
        "selected_layer": int(result.selected_layer), "highest_ratio_layer": highest, "profiles": profiles}))
    line = {
        "metric": METRIC, "impl": "reference", "value": round(value, 3), "unit": "prompts/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_seconds * 1000, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16/fp32",
        "data": "synthetic (seeded random-init weights, seeded random token-id prompts)",
        "config": {"workload": spec["text"].format(n=count) + "; reference CudaLlamaModel + "
                               "AttentionLayerScanner (stock path)",
                   "global_batch": count, "seq_len": round(sum(len(p.tokens) for p in prompts) / count, 1),
                   "parallelism": "one GPU (rank 0 under torchrun): the reference has no multi-GPU path"},
        "reference_device": "gpu",
        "reference_note": "the reference's path is CUDA (model.cu, kernels.cu): value is its stock scan on one "
                          "B200, wall clock around the synchronous AttentionLayerScanner::scan",
        "clocks": clocks,
        "selected_layer": int(result.selected_layer),
        "highest_ratio_layer": highest,
        "profiles": profiles,
        "e2e": {"value": round(value, 3), "unit": "prompts/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(shape, prompts[0])
    return line


# ---------------------------------------------------------------------------------------------
# Decode (generation after reranking, the answering step of CudaLlamaModel::generate): one
# prompt of the config-3 shape, greedy, a fixed number of new tokens (eos disabled). Decode does
# not shard: with N GPUs every rank runs its own replica and `value` is the sum over replicas.
DECODE_METRIC = "decode tokens/s (Qwen2.5-7B arch, greedy, one prompt)"


def decode_bytes_per_token(config, context: int) -> float:
    """Algorithmic HBM bytes of one decode step: every 16-bit weight matrix once (q|k|v, o, gate|up,
    down per layer; the tied output head) plus the K and V rows of `context` cached positions."""
    H, I, V = config.hidden_size, config.intermediate_size, config.vocab_size
    D = H // config.num_attention_heads
    qkv = (config.num_attention_heads + 2 * config.num_key_value_heads) * D
    per_layer = (qkv * H + H * config.num_attention_heads * D + 2 * I * H + H * I) * 2
    cache = 2 * config.num_key_value_heads * D * 2 * context
    return config.num_hidden_layers * (per_layer + cache) + V * H * 2


def decode_setup(args, plain: bool = False):
    """(config, prompt tokens) of the decode workload; `plain` gives the architecture as the
    numpy-only ModelShape (for the reference arm, which loads no library of this build)."""
    import dataclasses

    import probe_workloads as PW
    shape = PW.QWEN2_7B
    if getattr(args, "decode_layers", None):
        shape = dataclasses.replace(shape, num_hidden_layers=args.decode_layers)
    prompt = [int(t) for t in PW.token_prompts(1, shape.vocab_size, PW.QWEN_PROMPTS)[0].tokens]
    if plain:
        return shape, prompt
    from attnrank import synthetic
    config = synthetic.config_of(shape)
    config.tie_word_embeddings = True  # the reference harness ties the head to the embedding
    return config, prompt


def cpu_decode_baseline(config, context: int, layers: int = 2) -> dict:
    """The decode step restated in fp32 torch on the host cores (q|k|v, RoPE-free attention over
    `context` cached keys, o_proj, SwiGLU MLP per layer; the output head), timed on `layers`
    layers plus the head and scaled to the full depth. Random weights: the time does not depend
    on their values."""
    import torch
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    H, I, V = config.hidden_size, config.intermediate_size, config.vocab_size
    Hq, Hkv = config.num_attention_heads, config.num_key_value_heads
    D = H // Hq
    g = torch.Generator().manual_seed(0)
    w_qkv = torch.randn((Hq + 2 * Hkv) * D, H, generator=g) * 0.02
    w_o = torch.randn(H, Hq * D, generator=g) * 0.02
    w_gu = torch.randn(2 * I, H, generator=g) * 0.02
    w_d = torch.randn(H, I, generator=g) * 0.02
    head = torch.randn(V, H, generator=g) * 0.02
    keys = torch.randn(Hkv, context, D, generator=g)
    values = torch.randn(Hkv, context, D, generator=g)
    x = torch.randn(H, generator=g)

    def layer(h):
        n = h * torch.rsqrt(h.pow(2).mean() + 1e-6)
        qkv = w_qkv @ n
        q = qkv[:Hq * D].view(Hq, D)
        scores = torch.einsum("hd,hkd->hk", q, keys.repeat_interleave(Hq // Hkv, dim=0)) / math.sqrt(D)
        attn = torch.einsum("hk,hkd->hd", torch.softmax(scores, dim=-1), values.repeat_interleave(Hq // Hkv, dim=0))
        h = h + w_o @ attn.reshape(-1)
        n = h * torch.rsqrt(h.pow(2).mean() + 1e-6)
        gu = w_gu @ n
        return h + w_d @ (torch.nn.functional.silu(gu[:I]) * gu[I:])

    layer(x)
    start = time.perf_counter()
    h = x
    for _ in range(layers):
        h = layer(h)
    logits = head @ h
    seconds_layers = time.perf_counter() - start
    start = time.perf_counter()
    head @ h
    seconds_head = time.perf_counter() - start
    per_token = (seconds_layers - seconds_head) * config.num_hidden_layers / layers + seconds_head
    del logits
    return {"value": round(1.0 / per_token, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{layers} of {config.num_hidden_layers} layers + the output head of one decode step over "
                      f"{context} cached keys, fp32 torch on the host, scaled to all layers"}


def run_decode(args, rank, world, local_rank):
    import torch
    import attnrank as ar
    config, prompt = decode_setup(args)
    new = args.decode_tokens
    engine = ar.Engine.synthetic(config, seed=0, options=ar.RuntimeOptions(device_index=local_rank,
                                                                            max_sequence_length=4096))
    engine.config.eos_token_id = -1  # a fixed number of new tokens
    stream = torch.cuda.ExternalStream(engine.stream, device=torch.device("cuda", local_rank))
    for _ in range(max(args.warmup, 1)):
        engine.generate(prompt, max_new_tokens=new)
    torch.cuda.synchronize(local_rank)
    barrier(world)

    def timed(tokens):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        wall = time.perf_counter()
        result = engine.generate(prompt, max_new_tokens=tokens)
        stop.record(stream)
        stop.synchronize()
        return start.elapsed_time(stop) / 1000.0, time.perf_counter() - wall, result

    sampler = ClockSampler(local_rank)
    sampler.start()
    full, first, walls, results = [], [], [], None
    for _ in range(args.steps):
        seconds, wall, results = timed(new)
        full.append(seconds)
        walls.append(wall)
        first.append(timed(1)[0])
    clocks = sampler.stop()
    full_s = max_over_ranks(statistics.median(full), world)
    first_s = max_over_ranks(statistics.median(first), world)
    wall_s = max_over_ranks(statistics.median(walls), world)
    per_token = (full_s - first_s) / (new - 1)
    peak, kind = peaks()
    hbm = peak.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    context = len(prompt) + new // 2
    traffic = decode_bytes_per_token(config, context)
    achieved = traffic / per_token / 1e9
    result = {
        "metric": DECODE_METRIC, "value": round(world / per_token, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_token": round(per_token * 1000, 4),
        "ms_per_step": round(full_s * 1000, 3), "higher_is_better": True,
        "scaling": "weak (replicas only: one prompt's decode does not shard)", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (seeded random-init weights, seeded random token-id prompt)",
        "config": {"workload": f"greedy generate of {new} new tokens after one {len(prompt)}-token prompt "
                               "(config-3 shape), Qwen2.5-7B architecture, tied output head, eos disabled; "
                               "value = decode steps only: (T(generate N) - T(generate 1)) / (N - 1)",
                   "global_batch": 1, "seq_len": len(prompt) + new, "parallelism": f"{world} replica(s)",
                   "l2": "weights (14 GB) exceed L2 on every step: no flush needed"},
        "prefill_and_first_token_ms": round(first_s * 1000, 3),
        "e2e": {"value": round(world * new / wall_s, 2), "unit": "tokens/s (generate call, prefill included)",
                "h2d_bytes_per_step": 4 * len(prompt) + 8, "d2h_bytes_per_step": 8 * new},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "per_token_bytes": traffic,
                     "note": f"whole decode step (all kernels) against the {kind} copy bandwidth"},
        "clocks": clocks,
        "gpu_launches": args.steps * (new - 1) * (1 if engine.decode_mode == "persistent"
                                                   else 2 + 5 * config.num_hidden_layers),
        "decode_mode": engine.decode_mode,
        "tokens_head": results.generated_tokens[:8] if results else None,
    }
    engine.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_decode_baseline(config, context)
    return result


def run_decode_reference(args, rank, world, local_rank):
    from oracle import reference
    if reference.load_or_none() is None:
        return {"impl": "reference", "unavailable": "oracle/_ref/libattnrank_ref.so was not built (make -C oracle reference)"}
    config, prompt = decode_setup(args, plain=True)
    new = args.decode_tokens
    model = reference.ReferenceModel(config, seed=0, max_sequence_length=4096, device=local_rank)
    for _ in range(max(args.warmup, 1)):
        model.generate(prompt, max_new_tokens=min(new, 16))
    full, first = [], []
    tokens = None
    for _ in range(args.steps):
        tokens, seconds = model.generate(prompt, max_new_tokens=new)
        full.append(seconds)
        first.append(model.generate(prompt, max_new_tokens=1)[1])
    model.close()
    full_s = max_over_ranks(statistics.median(full), world)
    first_s = max_over_ranks(statistics.median(first), world)
    per_token = (full_s - first_s) / (new - 1)
    value = world / per_token
    return {
        "metric": DECODE_METRIC, "impl": "reference", "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_token": round(per_token * 1000, 4),
        "ms_per_step": round(full_s * 1000, 3), "higher_is_better": True, "scaling": "weak (replicas only)",
        "vs_baseline": None, "dtype": "fp16/fp32",
        "data": "synthetic (seeded random-init weights, seeded random token-id prompt)",
        "config": {"workload": f"reference CudaLlamaModel::generate, greedy, {new} new tokens after the same "
                               f"{len(prompt)}-token prompt (eos 2 never met in this run: "
                               f"{len(tokens) if tokens is not None else 0} tokens)",
                   "global_batch": 1, "parallelism": f"{world} replica(s)"},
        "prefill_and_first_token_ms": round(first_s * 1000, 3),
        "tokens_head": tokens[:8] if tokens else None,
        "reference_device": "gpu",
        "reference_note": "the reference's path is CUDA: wall clock around its synchronous generate on one B200",
        "cpu_baseline": cpu_decode_baseline(config, len(prompt) + new // 2),
        "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def emit(line: dict, out) -> None:
    out.write(json.dumps(line) + "\n")
    out.flush()


def main():
    args = parse_args()
    # stdout carries exactly one JSON line. Whatever a library prints there (NCCL's version
    # banner, for one) goes to stderr: file descriptor 1 points at stderr for the whole run, and
    # the JSON line is written through a saved copy of the original stdout.
    sys.stdout.flush()
    out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        # The reference has no multi-GPU path (README.md:17, :149): under torchrun rank 0 alone runs
        # it on its GPU and prints the line; the other ranks exit 0 without work.
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        import torch
        torch.cuda.set_device(local_rank)
        result = (run_decode_reference if args.decode else run_reference)(args, 0, 1, local_rank)
        result["n_gpus"] = int(os.environ.get("WORLD_SIZE", "1"))
        result["reference_gpus_used"] = 1
        emit(result, out)
        return
    rank, world, local_rank = init_distributed(args)
    if args.sweep:
        peak, kind = peaks()
        result = {"sweep": bandwidth_sweep(peak.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]), dtype=args.dtype),
                  "peak_source": f"{kind} hbm_gbs", "dtype": args.dtype,
                  "config": "tokens {1,64,1024,8192,32768} x hidden {2048,3584,4096,8192}, head_dim 128, "
                            "intermediate 3.5 x hidden, vocab 152064"}
    elif args.copy_under_cap:
        result = {"copy_under_power_cap": copy_under_power_cap(local_rank)}
    elif args.attention_compare:
        peak, kind = peaks()
        result = {"attention_comparison": attention_comparison(peak.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]),
                                                               dtype=args.dtype),
                  "peak_source": f"{kind} bf16_tflops (burst)", "dtype": args.dtype}
    elif args.kernels_only:
        from attnrank import synthetic
        peak, kind = peaks()
        result = {"kernels": kernel_rooflines(synthetic.qwen2_7b(), peak.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]),
                                              peak.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]),
                                              tokens=args.kernel_tokens, dtype=args.dtype),
                  "kernels_peak_source": f"{kind} hbm_gbs / bf16_tflops (burst)", "tokens": args.kernel_tokens}
    elif args.decode:
        result = run_decode(args, rank, world, local_rank)
    else:
        result = run_b200(args, rank, world, local_rank)
    if rank == 0:
        emit(result, out)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()

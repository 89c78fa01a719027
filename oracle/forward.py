"""fp32 CPU restatement of the reference's attention-capture forward pass. Test infrastructure only.

Follows, operation by operation:
  embedding_lookup_kernel          attnrank/src/kernels.cu:50-58
  rms_norm_kernel                  attnrank/src/kernels.cu:60-83   y = (x * rsqrt(mean(x^2) + eps)) * w
  rotary_embedding_kernel          attnrank/src/kernels.cu:85-115  rotate-half, inv_freq = theta^(-2i/D), pos = t
  softmax_causal_kernel            attnrank/src/kernels.cu:117-162 causal (+ sliding window) row softmax
  silu_multiply_kernel             attnrank/src/kernels.cu:164-170 g / (1 + e^-g) * u
  reduce_document_attention_kernel attnrank/src/kernels.cu:202-236 span sums over heads x query rows
  LlamaForwardPass                 attnrank/src/model.cu:324-419   block order, GQA map h -> h / group,
                                                                   scale 1/sqrt(D) (model.cu:444)
  measure_attention_by_layer       attnrank/src/model.cu:593-617   rows / (query_rows * Hq), unit sum
  measure_attention                attnrank/src/model.cu:567-591   layer-averaged variant
The reference evaluates prompts in prefill chunks of 512 tokens against a KV cache; the result is
the full causal attention, which is what this module computes in one piece. The chunk length only
matters for normalize_by_length divisors (the span end is clipped at the end of the query row's
chunk, kernels.cu:211 with key_count = chunk end), which this module reproduces.

Weights come from the seeded synthetic checkpoint (oracle/weights.py), generated one layer at a
time so that a 7B-shaped model needs about 1 GB of host memory at any moment.

`gemm_inputs` optionally rounds every projection-GEMM input the way an implementation does:
'fp16' mirrors the reference (model.cu:353-365 casts fp32 activations to fp16), 'bf16' mirrors
a bf16 build. None keeps pure fp32.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Sequence

import numpy as np
import torch

from oracle import weights as W


@dataclass(frozen=True)
class Shape:
    hidden: int
    intermediate: int
    layers: int
    heads: int
    kv_heads: int
    vocab: int
    eps: float
    theta: float
    window: int = 0
    bias: bool = False

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim


@dataclass
class Prompt:
    tokens: np.ndarray                  # int32 [T]
    query_span: tuple[int, int]         # prompt-relative, half-open
    spans: Sequence[tuple[int, int]]    # document spans, half-open


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    mean = (x * x).sum(-1, keepdim=True) / x.shape[-1]
    return (x * torch.rsqrt(mean + eps)) * weight


def rope_tables(positions: int, head_dim: int, theta: float) -> tuple[np.ndarray, np.ndarray]:
    index = np.arange(head_dim // 2, dtype=np.float32)
    inverse = np.power(np.float32(theta), (np.float32(-2.0) * index) / np.float32(head_dim)).astype(np.float32)
    angle = (np.arange(positions, dtype=np.float32)[:, None] * inverse[None, :]).astype(np.float32)
    return np.cos(angle.astype(np.float64)).astype(np.float32), np.sin(angle.astype(np.float64)).astype(np.float32)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    low, high = x[..., :half], x[..., half:]
    c, s = cos[:, None, :], sin[:, None, :]
    return torch.cat([low * c - high * s, high * c + low * s], dim=-1)


def silu_multiply(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    return (gate / (1.0 + torch.exp(-gate))) * up


def document_mass(probs: torch.Tensor, prompt: Prompt, chunk: int, normalize_by_length: bool) -> np.ndarray:
    """Sum of softmax probabilities over each document span, heads and query rows (fp64).

    probs: [Hq, T, T] causal softmax rows. Returns the raw reference accumulator for the layer.
    """
    T = probs.shape[-1]
    qb, qe = prompt.query_span
    qb = max(qb, 0)  # rows before token 0 do not exist (kernels.cu:218 keeps every row >= begin)
    qe = min(qe, T)
    out = np.zeros(len(prompt.spans), dtype=np.float64)
    if qe <= qb:
        return out
    rows = probs[:, qb:qe, :].to(torch.float64)  # [Hq, Tq, T]
    query_positions = np.arange(qb, qe)
    chunk_end = np.minimum(((query_positions // chunk) + 1) * chunk, T)
    for s, (b, e) in enumerate(prompt.spans):
        e_eff = min(e, T)
        if e_eff <= b:
            continue
        per_row = rows[:, :, b:e_eff].sum(-1)  # [Hq, Tq]
        if normalize_by_length:
            divisor = np.minimum(e, chunk_end) - b
            scale = np.where(divisor > 0, 1.0 / np.maximum(divisor, 1), 1.0)
            per_row = per_row * torch.from_numpy(scale)[None, :]
        out[s] = float(per_row.sum())
    return out


class OracleModel:
    def __init__(self, shape: Shape, seed: int = 0, std: float = 0.02, gemm_inputs: str | None = None,
                 threads: int | None = None, chunk: int = 512):
        self.shape = shape
        self.seed = seed
        self.std = std
        self.gemm_inputs = gemm_inputs
        self.chunk = chunk
        self._cached_layers: dict[int, dict[str, torch.Tensor]] = {}
        self._cached_rows: dict[bytes, torch.Tensor] = {}
        if threads:
            torch.set_num_threads(threads)

    def prepare(self, prompts: Sequence[Prompt], layers: int | None = None) -> None:
        """Generate the weights of the first `layers` layers and the embedding rows of `prompts`
        now, so that a timed probe() afterwards runs the forward pass alone."""
        for layer in range(self.shape.layers if layers is None else layers):
            self._cached_layers[layer] = self.layer_weights(layer)
        for p in prompts:
            self._cached_rows[np.asarray(p.tokens, dtype=np.int32).tobytes()] = self._embedding_rows(p.tokens)

    def _embedding_rows(self, tokens) -> torch.Tensor:
        cached = self._cached_rows.get(np.asarray(tokens, dtype=np.int32).tobytes())
        if cached is not None:
            return cached.clone()
        return torch.from_numpy(W.gather_rows(tokens, self.shape.hidden, self.seed, -1, W.EMBEDDING, self.std))

    # -- weights (generated per layer) -------------------------------------------------------
    def _matrix(self, rows: int, cols: int, layer: int, kind: int) -> torch.Tensor:
        return torch.from_numpy(W.matrix(rows, cols, self.seed, layer, kind, self.std))

    def layer_weights(self, layer: int) -> dict[str, torch.Tensor]:
        if layer in self._cached_layers:
            return self._cached_layers[layer]
        s = self.shape
        qd = s.heads * s.head_dim
        w = {
            "q": self._matrix(qd, s.hidden, layer, W.QUERY),
            "k": self._matrix(s.kv_width, s.hidden, layer, W.KEY),
            "v": self._matrix(s.kv_width, s.hidden, layer, W.VALUE),
            "o": self._matrix(s.hidden, qd, layer, W.OUTPUT),
            "gate": self._matrix(s.intermediate, s.hidden, layer, W.GATE),
            "up": self._matrix(s.intermediate, s.hidden, layer, W.UP),
            "down": self._matrix(s.hidden, s.intermediate, layer, W.DOWN),
            "input_norm": torch.from_numpy(W.f32(s.hidden, self.seed, layer, W.INPUT_NORM, 0.0, 1.0)),
            "post_norm": torch.from_numpy(W.f32(s.hidden, self.seed, layer, W.POST_NORM, 0.0, 1.0)),
        }
        if s.bias:
            w["q_bias"] = torch.from_numpy(W.f32(qd, self.seed, layer, W.QUERY_BIAS, self.std))
            w["k_bias"] = torch.from_numpy(W.f32(s.kv_width, self.seed, layer, W.KEY_BIAS, self.std))
            w["v_bias"] = torch.from_numpy(W.f32(s.kv_width, self.seed, layer, W.VALUE_BIAS, self.std))
        return w

    def _gemm_input(self, x: torch.Tensor) -> torch.Tensor:
        if self.gemm_inputs == "fp16":
            return x.to(torch.float16).to(torch.float32)
        if self.gemm_inputs == "bf16":
            return x.to(torch.bfloat16).to(torch.float32)
        return x

    def _linear(self, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
        return self._gemm_input(x) @ weight.T

    # -- forward ----------------------------------------------------------------------------
    def probe(self, prompts: Sequence[Prompt], layer_begin: int = 0, layer_end: int = -1,
              normalize_by_length: bool = False) -> tuple[list[np.ndarray], list[np.ndarray]]:
        """measure_attention_by_layer for each prompt.

        Returns (rows, raw_rows), each a list of [layers, spans] fp64 arrays: rows are unit-sum
        (model.cu:602-615), raw_rows are the totals divided by query_rows * Hq.
        """
        s = self.shape
        begin = 0 if layer_begin < 0 else layer_begin
        end = s.layers if layer_end < 0 else layer_end
        if not (0 <= begin < end <= s.layers):
            raise ValueError(f"probe layers [{begin},{end}) are out of range")
        longest = max(len(p.tokens) for p in prompts)
        cos_np, sin_np = rope_tables(longest, s.head_dim, s.theta)
        cos, sin = torch.from_numpy(cos_np), torch.from_numpy(sin_np)
        hidden = [self._embedding_rows(p.tokens) for p in prompts]
        raw = [np.zeros((end - begin, len(p.spans)), dtype=np.float64) for p in prompts]
        scale = 1.0 / math.sqrt(float(s.head_dim))
        group = s.heads // s.kv_heads
        for layer in range(end):
            w = self.layer_weights(layer)
            for index, prompt in enumerate(prompts):
                h = hidden[index]
                T = h.shape[0]
                x = rms_norm(h, w["input_norm"], s.eps)
                q = self._linear(x, w["q"])
                k = self._linear(x, w["k"])
                v = self._linear(x, w["v"])
                if s.bias:
                    q, k, v = q + w["q_bias"], k + w["k_bias"], v + w["v_bias"]
                q = apply_rope(q.view(T, s.heads, s.head_dim), cos[:T], sin[:T])
                k = apply_rope(k.view(T, s.kv_heads, s.head_dim), cos[:T], sin[:T])
                v = v.view(T, s.kv_heads, s.head_dim)
                kq = k.repeat_interleave(group, dim=1)  # kv head of query head h is h // group
                vq = v.repeat_interleave(group, dim=1)
                scores = torch.einsum("qhd,khd->hqk", q, kq) * scale
                key = torch.arange(T)[None, :]
                query = torch.arange(T)[:, None]
                visible = key <= query
                if s.window > 0:
                    visible &= key >= query + 1 - s.window
                scores = scores.masked_fill(~visible[None], float("-inf"))
                probs = torch.softmax(scores, dim=-1)
                if layer >= begin:
                    raw[index][layer - begin] = document_mass(probs, prompt, self.chunk, normalize_by_length)
                attn = torch.einsum("hqk,khd->qhd", probs, vq).reshape(T, s.heads * s.head_dim)
                h = h + self._linear(attn, w["o"])
                x = rms_norm(h, w["post_norm"], s.eps)
                a = silu_multiply(self._linear(x, w["gate"]), self._linear(x, w["up"]))
                hidden[index] = h + self._linear(a, w["down"])
        rows, raw_rows = [], []
        for index, prompt in enumerate(prompts):
            T = len(prompt.tokens)
            qb, qe = prompt.query_span
            observations = max(0, min(qe, T) - qb) * s.heads
            r = raw[index] / observations if observations > 0 else np.zeros_like(raw[index])
            raw_rows.append(r.copy())
            sums = r.sum(axis=1, keepdims=True)
            rows.append(np.where(sums > 0, r / np.where(sums > 0, sums, 1.0), r))
        return rows, raw_rows

    def next_token_logits(self, tokens: np.ndarray, tied: bool = True) -> np.ndarray:
        """The logits generation reads after a prompt (CudaLlamaModel::generate, model.cu:532-565):
        every layer over the whole sequence (the reference's chunked prefill and one-token decode
        steps against its KV cache compute this same causal forward), the final RMSNorm
        (model.norm.weight) and the output head on the last row (read_logits, model.cu:341-350):
        the embedding when tied (tie_word_embeddings), else lm_head.weight. fp32 [vocab]."""
        s = self.shape
        ids = np.asarray(tokens, dtype=np.int32)
        T = ids.size
        cos_np, sin_np = rope_tables(T, s.head_dim, s.theta)
        cos, sin = torch.from_numpy(cos_np), torch.from_numpy(sin_np)
        h = torch.from_numpy(W.gather_rows(ids, s.hidden, self.seed, -1, W.EMBEDDING, self.std))
        scale = 1.0 / math.sqrt(float(s.head_dim))
        group = s.heads // s.kv_heads
        key = torch.arange(T)[None, :]
        query = torch.arange(T)[:, None]
        visible = key <= query
        if s.window > 0:
            visible &= key >= query + 1 - s.window
        for layer in range(s.layers):
            w = self.layer_weights(layer)
            x = rms_norm(h, w["input_norm"], s.eps)
            q, k, v = self._linear(x, w["q"]), self._linear(x, w["k"]), self._linear(x, w["v"])
            if s.bias:
                q, k, v = q + w["q_bias"], k + w["k_bias"], v + w["v_bias"]
            q = apply_rope(q.view(T, s.heads, s.head_dim), cos, sin)
            k = apply_rope(k.view(T, s.kv_heads, s.head_dim), cos, sin)
            v = v.view(T, s.kv_heads, s.head_dim)
            kq = k.repeat_interleave(group, dim=1)
            vq = v.repeat_interleave(group, dim=1)
            scores = torch.einsum("qhd,khd->hqk", q, kq) * scale
            probs = torch.softmax(scores.masked_fill(~visible[None], float("-inf")), dim=-1)
            attn = torch.einsum("hqk,khd->qhd", probs, vq).reshape(T, s.heads * s.head_dim)
            h = h + self._linear(attn, w["o"])
            x = rms_norm(h, w["post_norm"], s.eps)
            h = h + self._linear(silu_multiply(self._linear(x, w["gate"]), self._linear(x, w["up"])), w["down"])
        final = torch.from_numpy(W.f32(s.hidden, self.seed, -1, W.FINAL_NORM, 0.0, 1.0))
        last = rms_norm(h[-1:], final, s.eps)
        head = self._matrix(s.vocab, s.hidden, -1, W.EMBEDDING if tied else W.LM_HEAD)
        return self._linear(last, head)[0].numpy().astype(np.float32)

    def measure_attention(self, prompt: Prompt, layer_begin: int, layer_end: int,
                          normalize_by_length: bool = False) -> np.ndarray:
        """CudaLlamaModel::measure_attention (model.cu:567-591)."""
        _, raw_rows = self.probe([prompt], layer_begin, layer_end, normalize_by_length)
        layers = raw_rows[0].shape[0]
        out = raw_rows[0].sum(axis=0) / layers
        total = out.sum()
        return out / total if total > 0 else out


# ---- isolated per-op restatements used by the kernel parity tests ----------------------------

def op_embedding_rms_norm(table_f32: np.ndarray, ids: np.ndarray, gamma: np.ndarray, eps: float):
    h = torch.from_numpy(table_f32[ids])
    return h.numpy(), rms_norm(h, torch.from_numpy(gamma), eps).numpy()


def op_rms_norm_residual(residual: np.ndarray, delta: np.ndarray, gamma: np.ndarray, eps: float):
    r = torch.from_numpy(residual) + torch.from_numpy(delta)
    return r.numpy(), rms_norm(r, torch.from_numpy(gamma), eps).numpy()


def op_rotary_bias(qkv: np.ndarray, bias: np.ndarray | None, positions: np.ndarray, heads: int, kv_heads: int,
                   head_dim: int, theta: float, tables: tuple[np.ndarray, np.ndarray] | None = None) -> np.ndarray:
    """Bias + rotate-half RoPE on a fused q|k|v block. `tables` (cos, sin) [positions, D/2] may be
    given to check the rotation arithmetic independently of how the tables were computed."""
    T = qkv.shape[0]
    x = torch.from_numpy(qkv.copy())
    if bias is not None:
        x = x + torch.from_numpy(bias)
    cos_np, sin_np = tables if tables is not None else rope_tables(int(positions.max()) + 1, head_dim, theta)
    cos = torch.from_numpy(cos_np)[positions]
    sin = torch.from_numpy(sin_np)[positions]
    rotated = (heads + kv_heads) * head_dim
    qk = x[:, :rotated].view(T, heads + kv_heads, head_dim)
    x[:, :rotated] = apply_rope(qk, cos, sin).reshape(T, rotated)
    return x.numpy()


def op_silu_multiply(gate: np.ndarray, up: np.ndarray) -> np.ndarray:
    return silu_multiply(torch.from_numpy(gate), torch.from_numpy(up)).numpy()


def op_attention(qkv: np.ndarray, offsets: Sequence[int], heads: int, kv_heads: int, head_dim: int,
                 window: int = 0) -> tuple[np.ndarray, np.ndarray, list[torch.Tensor]]:
    """Causal GQA attention per packed prompt. Returns (out [M, Hq*D], lse2 [M, Hq], probs per prompt)."""
    x = torch.from_numpy(qkv)
    group = heads // kv_heads
    out = torch.zeros(x.shape[0], heads * head_dim)
    lse2 = torch.zeros(x.shape[0], heads)
    probs_all = []
    qd, kvw = heads * head_dim, kv_heads * head_dim
    for p in range(len(offsets) - 1):
        a, b = offsets[p], offsets[p + 1]
        T = b - a
        q = x[a:b, :qd].view(T, heads, head_dim)
        k = x[a:b, qd:qd + kvw].view(T, kv_heads, head_dim).repeat_interleave(group, dim=1)
        v = x[a:b, qd + kvw:].view(T, kv_heads, head_dim).repeat_interleave(group, dim=1)
        scores = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(head_dim)
        key = torch.arange(T)[None, :]
        query = torch.arange(T)[:, None]
        visible = key <= query
        if window > 0:
            visible &= key >= query + 1 - window
        scores = scores.masked_fill(~visible[None], float("-inf"))
        lse = torch.logsumexp(scores.to(torch.float64), dim=-1).to(torch.float32)  # [Hq, T]
        probs = torch.softmax(scores, dim=-1)
        out[a:b] = torch.einsum("hqk,khd->qhd", probs, v).reshape(T, qd)
        lse2[a:b] = (lse / math.log(2.0)).T
        probs_all.append(probs)
    return out.numpy(), lse2.numpy(), probs_all

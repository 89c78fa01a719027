"""ctypes wrapper of oracle/_ref/libattnrank_ref.so: the reference's own implementation.

Test and benchmark infrastructure only. The library is built by `make -C oracle reference` from
the reference's unmodified sources (read in place) plus oracle/ref_harness.cpp; it exists on a
GPU box only if it was built before the repository snapshot was taken.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path
from typing import Sequence

import numpy as np

LIBRARY = Path(__file__).resolve().parent / "_ref" / "libattnrank_ref.so"


class RefConfig(ctypes.Structure):
    _fields_ = [("hidden_size", ctypes.c_int), ("intermediate_size", ctypes.c_int),
                ("num_hidden_layers", ctypes.c_int), ("num_attention_heads", ctypes.c_int),
                ("num_key_value_heads", ctypes.c_int), ("vocab_size", ctypes.c_int),
                ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
                ("sliding_window", ctypes.c_int), ("attention_bias", ctypes.c_int)]


class RefPrompt(ctypes.Structure):
    _fields_ = [("tokens", ctypes.c_void_p), ("token_count", ctypes.c_int), ("query_begin", ctypes.c_int),
                ("query_end", ctypes.c_int), ("spans", ctypes.c_void_p)]


_lib = None


def load_or_none():
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        return None
    try:  # one cuBLAS per process: PyTorch's copy first, which the reference's libcublas.so.12 then reuses
        import torch  # noqa: F401
    except ImportError:
        pass
    lib = ctypes.CDLL(str(LIBRARY))
    P, I, I64, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_double
    lib.ref_last_error.restype = ctypes.c_char_p
    lib.ref_create.argtypes = [ctypes.POINTER(RefConfig), ctypes.c_uint64, D, I, I, I]
    lib.ref_create.restype = P
    lib.ref_destroy.argtypes = [P]
    lib.ref_destroy.restype = None
    lib.ref_measure_attention_by_layer.argtypes = [P, ctypes.POINTER(RefPrompt), I, I, I, I, P, P, P]
    lib.ref_measure_attention.argtypes = [P, ctypes.POINTER(RefPrompt), I, I, I, I, P]
    lib.ref_scan.argtypes = [P, ctypes.POINTER(RefPrompt), I, I, I, I, I, D, P, P, P, P, P, P]
    lib.ref_from_accumulated.argtypes = [P, I, I64, P, P]
    lib.ref_basin_statistics.argtypes = [P, I, D, P]
    lib.ref_select_shallowest.argtypes = [P, P, I, I, D]
    lib.ref_resolve_position_order.argtypes = [P, I, I, P]
    lib.ref_rerank.argtypes = [ctypes.c_char_p, ctypes.c_uint64, I, P, I, I, I, P]
    lib.ref_generate.argtypes = [P, P, I, I, ctypes.c_float, ctypes.c_float, I, ctypes.c_uint64, P, P, P]
    lib.ref_sample.argtypes = [ctypes.c_float, ctypes.c_float, I, ctypes.c_uint64, P, I, I, P]
    lib.ref_prefill_logits.argtypes = [P, P, I, P]
    _lib = lib
    return lib


def _require():
    lib = load_or_none()
    if lib is None:
        raise RuntimeError(f"{LIBRARY} is not built (make -C oracle reference)")
    return lib


class _Prompts:
    def __init__(self, prompts: Sequence):
        self.keep = []
        self.array = (RefPrompt * len(prompts))()
        self.span_count = len(prompts[0].document_spans)
        for i, p in enumerate(prompts):
            tokens = np.ascontiguousarray(np.asarray(p.tokens, dtype=np.int32))
            spans = np.ascontiguousarray(np.array([(s.begin, s.end) for s in p.document_spans], dtype=np.int32))
            self.keep += [tokens, spans]
            self.array[i] = RefPrompt(tokens.ctypes.data, tokens.size, p.query_span.begin, p.query_span.end,
                                      spans.ctypes.data)


class ReferenceModel:
    """CudaLlamaModel of the reference on the seeded synthetic checkpoint (needs a GPU)."""

    def __init__(self, config, seed: int = 0, std: float = 0.02, max_sequence_length: int = 2048,
                 prefill_chunk_tokens: int = 512, device: int = 0):
        lib = _require()
        c = RefConfig(config.hidden_size, config.intermediate_size, config.num_hidden_layers,
                      config.num_attention_heads, config.num_key_value_heads, config.vocab_size,
                      config.rms_norm_eps, config.rope_theta, config.sliding_window, int(config.attention_bias))
        self.layers = config.num_hidden_layers
        self.handle = lib.ref_create(ctypes.byref(c), seed, std, max_sequence_length, prefill_chunk_tokens, device)
        if not self.handle:
            raise RuntimeError("reference model: " + lib.ref_last_error().decode())

    def close(self):
        if self.handle:
            _require().ref_destroy(self.handle)
            self.handle = None

    def __del__(self):
        self.close()

    def measure_attention_by_layer(self, prompt, layer_begin=0, layer_end=-1, normalize_by_length=False) -> np.ndarray:
        lib = _require()
        packed = _Prompts([prompt])
        rows = np.zeros((self.layers, packed.span_count), dtype=np.float64)
        first, count = ctypes.c_int(), ctypes.c_int()
        if lib.ref_measure_attention_by_layer(self.handle, packed.array, packed.span_count, layer_begin, layer_end,
                                              int(normalize_by_length), rows.ctypes.data, ctypes.byref(first),
                                              ctypes.byref(count)) != 0:
            raise RuntimeError(lib.ref_last_error().decode())
        return rows[:count.value]

    def measure_attention(self, prompt, layer_begin, layer_end, normalize_by_length=False) -> np.ndarray:
        lib = _require()
        packed = _Prompts([prompt])
        out = np.zeros(packed.span_count, dtype=np.float64)
        if lib.ref_measure_attention(self.handle, packed.array, packed.span_count, layer_begin, layer_end,
                                     int(normalize_by_length), out.ctypes.data) != 0:
            raise RuntimeError(lib.ref_last_error().decode())
        return out

    def scan(self, prompts, min_edge_ratio=1.3, layer_begin=0, layer_end=-1, normalize_by_length=False):
        """AttentionLayerScanner::scan + select_shallowest_basin_layer. Returns a ScanResult."""
        lib = _require()
        packed = _Prompts(prompts)
        S = packed.span_count
        attention = np.zeros((self.layers, S), dtype=np.float64)
        order = np.zeros((self.layers, S), dtype=np.int32)
        layer_index = np.zeros(self.layers, dtype=np.int32)
        count, selected, seconds = ctypes.c_int(), ctypes.c_int(), ctypes.c_double()
        if lib.ref_scan(self.handle, packed.array, len(prompts), S, layer_begin, layer_end, int(normalize_by_length),
                        min_edge_ratio, attention.ctypes.data, order.ctypes.data, layer_index.ctypes.data,
                        ctypes.byref(count), ctypes.byref(selected), ctypes.byref(seconds)) != 0:
            raise RuntimeError(lib.ref_last_error().decode())
        n = count.value
        return ScanResult(attention[:n], order[:n], layer_index[:n], selected.value, seconds.value)


    def generate(self, prompt_tokens, max_new_tokens: int, temperature: float = 0.0, top_p: float = 0.9,
                 top_k: int = 0, seed: int = 1234) -> tuple[list[int], float]:
        """CudaLlamaModel::generate with make_sampler's sampler: (generated ids, seconds)."""
        lib = _require()
        tokens = np.ascontiguousarray(np.asarray(prompt_tokens, dtype=np.int32))
        out = np.zeros(max(max_new_tokens, 1), dtype=np.int32)
        count, seconds = ctypes.c_int(), ctypes.c_double()
        if lib.ref_generate(self.handle, tokens.ctypes.data, tokens.size, max_new_tokens, temperature, top_p, top_k,
                            seed, out.ctypes.data, ctypes.byref(count), ctypes.byref(seconds)) != 0:
            raise RuntimeError(lib.ref_last_error().decode())
        return [int(t) for t in out[:count.value]], seconds.value


    def prefill_logits(self, prompt_tokens, vocab_size: int) -> np.ndarray:
        """The fp32 logits the reference's generate gives its sampler after prefilling the prompt."""
        lib = _require()
        tokens = np.ascontiguousarray(np.asarray(prompt_tokens, dtype=np.int32))
        out = np.zeros(vocab_size, dtype=np.float32)
        if lib.ref_prefill_logits(self.handle, tokens.ctypes.data, tokens.size, out.ctypes.data) != 0:
            raise RuntimeError(lib.ref_last_error().decode())
        return out


@dataclass
class ScanResult:
    attention: np.ndarray
    position_order: np.ndarray
    layer_index: np.ndarray
    selected_layer: int
    seconds: float


# ---- host-only functions of the reference (no GPU needed) -----------------------------------
def from_accumulated(accumulated: Sequence[float], sample_count: int):
    lib = _require()
    acc = np.ascontiguousarray(np.asarray(accumulated, dtype=np.float64))
    attention = np.zeros_like(acc)
    order = np.zeros(acc.size, dtype=np.int32)
    lib.ref_from_accumulated(acc.ctypes.data, acc.size, sample_count, attention.ctypes.data, order.ctypes.data)
    return attention, order


def basin_statistics(attention: Sequence[float], min_edge_ratio: float) -> np.ndarray:
    lib = _require()
    values = np.ascontiguousarray(np.asarray(attention, dtype=np.float64))
    out = np.zeros(5, dtype=np.float64)
    lib.ref_basin_statistics(values.ctypes.data, values.size, min_edge_ratio, out.ctypes.data)
    return out


def select_shallowest(attention: np.ndarray, layer_indices: Sequence[int], min_edge_ratio: float) -> int:
    lib = _require()
    matrix = np.ascontiguousarray(np.asarray(attention, dtype=np.float64))
    layers = np.ascontiguousarray(np.asarray(layer_indices, dtype=np.int32))
    return lib.ref_select_shallowest(matrix.ctypes.data, layers.ctypes.data, matrix.shape[0], matrix.shape[1],
                                     min_edge_ratio)


def resolve_position_order(preferred: Sequence[int], count: int) -> list[int]:
    lib = _require()
    pref = np.ascontiguousarray(np.asarray(preferred, dtype=np.int32))
    out = np.zeros(count, dtype=np.int32)
    lib.ref_resolve_position_order(pref.ctypes.data if pref.size else None, pref.size, count, out.ctypes.data)
    return [int(v) for v in out]


def rerank(strategy: str, count: int, calls: int = 1, seed: int = 1234, lim_start_first: bool = False,
           position_order: Sequence[int] = ()) -> list[list[int]]:
    """The reference's RerankerFactory reranker applied `calls` times to the ranking 0..count-1:
    the document index at each position after every call (the random reranker's state carries)."""
    lib = _require()
    order = np.ascontiguousarray(np.asarray(position_order, dtype=np.int32))
    out = np.zeros((max(calls, 1), max(count, 1)), dtype=np.int32)
    if lib.ref_rerank(strategy.encode(), seed, int(lim_start_first), order.ctypes.data if order.size else None,
                      order.size, count, calls, out.ctypes.data) != 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return [[int(v) for v in row[:count]] for row in out[:calls]]


def sample(logits_rows: np.ndarray, temperature: float, top_p: float, top_k: int, seed: int) -> list[int]:
    """The reference's make_sampler(config)->select over each row of logits_rows, one sampler."""
    lib = _require()
    rows = np.ascontiguousarray(np.asarray(logits_rows, dtype=np.float32))
    if rows.ndim == 1:
        rows = rows[None, :]
    out = np.zeros(rows.shape[0], dtype=np.int32)
    if lib.ref_sample(temperature, top_p, top_k, seed, rows.ctypes.data, rows.shape[1], rows.shape[0],
                      out.ctypes.data) != 0:
        raise RuntimeError(lib.ref_last_error().decode())
    return [int(v) for v in out]

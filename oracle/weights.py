"""Seeded synthetic checkpoint on the CPU (checker side). Test infrastructure only.

Wraps liboracle.so, built from oracle/synth_weights.c by oracle/Makefile. The element formula is
documented in synth_weights.c; the product's GPU generator (csrc/synthetic.cu) is an independent
implementation of the same definition.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liboracle.so"

# tensor kinds (csrc/synthetic.h)
EMBEDDING, QUERY, KEY, VALUE, OUTPUT = 0, 1, 2, 3, 4
QUERY_BIAS, KEY_BIAS, VALUE_BIAS = 5, 6, 7
GATE, UP, DOWN = 8, 9, 10
INPUT_NORM, POST_NORM, FINAL_NORM, LM_HEAD = 11, 12, 13, 14

_lib = None


def build() -> Path:
    """Compile liboracle.so (gcc, OpenMP)."""
    subprocess.run(["make", "-C", str(HERE), "liboracle.so"], check=True, capture_output=True)
    return LIBRARY


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            build()
        handle = ctypes.CDLL(str(LIBRARY))
        handle.oracle_fill_bf16.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint64,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_double]
        handle.oracle_fill_f32.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_uint64,
                                           ctypes.c_int, ctypes.c_int, ctypes.c_double, ctypes.c_float]
        handle.oracle_gather_rows_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                                  ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_double]
        handle.oracle_tensor_key.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        handle.oracle_tensor_key.restype = ctypes.c_uint64
        _lib = handle
    return _lib


def bf16_bits(count: int, seed: int, layer: int, kind: int, std: float = 0.02, first: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.uint16)
    lib().oracle_fill_bf16(out.ctypes.data, first, count, seed, layer, kind, std)
    return out


def f32(count: int, seed: int, layer: int, kind: int, std: float = 0.02, offset: float = 0.0, first: int = 0) -> np.ndarray:
    out = np.empty(count, dtype=np.float32)
    lib().oracle_fill_f32(out.ctypes.data, first, count, seed, layer, kind, std, offset)
    return out


def matrix(rows: int, cols: int, seed: int, layer: int, kind: int, std: float = 0.02) -> np.ndarray:
    return f32(rows * cols, seed, layer, kind, std).reshape(rows, cols)


def gather_rows(ids: np.ndarray, cols: int, seed: int, layer: int, kind: int, std: float = 0.02) -> np.ndarray:
    ids = np.ascontiguousarray(ids, dtype=np.int32)
    out = np.empty((ids.size, cols), dtype=np.float32)
    lib().oracle_gather_rows_f32(out.ctypes.data, ids.ctypes.data, ids.size, cols, seed, layer, kind, std)
    return out


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(values: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (finite inputs)."""
    bits = np.ascontiguousarray(values, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def round_bf16(values: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16_bits(values))


def set_threads(count: int | None = None) -> int:
    """OpenMP thread count used by liboracle.so (defaults to all host cores)."""
    count = count or os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(count)
    return count

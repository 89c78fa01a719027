"""Hugging Face checkpoint I/O for the engine: safetensors read (numpy memmap) and write.

The reference maps safetensors shards (attnrank/src/checkpoint.cpp:67-122, :178-216) and uploads
every tensor it needs by its Hugging Face name (model.cu:113-174). This module does the same from
Python and hands each tensor to the native engine (ar_engine_load_tensor), which converts it to
the resident bf16 / fp32 layout. Only the tensors of the profiling path are used.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Iterator

import numpy as np

from attnrank import _native
from attnrank._native import AttnRankError

_DTYPES = {
    "F32": (np.float32, _native.DTYPE_F32),
    "F16": (np.uint16, _native.DTYPE_F16),
    "BF16": (np.uint16, _native.DTYPE_BF16),
}


def read_header(path: Path) -> tuple[dict, int]:
    with open(path, "rb") as handle:
        prefix = handle.read(8)
        if len(prefix) < 8:
            raise AttnRankError(f"safetensors file too small: '{path}'")
        (length,) = struct.unpack("<Q", prefix)
        header = json.loads(handle.read(length))
    return header, 8 + length


def iter_tensors(path: Path) -> Iterator[tuple[str, np.ndarray, int]]:
    """(name, array view, native dtype code) for every tensor of one shard."""
    header, data_origin = read_header(path)
    mapped = np.memmap(path, dtype=np.uint8, mode="r")
    for name, entry in header.items():
        if name == "__metadata__":
            continue
        kind = entry["dtype"]
        if kind not in _DTYPES:
            raise AttnRankError(f"unsupported dtype '{kind}' for tensor '{name}'")
        numpy_type, code = _DTYPES[kind]
        begin, end = entry["data_offsets"]
        raw = mapped[data_origin + begin:data_origin + end]
        array = raw.view(numpy_type).reshape(entry["shape"])
        yield name, array, code


def load_directory(engine, directory: Path) -> None:
    shards = sorted(directory.glob("*.safetensors"))
    if not shards:
        raise AttnRankError(f"no *.safetensors shards in '{directory}'")
    for shard in shards:
        for name, array, code in iter_tensors(shard):
            engine.load_tensor(name, array, code)


def write_safetensors(path: Path, tensors: dict[str, tuple[np.ndarray, str]]) -> None:
    """Write {name: (array, dtype tag)} as one shard; bf16 arrays are given as uint16 bit patterns."""
    header, offset, blobs = {}, 0, []
    for name, (array, tag) in tensors.items():
        blob = np.ascontiguousarray(array).tobytes()
        header[name] = {"dtype": tag, "shape": list(array.shape), "data_offsets": [offset, offset + len(blob)]}
        offset += len(blob)
        blobs.append(blob)
    encoded = json.dumps(header).encode()
    encoded += b" " * ((8 - len(encoded) % 8) % 8)
    with open(path, "wb") as handle:
        handle.write(struct.pack("<Q", len(encoded)))
        handle.write(encoded)
        for blob in blobs:
            handle.write(blob)

"""Hugging Face checkpoint I/O for the engine: safetensors and PyTorch-archive shards in, safetensors out.

The reference selects a directory's shards (CheckpointLoader::select_shards, attnrank/src/
checkpoint.cpp:151-176): every `*.safetensors` file, or when there is none every
`pytorch_model*.bin` archive, in sorted order; a later shard's tensor replaces an earlier one of
the same name (WeightRegistry::add_source, :33-40). It maps each shard (:67-122 for safetensors,
with the header checks restated in `_safetensors_tensors`) and uploads every tensor it needs by
its Hugging Face name (model.cu:113-174). This module does the same from Python and hands each
16-bit or fp32 tensor to the native engine (ar_engine_load_tensor), which converts it to the
resident layout. Integer and bool tensors are accepted, as the reference's registry accepts them
(core.cpp:56-67), and skipped: no weight of the model has those types.

PyTorch archives are read with `torch.load(weights_only=True)`, a restricted unpickler that
rebuilds tensors and plain containers only, as the reference's own archive reader does
(checkpoint.cpp:236-886).
"""
from __future__ import annotations

import json
import struct
from pathlib import Path
from typing import Iterator

import numpy as np

from attnrank import _native
from attnrank._native import AttnRankError

# safetensors dtype -> (numpy view type, engine dtype code); None: accepted, never uploaded
_DTYPES = {
    "F32": (np.float32, _native.DTYPE_F32),
    "F16": (np.uint16, _native.DTYPE_F16),
    "BF16": (np.uint16, _native.DTYPE_BF16),
    "I64": (np.int64, None), "U64": (np.uint64, None),
    "I32": (np.int32, None), "U32": (np.uint32, None),
    "I16": (np.int16, None), "U16": (np.uint16, None),
    "I8": (np.int8, None), "U8": (np.uint8, None),
    "BOOL": (np.bool_, None),
}
_BIAS_SUFFIXES = ("self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias")


def select_shards(directory: Path) -> list[Path]:
    """The weight shards of a checkpoint directory (checkpoint.cpp:151-176)."""
    directory = Path(directory)
    if not directory.is_dir():
        raise AttnRankError(f"model path is not a directory: '{directory}'")
    files = [entry for entry in directory.iterdir() if entry.is_file()]
    safetensors = [entry for entry in files if entry.name.endswith(".safetensors")]
    archives = [entry for entry in files if entry.name.endswith(".bin") and entry.name.startswith("pytorch_model")]
    selected = safetensors or archives
    if not selected:
        raise AttnRankError(f"no weight shards (*.safetensors or pytorch_model*.bin) under '{directory}'")
    return sorted(selected, key=str)


def read_header(path: Path) -> tuple[dict, int]:
    """The JSON header of a safetensors file and the byte offset of its data section."""
    size = Path(path).stat().st_size
    if size < 8:
        raise AttnRankError(f"safetensors file too small: '{path}'")
    with open(path, "rb") as handle:
        (length,) = struct.unpack("<Q", handle.read(8))
        if length == 0 or length > size - 8:
            raise AttnRankError(f"invalid safetensors header length in '{path}'")
        try:
            header = json.loads(handle.read(length))
        except ValueError as error:
            raise AttnRankError(f"invalid safetensors header in '{path}': {error}") from None
    if not isinstance(header, dict):
        raise AttnRankError("safetensors header is not an object")
    return header, 8 + length


def _safetensors_tensors(path: Path, uploadable_only: bool) -> Iterator[tuple[str, np.ndarray, int | None]]:
    header, data_origin = read_header(path)
    size = Path(path).stat().st_size
    mapped = np.memmap(path, dtype=np.uint8, mode="r") if size > data_origin else np.zeros(0, np.uint8)
    for name, entry in header.items():
        if name == "__metadata__":
            continue
        kind = entry.get("dtype")
        if kind not in _DTYPES:
            raise AttnRankError(f"unsupported dtype '{kind}' for tensor '{name}'")
        numpy_type, code = _DTYPES[kind]
        offsets = entry.get("data_offsets")
        if not isinstance(offsets, list) or len(offsets) != 2:
            raise AttnRankError(f"bad data_offsets for tensor '{name}'")
        begin, end = int(offsets[0]), int(offsets[1])
        if end < begin:
            raise AttnRankError(f"inverted data_offsets for tensor '{name}'")
        if begin < 0 or data_origin + end > size:
            raise AttnRankError(f"tensor '{name}' lies outside '{path}'")
        shape = [int(extent) for extent in entry.get("shape", [])]
        if int(np.prod(shape, dtype=np.int64)) * np.dtype(numpy_type).itemsize != end - begin:
            raise AttnRankError(f"tensor '{name}' byte size mismatch")
        if code is None and uploadable_only:
            continue
        yield name, mapped[data_origin + begin:data_origin + end].view(numpy_type).reshape(shape), code


def _torch_archive_tensors(path: Path, uploadable_only: bool) -> Iterator[tuple[str, np.ndarray, int | None]]:
    import torch

    try:
        state = torch.load(path, map_location="cpu", weights_only=True, mmap=True)
    except Exception as error:  # noqa: BLE001 - any unreadable archive is a checkpoint error
        raise AttnRankError(f"cannot read torch archive '{path}': {error}") from None
    if not isinstance(state, dict):
        raise AttnRankError(f"'{path}' does not contain a state dict")
    for name, tensor in state.items():
        if not isinstance(tensor, torch.Tensor):
            continue
        tensor = tensor.detach().contiguous()
        if tensor.dtype == torch.float32:
            yield name, tensor.numpy(), _native.DTYPE_F32
        elif tensor.dtype in (torch.float16, torch.bfloat16):
            bits = tensor.view(torch.int16).numpy().view(np.uint16)
            yield name, bits, _native.DTYPE_F16 if tensor.dtype == torch.float16 else _native.DTYPE_BF16
        elif tensor.dtype in (torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8, torch.bool):
            if not uploadable_only:
                yield name, tensor.numpy(), None
        else:
            raise AttnRankError(f"unsupported dtype '{tensor.dtype}' for tensor '{name}'")


def iter_tensors(path: Path, uploadable_only: bool = True) -> Iterator[tuple[str, np.ndarray, int | None]]:
    """(name, array view, engine dtype code) for every tensor of one shard; with
    `uploadable_only`, the fp32 / fp16 / bf16 ones (16-bit values as uint16 bit patterns)."""
    path = Path(path)
    if path.name.endswith(".safetensors"):
        return _safetensors_tensors(path, uploadable_only)
    if path.suffix in (".bin", ".pth", ".pt"):
        return _torch_archive_tensors(path, uploadable_only)
    raise AttnRankError(f"no registered loader accepts shard '{path}'")


def tensor_names(directory: Path) -> set[str]:
    """Names of every tensor the directory's shards hold (safetensors: headers only)."""
    names: set[str] = set()
    for shard in select_shards(directory):
        if shard.name.endswith(".safetensors"):
            names.update(name for name in read_header(shard)[0] if name != "__metadata__")
        else:
            names.update(name for name, _, _ in _torch_archive_tensors(shard, uploadable_only=False))
    return names


def has_attention_bias(directory: Path) -> bool:
    """Whether the checkpoint holds q/k/v projection biases. The reference uploads them whenever
    they are present and skips them otherwise (optional_floating, model.cu:160-162), whatever
    config.json says."""
    return any(name.endswith(_BIAS_SUFFIXES) for name in tensor_names(directory))


def load_directory(engine, directory: Path) -> None:
    for shard in select_shards(directory):
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

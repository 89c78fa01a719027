"""Checkpoint reading on the host (attnrank/checkpoint.py), no GPU: shard selection, safetensors
header checks, PyTorch archives and the presence test for q/k/v biases, against the behaviour of
the reference's CheckpointLoader (attnrank/src/checkpoint.cpp:67-216)."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest
import torch

from attnrank import _native
from attnrank.checkpoint import (has_attention_bias, iter_tensors, load_directory, select_shards, tensor_names,
                                 write_safetensors)
from attnrank._native import AttnRankError


def _tensors():
    rng = np.random.default_rng(0)
    weight = rng.standard_normal((6, 4)).astype(np.float32)
    return {
        "model.layers.0.self_attn.q_proj.weight": torch.from_numpy(weight).to(torch.bfloat16),
        "model.layers.0.self_attn.q_proj.bias": torch.from_numpy(weight[0]).clone(),
        "model.norm.weight": torch.from_numpy(weight[1]).to(torch.float16),
        "model.position_ids": torch.arange(5, dtype=torch.int64),
        "model.mask": torch.tensor([True, False]),
    }


def _as_safetensors(tensors):
    out = {}
    for name, tensor in tensors.items():
        if tensor.dtype == torch.bfloat16:
            out[name] = (tensor.view(torch.int16).numpy().view(np.uint16), "BF16")
        elif tensor.dtype == torch.float16:
            out[name] = (tensor.numpy().view(np.uint16), "F16")
        elif tensor.dtype == torch.float32:
            out[name] = (tensor.numpy(), "F32")
        elif tensor.dtype == torch.int64:
            out[name] = (tensor.numpy(), "I64")
        else:
            out[name] = (tensor.numpy(), "BOOL")
    return out


def _uploadable(path):
    return {name: (np.array(array), code) for name, array, code in iter_tensors(path)}


def test_shard_selection_follows_the_reference(tmp_path):
    with pytest.raises(AttnRankError, match="not a directory"):
        select_shards(tmp_path / "missing")
    (tmp_path / "training_args.bin").write_bytes(b"x")
    with pytest.raises(AttnRankError, match=r"no weight shards \(\*\.safetensors or pytorch_model\*\.bin\)"):
        select_shards(tmp_path)
    torch.save({}, tmp_path / "pytorch_model-00002-of-00002.bin")
    torch.save({}, tmp_path / "pytorch_model-00001-of-00002.bin")
    assert [p.name for p in select_shards(tmp_path)] == ["pytorch_model-00001-of-00002.bin",
                                                        "pytorch_model-00002-of-00002.bin"]
    write_safetensors(tmp_path / "model-00002.safetensors", {})
    write_safetensors(tmp_path / "model-00001.safetensors", {})
    assert [p.name for p in select_shards(tmp_path)] == ["model-00001.safetensors", "model-00002.safetensors"]


def test_safetensors_and_torch_archive_give_the_same_tensors(tmp_path):
    tensors = _tensors()
    safetensors_dir, archive_dir = tmp_path / "st", tmp_path / "pt"
    safetensors_dir.mkdir()
    archive_dir.mkdir()
    write_safetensors(safetensors_dir / "model.safetensors", _as_safetensors(tensors))
    torch.save(tensors, archive_dir / "pytorch_model.bin")
    from_safetensors = _uploadable(safetensors_dir / "model.safetensors")
    from_archive = _uploadable(archive_dir / "pytorch_model.bin")
    # integer and bool tensors are accepted and never uploaded
    assert set(from_safetensors) == set(from_archive) == {
        "model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.q_proj.bias", "model.norm.weight"}
    for name, (array, code) in from_safetensors.items():
        other, other_code = from_archive[name]
        assert code == other_code
        np.testing.assert_array_equal(array, other)
    assert from_safetensors["model.layers.0.self_attn.q_proj.weight"][1] == _native.DTYPE_BF16
    assert from_safetensors["model.norm.weight"][1] == _native.DTYPE_F16
    assert from_safetensors["model.layers.0.self_attn.q_proj.bias"][1] == _native.DTYPE_F32
    bias = torch.from_numpy(from_safetensors["model.layers.0.self_attn.q_proj.bias"][0])
    assert torch.equal(bias, tensors["model.layers.0.self_attn.q_proj.bias"])
    every = {name for name, _, _ in iter_tensors(safetensors_dir / "model.safetensors", uploadable_only=False)}
    assert every == set(tensors) == tensor_names(safetensors_dir) == tensor_names(archive_dir)


def test_attention_bias_is_decided_by_the_checkpoint(tmp_path):
    tensors = _tensors()
    write_safetensors(tmp_path / "model.safetensors", _as_safetensors(tensors))
    assert has_attention_bias(tmp_path)
    del tensors["model.layers.0.self_attn.q_proj.bias"]
    (tmp_path / "model.safetensors").unlink()
    torch.save(tensors, tmp_path / "pytorch_model.bin")
    assert not has_attention_bias(tmp_path)


def test_later_shards_replace_earlier_tensors(tmp_path):
    write_safetensors(tmp_path / "a.safetensors", {"w": (np.array([1.0], np.float32), "F32")})
    write_safetensors(tmp_path / "b.safetensors", {"w": (np.array([2.0], np.float32), "F32")})

    class Recorder:
        def __init__(self):
            self.values = {}

        def load_tensor(self, name, array, code):
            self.values[name] = float(np.asarray(array)[0])

    recorder = Recorder()
    load_directory(recorder, tmp_path)
    assert recorder.values == {"w": 2.0}


def _raw_shard(path, header: dict | bytes, data: bytes = b"", length: int | None = None):
    encoded = header if isinstance(header, bytes) else json.dumps(header).encode()
    with open(path, "wb") as handle:
        handle.write(struct.pack("<Q", len(encoded) if length is None else length))
        handle.write(encoded)
        handle.write(data)


@pytest.mark.parametrize("header,data,length,message", [
    (b"", b"", None, "too small"),
    ({"w": {"dtype": "F32", "shape": [1], "data_offsets": [0, 4]}}, b"\0" * 4, 10 ** 6, "header length"),
    ([1, 2], b"", None, "not an object"),
    ({"w": {"dtype": "F64", "shape": [1], "data_offsets": [0, 8]}}, b"\0" * 8, None, "unsupported dtype 'F64'"),
    ({"w": {"dtype": "F32", "shape": [1], "data_offsets": [0]}}, b"\0" * 4, None, "bad data_offsets"),
    ({"w": {"dtype": "F32", "shape": [1], "data_offsets": [4, 0]}}, b"\0" * 4, None, "inverted data_offsets"),
    ({"w": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}, b"\0" * 4, None, "byte size mismatch"),
    ({"w": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, b"\0" * 4, None, "lies outside"),
])
def test_corrupt_safetensors_are_reported(tmp_path, header, data, length, message):
    path = tmp_path / "model.safetensors"
    if header == b"":
        path.write_bytes(b"\1\2\3")
    else:
        _raw_shard(path, header, data, length)
    with pytest.raises(AttnRankError, match=message):
        list(iter_tensors(path))


class _NotATensor:
    pass


def test_torch_archives_are_read_without_running_pickled_code(tmp_path):
    """weights_only: an archive that pickles an arbitrary object is refused, not executed."""
    torch.save({"w": torch.zeros(2), "extra": _NotATensor()}, tmp_path / "pytorch_model.bin")
    with pytest.raises(AttnRankError, match="cannot read torch archive"):
        list(iter_tensors(tmp_path / "pytorch_model.bin"))
    torch.save([torch.zeros(2)], tmp_path / "pytorch_model.bin")
    with pytest.raises(AttnRankError, match="does not contain a state dict"):
        list(iter_tensors(tmp_path / "pytorch_model.bin"))
    with pytest.raises(AttnRankError, match="no registered loader"):
        iter_tensors(tmp_path / "weights.npz")


def test_a_torch_archive_directory_is_a_model_directory(tmp_path):
    """is_model_directory (reference engine.py:79-82): config.json plus safetensors or
    pytorch_model*.bin shards."""
    import attnrank as ar
    (tmp_path / "config.json").write_text("{}")
    assert not ar.is_model_directory(path=tmp_path)
    torch.save({}, tmp_path / "pytorch_model.bin")
    assert ar.is_model_directory(path=tmp_path)

"""Loading a Hugging Face checkpoint directory (ar.from_pretrained) through the C ABI.

The seeded synthetic weights are written as a safetensors checkpoint with the reference's tensor
names (model.cu:120-166) and a config.json, then loaded with `from_pretrained`, which reads each
shard and uploads every tensor with ar_engine_load_tensor. That is host data -> device, with the
engine's conversions: bf16 or fp32 matrices -> fp16 by round-to-nearest-even, fp32 biases and
norms, and the fp16 copy of the q|k|v bias used by the GEMM epilogue. The engine built on the
synthetic generator converts the same values by the same rule. The two engines may still pick
different cuBLASLt algorithms (each times its candidates), which changes GEMM rounding in the last
bits, so rows are compared at rel 1e-4: a wrong tensor, shape or conversion moves them by O(1).
"""
from __future__ import annotations

import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _config():
    import attnrank as ar
    return ar.LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                          num_key_value_heads=2, vocab_size=2000, max_position_embeddings=4096, rms_norm_eps=1e-6,
                          rope_theta=1e6, attention_bias=True)


def _write_checkpoint(directory, config, matrix_dtype: str) -> None:
    """Every tensor the reference uploads, from the seeded generator (seed 0, std 0.02)."""
    from attnrank.checkpoint import write_safetensors
    from oracle import weights as W

    H, I, V = config.hidden_size, config.intermediate_size, config.vocab_size
    Hq, Hkv = config.num_attention_heads, config.num_key_value_heads
    D = H // Hq
    seed, std = 0, 0.02

    def matrix(rows, cols, layer, kind):
        bits = W.bf16_bits(rows * cols, seed, layer, kind, std).reshape(rows, cols)
        if matrix_dtype == "BF16":
            return bits, "BF16"
        return W.bf16_to_f32(bits), "F32"

    def vector(count, layer, kind, scale, offset=0.0):
        return W.f32(count, seed, layer, kind, scale, offset).astype(np.float32), "F32"

    tensors = {"model.embed_tokens.weight": matrix(V, H, -1, W.EMBEDDING),
               "model.norm.weight": vector(H, -1, W.FINAL_NORM, 0.0, 1.0),
               "lm_head.weight": matrix(V, H, -1, W.LM_HEAD)}
    for layer in range(config.num_hidden_layers):
        prefix = f"model.layers.{layer}."
        tensors[prefix + "self_attn.q_proj.weight"] = matrix(Hq * D, H, layer, W.QUERY)
        tensors[prefix + "self_attn.k_proj.weight"] = matrix(Hkv * D, H, layer, W.KEY)
        tensors[prefix + "self_attn.v_proj.weight"] = matrix(Hkv * D, H, layer, W.VALUE)
        tensors[prefix + "self_attn.q_proj.bias"] = vector(Hq * D, layer, W.QUERY_BIAS, std)
        tensors[prefix + "self_attn.k_proj.bias"] = vector(Hkv * D, layer, W.KEY_BIAS, std)
        tensors[prefix + "self_attn.v_proj.bias"] = vector(Hkv * D, layer, W.VALUE_BIAS, std)
        tensors[prefix + "self_attn.o_proj.weight"] = matrix(H, Hq * D, layer, W.OUTPUT)
        tensors[prefix + "mlp.gate_proj.weight"] = matrix(I, H, layer, W.GATE)
        tensors[prefix + "mlp.up_proj.weight"] = matrix(I, H, layer, W.UP)
        tensors[prefix + "mlp.down_proj.weight"] = matrix(H, I, layer, W.DOWN)
        tensors[prefix + "input_layernorm.weight"] = vector(H, layer, W.INPUT_NORM, 0.0, 1.0)
        tensors[prefix + "post_attention_layernorm.weight"] = vector(H, layer, W.POST_NORM, 0.0, 1.0)
    write_safetensors(directory / "model.safetensors", tensors)
    (directory / "config.json").write_text(json.dumps({
        "model_type": "qwen2", "hidden_size": H, "intermediate_size": I,
        "num_hidden_layers": config.num_hidden_layers, "num_attention_heads": Hq, "num_key_value_heads": Hkv,
        "vocab_size": V, "max_position_embeddings": config.max_position_embeddings,
        "rms_norm_eps": config.rms_norm_eps, "rope_theta": config.rope_theta}))


@pytest.mark.parametrize("matrix_dtype", ["BF16", "F32"])
def test_from_pretrained_equals_synthetic_engine(cuda, tmp_path, matrix_dtype):
    import attnrank as ar
    from attnrank import synthetic
    config = _config()
    _write_checkpoint(tmp_path, config, matrix_dtype)
    loaded = ar.from_pretrained(model=tmp_path)
    assert loaded.config.attention_bias and loaded.num_layers == config.num_hidden_layers
    reference = ar.Engine.synthetic(config, seed=0)
    shape = synthetic.PromptShape(documents=5, document_min=20, document_max=90, question=12)
    prompts = synthetic.prompts(4, config.vocab_size, shape, seed=8)
    got, _ = loaded.probe_rows(prompts)
    want, _ = reference.probe_rows(prompts)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-9)
    loaded.close()
    reference.close()


def test_from_pretrained_reads_a_torch_archive_and_finds_its_biases(cuda, tmp_path):
    """The same weights as a pytorch_model.bin archive (the reference's fallback when a directory
    has no safetensors, checkpoint.cpp:157-172), with a config.json that names no attention bias
    (model_type "llama"): the biases are used because the checkpoint holds them, as the
    reference's optional bias upload does (model.cu:160-162)."""
    import torch

    import attnrank as ar
    from attnrank import synthetic
    from attnrank.checkpoint import iter_tensors
    config = _config()
    _write_checkpoint(tmp_path, config, "BF16")
    shard = tmp_path / "model.safetensors"
    state = {}
    for name, array, code in iter_tensors(shard):
        values = torch.from_numpy(np.array(array))
        state[name] = values.view(torch.bfloat16) if code == 2 else values
    shard.unlink()
    torch.save(state, tmp_path / "pytorch_model.bin")
    settings = json.loads((tmp_path / "config.json").read_text())
    settings["model_type"] = "llama"
    (tmp_path / "config.json").write_text(json.dumps(settings))
    assert not ar.LlamaConfig.from_file(tmp_path / "config.json").attention_bias
    loaded = ar.from_pretrained(model=tmp_path)
    assert loaded.config.attention_bias
    reference = ar.Engine.synthetic(config, seed=0)
    shape = synthetic.PromptShape(documents=5, document_min=20, document_max=90, question=12)
    prompts = synthetic.prompts(3, config.vocab_size, shape, seed=8)
    got, _ = loaded.probe_rows(prompts)
    want, _ = reference.probe_rows(prompts)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-9)
    loaded.close()
    reference.close()


def test_from_pretrained_reports_a_missing_tensor(cuda, tmp_path):
    import attnrank as ar
    from attnrank import synthetic
    from attnrank.checkpoint import iter_tensors, write_safetensors
    config = _config()
    _write_checkpoint(tmp_path, config, "BF16")
    shard = tmp_path / "model.safetensors"
    kept = {}
    for name, array, code in iter_tensors(shard):
        if name != "model.layers.1.mlp.down_proj.weight":
            kept[name] = (np.array(array), {0: "F32", 1: "F16", 2: "BF16"}[code])
    shard.unlink()
    write_safetensors(shard, kept)
    engine = ar.from_pretrained(model=tmp_path)
    prompt = synthetic.prompts(1, config.vocab_size,
                               synthetic.PromptShape(documents=5, document_min=20, document_max=40, question=8))[0]
    with pytest.raises(ar.AttnRankError, match="down_proj"):
        engine.measure_attention_by_layer(prompt)
    engine.close()

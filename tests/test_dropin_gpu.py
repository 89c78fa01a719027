"""The drop-in, run on a B200: the reference's own layer scan over this library.

INTEGRATION.md gives a reference maintainer one class, B200AttentionProvider, an IAttentionProvider
(include/attnrank/model.hpp:79-86) over this library's C ABI. oracle/Makefile compiles that class
from the document's code against the reference's headers, with a small harness, into
oracle/_ref/libb200_provider_ref.so, linked with the reference's compiled sources. Here the
reference's unchanged AttentionLayerScanner::scan (attnrank/src/attnrank.cpp:364-375) and
select_shallowest_basin_layer (:257-265) run over that provider on the Qwen2.5-7B architecture,
and their result is compared with the same scanner over the reference's own CudaLlamaModel:
every layer's mass row (rel 1e-3), slot order and the pick (exact).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
PROVIDER_LIBRARY = ROOT / "oracle" / "_ref" / "libb200_provider_ref.so"


def _provider_lib():
    from oracle import reference
    if reference.load_or_none() is None or not PROVIDER_LIBRARY.exists():
        pytest.skip("oracle/_ref is not built (make -C oracle reference provider)")
    lib = ctypes.CDLL(str(PROVIDER_LIBRARY))
    P, I, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
    lib.prov_last_error.restype = ctypes.c_char_p
    lib.prov_create.argtypes = [ctypes.POINTER(reference.RefConfig), ctypes.c_uint64, D, I, I, I]
    lib.prov_create.restype = P
    lib.prov_destroy.argtypes = [P]
    lib.prov_destroy.restype = None
    lib.prov_scan.argtypes = [P, ctypes.POINTER(reference.RefPrompt), I, I, I, I, I, D, P, P, P, P, P, P]
    return lib


@pytest.mark.slow
def test_reference_scanner_over_the_b200_provider_matches_its_own_model(cuda):
    from attnrank import synthetic
    from oracle import reference
    lib = _provider_lib()
    config = synthetic.qwen2_7b()
    prompts = synthetic.prompts(48, config.vocab_size)
    c = reference.RefConfig(config.hidden_size, config.intermediate_size, config.num_hidden_layers,
                            config.num_attention_heads, config.num_key_value_heads, config.vocab_size,
                            config.rms_norm_eps, config.rope_theta, config.sliding_window, int(config.attention_bias))
    provider = lib.prov_create(ctypes.byref(c), 0, 0.02, 2048, 512, 0)
    assert provider, lib.prov_last_error().decode()
    packed = reference._Prompts(prompts)
    L, S = config.num_hidden_layers, packed.span_count
    attention = np.zeros((L, S), dtype=np.float64)
    order = np.zeros((L, S), dtype=np.int32)
    layer_index = np.zeros(L, dtype=np.int32)
    count, selected, seconds = ctypes.c_int(), ctypes.c_int(), ctypes.c_double()
    try:
        status = lib.prov_scan(provider, packed.array, len(prompts), S, 0, -1, 0, 1.3, attention.ctypes.data,
                               order.ctypes.data, layer_index.ctypes.data, ctypes.byref(count), ctypes.byref(selected),
                               ctypes.byref(seconds))
        assert status == 0, lib.prov_last_error().decode()
    finally:
        lib.prov_destroy(provider)
    assert count.value == L
    model = reference.ReferenceModel(config, seed=0, max_sequence_length=2048)
    try:
        want = model.scan(prompts, min_edge_ratio=1.3)
    finally:
        model.close()
    assert selected.value == want.selected_layer
    np.testing.assert_array_equal(layer_index, want.layer_index)
    error = np.abs(attention - want.attention) / np.abs(want.attention)
    assert error.max() <= 1e-3, error.max()
    np.testing.assert_array_equal(order, want.position_order)

"""The C-ABI library loads on any host and exports every symbol include/attnrank_b200.h declares."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "attnrank_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ar_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ["ar_embedding_rms_norm", "ar_rms_norm_residual", "ar_rotary_embedding", "ar_silu_multiply",
                     "ar_causal_attention", "ar_document_attention_mass", "ar_engine_create",
                     "ar_engine_measure_attention_by_layer", "ar_engine_scan", "ar_profile_from_accumulated",
                     "ar_basin_statistics", "ar_select_shallowest_basin_layer", "ar_resolve_position_order"]:
        assert required in names


def test_library_exports_every_declared_symbol():
    from attnrank import _native
    library = ctypes.CDLL(str(_native.LIBRARY_PATH))
    missing = [name for name in declared_functions() if not hasattr(library, name)]
    assert not missing, f"symbols declared but not exported: {missing}"
    # and the Python binding covers all of them
    assert set(declared_functions()) <= set(_native.SIGNATURES)


def test_library_is_sm100a_build():
    from attnrank import _native
    assert "sm_100a" in _native.version()


def test_engine_creation_without_gpu_fails_loudly():
    """No CPU fallback: without a CUDA device the engine refuses to start."""
    import pytest

    import attnrank as ar
    from conftest import has_gpu
    if has_gpu():
        pytest.skip("a GPU is present")
    config = ar.LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=1, num_attention_heads=4,
                            num_key_value_heads=2, vocab_size=100)
    with pytest.raises(ar.AttnRankError):
        ar.Engine.synthetic(config)

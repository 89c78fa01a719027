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


def _c_declarations(text: str) -> str:
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.sub(r"//[^\n]*", "", text)


def _ctype_of(declaration: str):
    """ctypes class of one C parameter or field declaration (the name dropped)."""
    if "*" in declaration:
        return "pointer"
    kind = declaration.replace("const", " ").split()[0]
    return {"int": ctypes.c_int, "int32_t": ctypes.c_int32, "int64_t": ctypes.c_int64, "uint64_t": ctypes.c_uint64,
            "uint32_t": ctypes.c_uint32,
            "float": ctypes.c_float, "double": ctypes.c_double}[kind]


def _same(expected, actual) -> bool:
    if expected == "pointer":
        return actual in (ctypes.c_void_p, ctypes.c_char_p) or hasattr(actual, "_type_") and actual.__name__.startswith("LP_")
    return ctypes.sizeof(actual) == ctypes.sizeof(expected) and actual._type_ == expected._type_


def test_python_binding_argument_types_match_the_header():
    """Every ctypes argtypes list has the header's arity and, position by position, its C types
    (a float passed where the library takes a double, or an int where it takes int64_t, would
    read garbage without any error)."""
    from attnrank import _native
    text = _c_declarations(HEADER.read_text())
    prototypes = re.findall(r"\b(ar_[a-z0-9_]+)\s*\(([^;{)]*)\)\s*;", text)
    assert len(prototypes) == len(declared_functions())
    for name, parameters in prototypes:
        parameters = parameters.strip()
        declared = [] if parameters in ("", "void") else [p.strip() for p in parameters.split(",")]
        bound = _native.SIGNATURES[name]
        assert len(bound) == len(declared), f"{name}: {len(bound)} ctypes arguments, {len(declared)} in the header"
        for index, (c_declaration, ctype) in enumerate(zip(declared, bound)):
            assert _same(_ctype_of(c_declaration), ctype), f"{name} argument {index}: `{c_declaration}` vs {ctype}"


def test_python_structures_match_the_header_layout():
    """Field order, types and size of each ctypes Structure against its typedef struct."""
    from attnrank import _native
    text = _c_declarations(HEADER.read_text())
    structures = {"ar_llama_config": _native.LlamaConfigStruct, "ar_runtime_options": _native.RuntimeOptionsStruct,
                  "ar_prompt": _native.PromptStruct, "ar_sampler_config": _native.SamplerConfigStruct,
                  "ar_basin_stats": _native.BasinStatsStruct}
    for c_name, structure in structures.items():
        body = re.search(r"typedef struct\s*\{([^}]*)\}\s*" + c_name + r"\s*;", text)
        assert body, c_name
        fields = [f.strip() for f in body.group(1).split(";") if f.strip()]
        assert [f.split()[-1].lstrip("*") for f in fields] == [n for n, _ in structure._fields_], c_name
        for c_field, (field_name, ctype) in zip(fields, structure._fields_):
            assert _same(_ctype_of(c_field), ctype), f"{c_name}.{field_name}: `{c_field}` vs {ctype}"

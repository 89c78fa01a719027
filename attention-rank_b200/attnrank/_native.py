"""ctypes binding of libattnrank_b200.so (C ABI declared in include/attnrank_b200.h).

The shared library is the product: every probe runs through its CUDA kernels. There is no
Python or CPU fallback; if the library is missing, importing this module raises ImportError with
the build command.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIBRARY_PATH = Path(__file__).resolve().parent / "libattnrank_b200.so"

AR_OK = 0
AR_ERR_INVALID = 1
AR_ERR_CUDA = 2
AR_ERR_DEVICE = 3
AR_ERR_INTERNAL = 4

DTYPE_F32, DTYPE_F16, DTYPE_BF16 = 0, 1, 2
KERNEL_CLASS_COUNT = 12  # AR_KERNEL_CLASS_COUNT


class AttnRankError(RuntimeError):
    """Raised for every failure reported by the native library (reference: _core.AttnRankError)."""


class LlamaConfigStruct(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_int),
        ("intermediate_size", ctypes.c_int),
        ("num_hidden_layers", ctypes.c_int),
        ("num_attention_heads", ctypes.c_int),
        ("num_key_value_heads", ctypes.c_int),
        ("vocab_size", ctypes.c_int),
        ("max_position_embeddings", ctypes.c_int),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("sliding_window", ctypes.c_int),
        ("attention_bias", ctypes.c_int),
        ("tie_word_embeddings", ctypes.c_int),
    ]


class RuntimeOptionsStruct(ctypes.Structure):
    _fields_ = [
        ("device_index", ctypes.c_int),
        ("max_sequence_length", ctypes.c_int),
        ("prefill_chunk_tokens", ctypes.c_int),
        ("max_batch_tokens", ctypes.c_int),
        ("max_batch_prompts", ctypes.c_int),
        ("activation_dtype", ctypes.c_int),
        ("attention_kernel", ctypes.c_int),
    ]


class SamplerConfigStruct(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("top_p", ctypes.c_float),
        ("top_k", ctypes.c_int),
        ("seed", ctypes.c_uint64),
    ]


class PromptStruct(ctypes.Structure):
    _fields_ = [
        ("tokens", ctypes.c_void_p),
        ("token_count", ctypes.c_int),
        ("query_begin", ctypes.c_int),
        ("query_end", ctypes.c_int),
        ("spans", ctypes.c_void_p),
    ]


class BasinStatsStruct(ctypes.Structure):
    _fields_ = [
        ("first", ctypes.c_double),
        ("last", ctypes.c_double),
        ("interior_mean", ctypes.c_double),
        ("edge_ratio", ctypes.c_double),
        ("is_basin", ctypes.c_int),
    ]


_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_U64 = ctypes.c_uint64
_F = ctypes.c_float
_D = ctypes.c_double

# name -> argument types (all return int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "ar_last_error": [],
    "ar_version": [],
    "ar_embedding_rms_norm": [_P, _I, _P, _I, _I, _P, _F, _P, _P, _P, _I, _P],
    "ar_rms_norm_residual": [_P, _P, _P, _I, _I, _F, _P, _I, _P],
    "ar_rotary_embedding": [_P, _P, _P, _I, _I, _I, _I, _P, _P, _I, _P, _I, _P],
    "ar_rope_table": [_P, _P, _I, _I, _F, _P],
    "ar_silu_multiply": [_P, _P, _I64, _P, _I64, _I, _I, _I, _P],
    "ar_causal_attention": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "ar_causal_attention_mma": [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _I, _P],
    "ar_document_attention_mass": [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _P],
    "ar_document_attention_mass_noalloc": [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I, _I, _I, _I, _I, _P, _I, _P],
    "ar_synthetic_fill": [_P, _I64, _U64, _I, _I, _F, _I, _P],
    "ar_engine_create": [ctypes.POINTER(LlamaConfigStruct), ctypes.POINTER(RuntimeOptionsStruct), ctypes.POINTER(_P)],
    "ar_engine_destroy": [_P],
    "ar_engine_load_tensor": [_P, ctypes.c_char_p, _I, _P, _I, _P],
    "ar_engine_init_synthetic": [_P, _U64, _F],
    "ar_engine_measure_attention_by_layer": [_P, ctypes.POINTER(PromptStruct), _I, _I, _I, _I, _I, _P, _P, _P],
    "ar_engine_measure_attention": [_P, ctypes.POINTER(PromptStruct), _I, _I, _I, _I, _P],
    "ar_engine_scan": [_P, ctypes.POINTER(PromptStruct), _I, _I, _I, _I, _I, _P, _P],
    "ar_engine_prepare_scan": [_P, ctypes.POINTER(PromptStruct), _I, _I, _I, _I, _I, ctypes.POINTER(_P)],
    "ar_engine_run_prepared_scan": [_P, _P, _P, _I],
    "ar_prepared_scan_destroy": [_P],
    "ar_prepared_scan_bytes": [_P],
    "ar_engine_synchronize": [_P],
    "ar_engine_set_kernel_timing": [_P, _I],
    "ar_engine_kernel_timing": [_P, _P, _P, _P],
    "ar_kernel_class_name": [_I],
    "ar_kernel_class_is_tensor": [_I],
    "ar_engine_stream": [_P],
    "ar_engine_device": [_P],
    "ar_engine_generate": [_P, _P, _I, _I, _I, ctypes.POINTER(SamplerConfigStruct), _P, _P],
    "ar_engine_generation_begin": [_P, _P, _I, _P],
    "ar_engine_generation_step": [_P, ctypes.c_int32, _P],
    "ar_engine_generation_position": [_P],
    "ar_engine_decode_mode": [_P],
    "ar_sampler_create": [ctypes.POINTER(SamplerConfigStruct), ctypes.POINTER(_P)],
    "ar_sampler_select": [_P, _P, _I, _P],
    "ar_sampler_destroy": [_P],
    "ar_decode_gemv": [_P, _P, _I, _I, _P, _I, _I, _P],
    "ar_decode_gate_up": [_P, _P, _I, _I, _P, _I, _P],
    "ar_decode_attention": [_P, _P, _P, _I, _I, _I, _I, _I, _I, _P, _I, _P],
    "ar_bounded_wait_selftest": [_I, ctypes.c_uint32, _P],
    "ar_profile_from_accumulated": [_P, _I, _I64, _P, _P],
    "ar_position_order": [_P, _I, _P],
    "ar_basin_statistics": [_P, _I, _D, ctypes.POINTER(BasinStatsStruct)],
    "ar_select_shallowest_basin_layer": [_P, _P, _I, _I, _D, _P],
    "ar_resolve_position_order": [_P, _I, _I, _P],
}
_RESTYPES = {
    "ar_last_error": ctypes.c_char_p,
    "ar_version": ctypes.c_char_p,
    "ar_engine_destroy": None,
    "ar_prepared_scan_destroy": None,
    "ar_sampler_destroy": None,
    "ar_prepared_scan_bytes": ctypes.c_int64,
    "ar_kernel_class_name": ctypes.c_char_p,
    "ar_engine_stream": ctypes.c_void_p,
    "ar_engine_device": ctypes.c_int,
}


def _load_cublas_once() -> None:
    """One process must hold one cuBLAS. When PyTorch is installed, its bundled cuBLAS and cuBLASLt
    are loaded first, so that this library's libcublasLt.so.12 resolves to that same copy: the
    dynamic linker reuses a loaded soname, and a CUDA-toolkit cuBLASLt of another version loaded
    first under the same name makes torch's own cuBLAS calls fail (CUBLAS_STATUS_INVALID_VALUE)."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass


def _load() -> ctypes.CDLL:
    _load_cublas_once()
    if not LIBRARY_PATH.exists():
        raise ImportError(
            f"{LIBRARY_PATH.name} is not built; run `make -C attention-rank_b200/csrc` "
            "(or __graft_entry__.build()) on a machine with nvcc 12.9"
        )
    library = ctypes.CDLL(str(LIBRARY_PATH))
    for name, argtypes in SIGNATURES.items():
        function = getattr(library, name)
        function.argtypes = argtypes
        function.restype = _RESTYPES.get(name, ctypes.c_int)
    return library


lib = _load()


def check(status: int) -> None:
    if status != AR_OK:
        message = lib.ar_last_error().decode("utf-8", "replace")
        raise AttnRankError(message or f"attnrank_b200 call failed with status {status}")


def version() -> str:
    return lib.ar_version().decode()

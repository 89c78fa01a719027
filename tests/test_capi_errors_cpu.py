"""The C ABI's error contract, on a host without a GPU: every entry point rejects a bad argument
with AR_ERR_INVALID and a message before any device work (the reference throws attnrank::Error
for these, model.cu:638-647, and pybind turns it into AttnRankError), and the query functions
answer a null handle with their documented sentinel. No call here reaches a kernel."""
from __future__ import annotations

import ctypes

import pytest

from attnrank import _native

lib = _native.lib
F16 = _native.DTYPE_F16


def _handle():
    return ctypes.c_void_p()


CASES = {
    "embedding hidden size": (lambda: lib.ar_embedding_rms_norm(None, 4, None, 100, 12, None, 1e-6, None, None, None,
                                                                F16, None), "multiple of 8"),
    "rms norm hidden size": (lambda: lib.ar_rms_norm_residual(None, None, None, 4, 10, 1e-6, None, F16, None),
                             "multiple of 8"),
    "rotary head dim": (lambda: lib.ar_rotary_embedding(None, None, None, 4, 4, 2, 12, None, None, 64, None, F16, None),
                        "multiple of 16"),
    "rope table positions": (lambda: lib.ar_rope_table(None, None, -1, 128, 1e6, None), "invalid sizes"),
    "silu width": (lambda: lib.ar_silu_multiply(None, None, 16, None, 16, 4, 12, F16, None), "multiples of 8"),
    "attention head dim": (lambda: lib.ar_causal_attention(None, None, None, None, None, 1, 4, 2, 64, 0, F16, None),
                           "head_dim must be 128"),
    "attention prompts": (lambda: lib.ar_causal_attention(None, None, None, None, None, 0, 4, 2, 128, 0, F16, None),
                          "head_dim must be 128"),
    "decode gemv k": (lambda: lib.ar_decode_gemv(None, None, 4, 12, None, 0, F16, None), "multiple of 8"),
    "decode gate|up k": (lambda: lib.ar_decode_gate_up(None, None, 4, 12, None, F16, None), "multiple of 8"),
    "decode attention position": (lambda: lib.ar_decode_attention(None, None, None, 16, 16, 4, 2, 128, 0, None, F16,
                                                                  None), "position outside the cache"),
    "decode attention group": (lambda: lib.ar_decode_attention(None, None, None, 16, 3, 34, 2, 128, 0, None, F16,
                                                               None), "multiple"),
    "engine create": (lambda: lib.ar_engine_create(None, None, ctypes.byref(_handle())), "null argument"),
    "engine load": (lambda: lib.ar_engine_load_tensor(None, b"x", 0, None, 0, None), "null argument"),
    "engine synthetic": (lambda: lib.ar_engine_init_synthetic(None, 0, 0.02), "null engine"),
    "engine probe": (lambda: lib.ar_engine_measure_attention_by_layer(None, None, 1, 5, 0, -1, 0, None, None, None),
                     "null argument"),
    "engine measure": (lambda: lib.ar_engine_measure_attention(None, None, 5, 0, 1, 0, None), "null argument"),
    "engine scan": (lambda: lib.ar_engine_scan(None, None, 1, 5, 0, -1, 0, None, None), "null argument"),
    "engine prepare": (lambda: lib.ar_engine_prepare_scan(None, None, 1, 5, 0, -1, 0, ctypes.byref(_handle())),
                       "null argument"),
    "engine run prepared": (lambda: lib.ar_engine_run_prepared_scan(None, None, None, 1), "null argument"),
    "engine synchronize": (lambda: lib.ar_engine_synchronize(None), "null engine"),
    "engine timing": (lambda: lib.ar_engine_set_kernel_timing(None, 1), "null engine"),
    "engine generate": (lambda: lib.ar_engine_generate(None, None, 1, 4, 2, None, None, None), "null argument"),
    "generation begin": (lambda: lib.ar_engine_generation_begin(None, None, 1, None), "null engine"),
    "generation step": (lambda: lib.ar_engine_generation_step(None, 1, None), "null engine"),
    "sampler create": (lambda: lib.ar_sampler_create(None, ctypes.byref(_handle())), "null argument"),
    "sampler select": (lambda: lib.ar_sampler_select(None, None, 4, None), "null argument"),
    "profile slots": (lambda: lib.ar_profile_from_accumulated(None, -1, 1, None, None), "invalid arguments"),
    "position order count": (lambda: lib.ar_resolve_position_order(None, 0, -1, (ctypes.c_int * 1)()), ""),
    "wait selftest ctas": (lambda: lib.ar_bounded_wait_selftest(0, 16, None), "ctas must be 1..1024"),
    "wait selftest limit": (lambda: lib.ar_bounded_wait_selftest(4, (1 << 22) + 1, None), "spin_limit 1..4194304"),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_bad_arguments_are_rejected_with_a_message(name):
    call, message = CASES[name]
    assert call() == _native.AR_ERR_INVALID
    text = lib.ar_last_error().decode()
    assert text and message in text, text


def test_query_functions_answer_a_null_handle():
    assert lib.ar_engine_device(None) == -1
    assert lib.ar_engine_decode_mode(None) == -1
    assert lib.ar_engine_generation_position(None) == -1
    assert lib.ar_engine_stream(None) is None
    assert lib.ar_prepared_scan_bytes(None) == 0
    lib.ar_engine_destroy(None)          # no-ops
    lib.ar_prepared_scan_destroy(None)
    lib.ar_sampler_destroy(None)


def test_last_error_is_cleared_by_a_successful_call():
    assert lib.ar_engine_synchronize(None) == _native.AR_ERR_INVALID
    assert lib.ar_last_error()
    order = (ctypes.c_int * 3)()
    assert lib.ar_resolve_position_order((ctypes.c_int * 1)(1), 1, 3, order) == _native.AR_OK
    assert lib.ar_last_error() == b"" and list(order) == [1, 0, 2]


# --- the two kernel-level mass entry points: every argument check runs on the host before any
# CUDA call, so both reject the same bad inputs here, without a GPU
_MASS_FUNCTIONS = ("ar_document_attention_mass", "ar_document_attention_mass_noalloc")
_FAKE_DEVICE_POINTER = ctypes.c_void_p(256)  # never dereferenced: each call below fails its checks first


def _mass_call(name, offsets, query_spans, spans, span_count, qkv_rows=None, heads=28, kv_heads=4, head_dim=128,
               qkv=_FAKE_DEVICE_POINTER):
    import numpy as np
    offsets = np.ascontiguousarray(offsets, dtype=np.int32)
    query_spans = np.ascontiguousarray(query_spans, dtype=np.int32)
    spans = np.ascontiguousarray(spans, dtype=np.int32)
    prompt_count = len(offsets) - 1
    out = np.zeros(max(prompt_count, 1) * max(span_count, 1), dtype=np.float64)
    rows = int(offsets[-1]) if qkv_rows is None else qkv_rows
    return getattr(lib, name)(qkv, rows, _FAKE_DEVICE_POINTER, offsets.ctypes.data, prompt_count,
                              query_spans.ctypes.data, spans.ctypes.data, span_count, heads, kv_heads, head_dim, 0,
                              512, 0, out.ctypes.data, F16, None)


_ONE_PROMPT = dict(offsets=[0, 300], query_spans=[260, 300], spans=[0, 50, 50, 100, 100, 150, 150, 200, 200, 260],
                   span_count=5)

MASS_CASES = {
    "no spans": (dict(_ONE_PROMPT, span_count=0), "1..32 spans"),
    "33 spans": (dict(_ONE_PROMPT, spans=[0, 1] * 33, span_count=33), "1..32 spans"),
    "head dim 64": (dict(_ONE_PROMPT, head_dim=64), "head_dim must be 128"),
    "heads not a multiple": (dict(_ONE_PROMPT, heads=6, kv_heads=4), "multiple of kv_heads"),
    "null qkv": (dict(_ONE_PROMPT, qkv=None), "null argument"),
    "offsets past qkv rows": (dict(_ONE_PROMPT, qkv_rows=299), "exceed qkv rows"),
    "negative first offset": (dict(_ONE_PROMPT, offsets=[-100, 50], qkv_rows=50), "start at 0"),
    "decreasing offsets": (dict(offsets=[0, 300, 200], query_spans=[260, 300, 0, 10], spans=[0, 10] * 10,
                                span_count=5, qkv_rows=300), "non-decreasing"),
    "reversed query span": (dict(_ONE_PROMPT, query_spans=[300, 260]), "invalid query span"),
    "negative query span": (dict(_ONE_PROMPT, query_spans=[-1, 300]), "invalid query span"),
    "negative document span": (dict(_ONE_PROMPT, spans=[-5, 50] + _ONE_PROMPT["spans"][2:]), "invalid document span"),
    "reversed document span": (dict(_ONE_PROMPT, spans=[50, 0] + _ONE_PROMPT["spans"][2:]), "invalid document span"),
}


@pytest.mark.parametrize("function", _MASS_FUNCTIONS)
@pytest.mark.parametrize("case", sorted(MASS_CASES))
def test_mass_entry_points_reject_bad_arguments_alike(function, case):
    kwargs, message = MASS_CASES[case]
    assert _mass_call(function, **kwargs) == _native.AR_ERR_INVALID
    text = lib.ar_last_error().decode()
    assert message in text and function[3:] in text, text


def test_noalloc_rejects_a_batch_beyond_its_fixed_scratch_before_any_device_work():
    """One 32K-token prompt probed on every row with 32 spans partitioning it needs 4 KV heads x
    1792 row tiles x 64 key runs = 458752 work items, ~59 MB of per-CTA partial sums: more than
    the fixed 8 MiB array, so the call is refused on the host."""
    T, S = 32768, 32
    edges = [T * i // S for i in range(S + 1)]
    spans = [v for i in range(S) for v in (edges[i], edges[i + 1])]
    status = _mass_call("ar_document_attention_mass_noalloc", [0, T], [0, T], spans, S)
    assert status == _native.AR_ERR_INVALID
    text = lib.ar_last_error().decode()
    assert "fixed array holds 8388608" in text and "ar_document_attention_mass" in text, text

"""The allocation-free mass entry point (ar_document_attention_mass_noalloc) through the C ABI.

It serves callers that cannot let the library allocate device memory while they run (a fixed
memory budget, a latency-critical loop, a host framework that owns all device allocations): its
scratch is a fixed device array reserved when the library loads. This file is collected last so
that a run stopping at the first failure has already run every other test; it must also pass on
its own in a fresh process (its first call on the device looks up the array's address).

Checks: two calls in a row give bit-for-bit the result of the allocating entry point
(ar_document_attention_mass) on the same inputs -- the same kernels run on the same data, only the
scratch differs -- and the span masses agree with the fp32 CPU oracle's softmax rows within the
mass tolerance of the other GPU tests (rel 1e-3); a batch whose scratch exceeds the fixed array
is rejected with a clear error.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MASS_REL = 1e-3


def _inputs(cuda, lengths, heads=28, kv_heads=4, queries=40, span_count=5, seed=3):
    import torch
    from attnrank import _native
    D = 128
    width = (heads + 2 * kv_heads) * D
    total = int(sum(lengths))
    gen = torch.Generator(device=cuda).manual_seed(seed)
    qkv = torch.randn(total, width, device=cuda, generator=gen).to(torch.float16)
    out = torch.empty(total, heads * D, device=cuda, dtype=torch.float16)
    lse = torch.empty(total, heads, device=cuda, dtype=torch.float32)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    offsets_d = torch.from_numpy(offsets).to(cuda)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _native.check(_native.lib.ar_causal_attention(ctypes.c_void_p(qkv.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                                  ctypes.c_void_p(lse.data_ptr()), offsets.ctypes.data,
                                                  ctypes.c_void_p(offsets_d.data_ptr()), len(lengths), heads, kv_heads,
                                                  D, 0, _native.DTYPE_F16, stream))
    rng = np.random.default_rng(seed)
    query_spans, spans = [], []
    for T in lengths:
        qb = max(0, T - queries)
        query_spans += [qb, T]
        if qb > 0:  # random (possibly overlapping) spans before the query
            cuts = np.sort(rng.integers(0, qb, size=2 * span_count))
        else:       # query covers the prompt: spans partition it
            edges = np.linspace(0, T, span_count + 1).astype(np.int64)
            cuts = np.stack([edges[:-1], edges[1:]], axis=1).reshape(-1)
        spans += [int(v) for v in cuts]
    return dict(qkv=qkv, lse=lse, offsets=offsets, query_spans=np.ascontiguousarray(np.array(query_spans, np.int32)),
                spans=np.ascontiguousarray(np.array(spans, np.int32)), heads=heads, kv_heads=kv_heads,
                span_count=span_count, stream=stream, keep=(out, offsets_d))


def _call(function, data, normalize=0):
    from attnrank import _native
    prompt_count = len(data["offsets"]) - 1
    out = np.zeros((prompt_count, data["span_count"]), dtype=np.float64)
    status = function(ctypes.c_void_p(data["qkv"].data_ptr()), int(data["offsets"][-1]),
                      ctypes.c_void_p(data["lse"].data_ptr()), data["offsets"].ctypes.data, prompt_count,
                      data["query_spans"].ctypes.data, data["spans"].ctypes.data, data["span_count"], data["heads"],
                      data["kv_heads"], 128, 0, 512, normalize, out.ctypes.data, _native.DTYPE_F16, data["stream"])
    return status, out


@pytest.mark.parametrize("normalize", [0, 1])
def test_noalloc_matches_allocating_entry_point_twice(cuda, normalize):
    from attnrank import _native
    data = _inputs(cuda, [940, 700, 1200, 64])
    status, want = _call(_native.lib.ar_document_attention_mass, data, normalize)
    _native.check(status)
    for _ in range(2):  # the fixed array keeps the previous call's contents; results must not depend on them
        status, got = _call(_native.lib.ar_document_attention_mass_noalloc, data, normalize)
        _native.check(status)
        np.testing.assert_array_equal(got, want)


def test_noalloc_matches_the_oracle_span_mass(cuda):
    """Span sums of the oracle's exact softmax rows (fp32 CPU, the same fp16 qkv values), divided
    by query rows x heads as the reference does before its unit-sum step (model.cu:602-615)."""
    import torch
    from attnrank import _native
    from oracle import forward as F
    lengths = [940, 300, 64]
    data = _inputs(cuda, lengths, seed=8)
    status, got = _call(_native.lib.ar_document_attention_mass_noalloc, data)
    _native.check(status)
    qkv = data["qkv"].to(torch.float32).cpu().numpy()
    _, _, probs = F.op_attention(qkv, data["offsets"], data["heads"], data["kv_heads"], 128, 0)
    for p, T in enumerate(lengths):
        query = tuple(int(v) for v in data["query_spans"][2 * p:2 * p + 2])
        spans = data["spans"].reshape(len(lengths), data["span_count"], 2)[p]
        prompt = F.Prompt(tokens=np.zeros(T, np.int32), query_span=query, spans=[(int(a), int(b)) for a, b in spans])
        want = F.document_mass(probs[p], prompt, 512, False) / ((query[1] - query[0]) * data["heads"])
        np.testing.assert_allclose(got[p], want, rtol=MASS_REL, atol=1e-9)


def test_noalloc_rejects_batches_beyond_its_fixed_scratch(cuda):
    """A valid batch that needs more scratch than the fixed array (one 32K-token prompt probed on
    every row, 32 spans partitioning it: 4 KV heads x 1792 row tiles x 64 key runs = 458752 CTAs,
    ~59 MB of partial sums) is refused before any device work."""
    from attnrank import _native
    data = _inputs(cuda, [32768], queries=32768, span_count=32)
    status, _ = _call(_native.lib.ar_document_attention_mass_noalloc, data)
    assert status == _native.AR_ERR_INVALID
    assert "fixed array" in _native.lib.ar_last_error().decode()

"""Kernel parity through the C ABI on a B200: each CUDA kernel against the fp32 CPU oracle.

Tolerances (from the build's parity bar), for both 16-bit activation types:
  * integer / bit work (synthetic weights, residual gather): bit-exact;
  * 16-bit activations: within 2 ulp of the oracle, i.e. |x - ref| <= 2 ulp * |ref| + tiny
    (2^-7 relative for bf16, 2^-10 for fp16; the bf16 bar is the rel 1e-2 of the spec); attention
    outputs the same, with the fp32-accumulation floor of a P.V product over a 16-bit P
    (assert_attention_close);
  * fp32 attention mass: rel 1e-3;  log-sum-exp: abs 2e-3 (log2 units).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DTYPES = ["fp16", "bf16"]
TWO_ULP = {"bf16": 2.0 ** -7, "fp16": 2.0 ** -10}   # two ulp, relative
MASS_REL = 1e-3


def _lib():
    from attnrank import _native
    return _native


def _code(dtype: str) -> int:
    from attnrank import _native
    return _native.DTYPE_F16 if dtype == "fp16" else _native.DTYPE_BF16


def _ptr(tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(tensor.data_ptr())


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _torch_dtype(dtype: str):
    import torch
    return torch.float16 if dtype == "fp16" else torch.bfloat16


def _half_tensor(values: np.ndarray, device, dtype: str):
    """values rounded to the 16-bit type with round-to-nearest-even."""
    import torch
    from oracle import weights as W
    if dtype == "fp16":
        return torch.from_numpy(values.astype(np.float32).astype(np.float16)).to(device)
    bits = W.f32_to_bf16_bits(values.astype(np.float32))
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(device)


def _to_np(tensor) -> np.ndarray:
    import torch
    return tensor.detach().to(torch.float32).cpu().numpy()


def assert_half_close(actual: np.ndarray, expected: np.ndarray, dtype: str, floor: float = 1e-6):
    error = np.abs(actual - expected)
    bound = TWO_ULP[dtype] * np.abs(expected) + floor
    worst = np.argmax(error - bound)
    assert np.all(error <= bound), (
        f"{dtype} mismatch at {np.unravel_index(worst, error.shape)}: got {actual.flat[worst]}, "
        f"want {expected.flat[worst]} (bound {bound.flat[worst]})")


@pytest.mark.parametrize("dtype", DTYPES)
def test_synthetic_fill_matches_checker_bit_exact(cuda, dtype):
    """The seeded generator gives the checker's bf16 bits; the fp16 engine stores each bf16 value
    converted to fp16 with round-to-nearest-even."""
    import torch
    from oracle import weights as W
    native = _lib()
    count = 1 << 20
    for layer, kind, std in [(-1, W.EMBEDDING, 0.02), (3, W.QUERY, 0.02), (27, W.DOWN, 0.05)]:
        out = torch.empty(count, dtype=torch.int16, device=cuda)
        native.check(native.lib.ar_synthetic_fill(_ptr(out), count, 0, layer, kind, std, _code(dtype), _stream()))
        torch.cuda.synchronize()
        expected = W.bf16_bits(count, 0, layer, kind, std)
        if dtype == "fp16":
            expected = (expected.astype(np.uint32) << 16).view(np.float32).astype(np.float16).view(np.uint16)
        got = out.cpu().numpy().view(np.uint16)
        assert np.array_equal(got, expected)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("hidden", [2048, 3584, 8192])
def test_embedding_rms_norm(cuda, hidden, dtype):
    import torch
    from oracle import forward as F
    native = _lib()
    rng = np.random.default_rng(hidden)
    vocab = 1000
    table = rng.standard_normal((vocab, hidden)).astype(np.float32) * 0.02
    table_bf = _half_tensor(table, cuda, dtype)
    table_exact = _to_np(table_bf)
    ids = np.concatenate([[0, vocab - 1], rng.integers(0, vocab, 61)]).astype(np.int32)
    gamma = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    ids_d = torch.from_numpy(ids).to(cuda)
    gamma_d = torch.from_numpy(gamma).to(cuda)
    residual = torch.empty((ids.size, hidden), dtype=torch.float32, device=cuda)
    normed = torch.empty((ids.size, hidden), dtype=_torch_dtype(dtype), device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    native.check(native.lib.ar_embedding_rms_norm(_ptr(ids_d), ids.size, _ptr(table_bf), vocab, hidden, _ptr(gamma_d),
                                                  1e-6, _ptr(residual), _ptr(normed), _ptr(status), _code(dtype),
                                                  _stream()))
    torch.cuda.synchronize()
    want_residual, want_normed = F.op_embedding_rms_norm(table_exact, ids, gamma, 1e-6)
    assert int(status.item()) == 0
    assert np.array_equal(_to_np(residual), want_residual)
    assert_half_close(_to_np(normed), want_normed, dtype)


def test_embedding_reports_out_of_range_token(cuda):
    import torch
    native = _lib()
    hidden, vocab = 256, 16
    table = torch.zeros((vocab, hidden), dtype=torch.float16, device=cuda)
    ids = torch.tensor([3, vocab, -1], dtype=torch.int32, device=cuda)
    gamma = torch.ones(hidden, dtype=torch.float32, device=cuda)
    residual = torch.full((3, hidden), 7.0, dtype=torch.float32, device=cuda)
    normed = torch.empty((3, hidden), dtype=torch.float16, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    native.check(native.lib.ar_embedding_rms_norm(_ptr(ids), 3, _ptr(table), vocab, hidden, _ptr(gamma), 1e-6,
                                                  _ptr(residual), _ptr(normed), _ptr(status), _code("fp16"),
                                                  _stream()))
    torch.cuda.synchronize()
    assert int(status.item()) == 1
    assert float(residual[1:].abs().max()) == 0.0


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens,hidden", [(1, 3584), (64, 4096), (1000, 3584), (33, 8192)])
def test_rms_norm_residual(cuda, tokens, hidden, dtype):
    import torch
    from oracle import forward as F
    native = _lib()
    rng = np.random.default_rng(tokens * hidden)
    residual = rng.standard_normal((tokens, hidden)).astype(np.float32)
    delta = rng.standard_normal((tokens, hidden)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    delta_d = _half_tensor(delta, cuda, dtype)
    residual_d = torch.from_numpy(residual).to(cuda)
    gamma_d = torch.from_numpy(gamma).to(cuda)
    normed = torch.empty((tokens, hidden), dtype=_torch_dtype(dtype), device=cuda)
    native.check(native.lib.ar_rms_norm_residual(_ptr(residual_d), _ptr(delta_d), _ptr(gamma_d), tokens, hidden, 1e-6,
                                                 _ptr(normed), _code(dtype), _stream()))
    torch.cuda.synchronize()
    want_residual, want_normed = F.op_rms_norm_residual(residual, _to_np(delta_d), gamma, 1e-6)
    np.testing.assert_allclose(_to_np(residual_d), want_residual, rtol=1e-6, atol=1e-6)
    assert_half_close(_to_np(normed), want_normed, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens,hidden", [(64, 3584), (33, 8192), (1, 4096)])
def test_rms_norm_without_delta(cuda, tokens, hidden, dtype):
    """delta = NULL: the engine's form after a projection GEMM has accumulated into the residual.
    The residual is read, not written (bit-identical afterwards), and the normed row is the
    oracle's rms_norm of it (kernels.cu:60-83)."""
    import torch
    from oracle import forward as F
    native = _lib()
    rng = np.random.default_rng(tokens + hidden)
    residual = rng.standard_normal((tokens, hidden)).astype(np.float32)
    gamma = (1.0 + 0.1 * rng.standard_normal(hidden)).astype(np.float32)
    residual_d = torch.from_numpy(residual).to(cuda)
    gamma_d = torch.from_numpy(gamma).to(cuda)
    normed = torch.empty((tokens, hidden), dtype=_torch_dtype(dtype), device=cuda)
    native.check(native.lib.ar_rms_norm_residual(_ptr(residual_d), None, _ptr(gamma_d), tokens, hidden, 1e-6,
                                                 _ptr(normed), _code(dtype), _stream()))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(_to_np(residual_d), residual)
    _, want_normed = F.op_rms_norm_residual(residual, np.zeros_like(residual), gamma, 1e-6)
    assert_half_close(_to_np(normed), want_normed, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("heads,kv_heads,bias", [(28, 4, True), (32, 8, False), (3, 1, True)])
def test_rotary_bias(cuda, heads, kv_heads, bias, dtype):
    import torch
    from oracle import forward as F
    native = _lib()
    D, tokens, theta = 128, 300, 1e6 if bias else 5e5
    width = (heads + 2 * kv_heads) * D
    rng = np.random.default_rng(heads)
    qkv = rng.standard_normal((tokens, width)).astype(np.float32)
    qkv_d = _half_tensor(qkv, cuda, dtype)
    qkv_exact = _to_np(qkv_d)
    bias_np = (0.02 * rng.standard_normal(width)).astype(np.float32) if bias else None
    positions = np.concatenate([np.arange(100), np.arange(200) + 4000]).astype(np.int32)
    table_positions = 8192
    cos = torch.empty((table_positions, D // 2), dtype=torch.float32, device=cuda)
    sin = torch.empty_like(cos)
    native.check(native.lib.ar_rope_table(_ptr(cos), _ptr(sin), table_positions, D, theta, _stream()))
    pos_d = torch.from_numpy(positions).to(cuda)
    bias_d = torch.from_numpy(bias_np).to(cuda) if bias else None
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    native.check(native.lib.ar_rotary_embedding(_ptr(qkv_d), _ptr(bias_d) if bias else None, _ptr(pos_d), tokens, heads,
                                                kv_heads, D, _ptr(cos), _ptr(sin), table_positions, _ptr(status),
                                                _code(dtype), _stream()))
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # the rotation arithmetic, on the kernel's own cos/sin table
    tables = (cos.cpu().numpy(), sin.cpu().numpy())
    want = F.op_rotary_bias(qkv_exact, bias_np, positions, heads, kv_heads, D, theta, tables=tables)
    got = _to_np(qkv_d)
    assert_half_close(got, want, dtype, floor=1e-6 * np.abs(want).max())
    if not bias:  # value heads untouched without a bias
        assert np.array_equal(got[:, (heads + kv_heads) * D:], qkv_exact[:, (heads + kv_heads) * D:])


@pytest.mark.parametrize("theta", [1e4, 5e5, 1e6])
def test_rope_table(cuda, theta):
    """cos/sin(pos * theta^(-2i/D)) against fp64. The fp32 angle carries pos x (a few ulp of the
    fp32 inverse frequency) of rounding, exactly as the reference's per-element powf/cosf/sinf
    (kernels.cu:95-98), so the bound grows with the position."""
    import torch
    native = _lib()
    D, positions = 128, 32768
    cos = torch.empty((positions, D // 2), dtype=torch.float32, device=cuda)
    sin = torch.empty_like(cos)
    native.check(native.lib.ar_rope_table(_ptr(cos), _ptr(sin), positions, D, theta, _stream()))
    torch.cuda.synchronize()
    index = np.arange(D // 2, dtype=np.float64)
    inverse = theta ** (-2.0 * index / D)
    angle = np.arange(positions, dtype=np.float64)[:, None] * inverse[None, :]
    bound = 1e-6 + np.arange(positions)[:, None] * inverse[None, :] * 2.0 ** -21  # ~4 ulp of inv_freq, times pos
    assert np.all(np.abs(cos.cpu().numpy() - np.cos(angle)) <= bound)
    assert np.all(np.abs(sin.cpu().numpy() - np.sin(angle)) <= bound)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("tokens,width", [(1, 18944), (257, 18944), (64, 14336), (3, 8)])
def test_silu_multiply(cuda, tokens, width, dtype):
    import torch
    from oracle import forward as F
    native = _lib()
    rng = np.random.default_rng(width + tokens)
    gate_up = rng.standard_normal((tokens, 2 * width)).astype(np.float32) * 2
    gu_d = _half_tensor(gate_up, cuda, dtype)
    exact = _to_np(gu_d)
    out = torch.empty((tokens, width), dtype=_torch_dtype(dtype), device=cuda)
    native.check(native.lib.ar_silu_multiply(_ptr(gu_d), ctypes.c_void_p(gu_d.data_ptr() + 2 * width), 2 * width,
                                             _ptr(out), width, tokens, width, _code(dtype), _stream()))
    torch.cuda.synchronize()
    want = F.op_silu_multiply(exact[:, :width], exact[:, width:])
    assert_half_close(_to_np(out), want, dtype, floor=1e-4)


UNIT_ROUNDOFF = {"bf16": 2.0 ** -8, "fp16": 2.0 ** -11}


def assert_attention_close(got: np.ndarray, want: np.ndarray, qkv: np.ndarray, offsets, probs, heads: int,
                           kv_heads: int, dtype: str):
    """Per element: |got - want| <= 2 ulp * |want| + floor. The floor is the fp32-accumulation
    term of a P.V product whose P operand is rounded to the 16-bit type: 4 u sqrt(sum_k p_k^2 v_k^2)
    (u the type's unit roundoff), about seven standard deviations of the rounding noise. It
    matters only where the output is small against the terms it sums."""
    import torch
    D = 128
    group = heads // kv_heads
    floor = np.zeros_like(want)
    v_at = (heads + kv_heads) * D
    for p in range(len(offsets) - 1):
        a, b = int(offsets[p]), int(offsets[p + 1])
        v = torch.from_numpy(qkv[a:b, v_at:v_at + kv_heads * D]).view(b - a, kv_heads, D)
        v = v.repeat_interleave(group, dim=1)
        spread = torch.einsum("hqk,khd->qhd", probs[p].double() ** 2, v.double() ** 2).sqrt()
        floor[a:b] = (4 * UNIT_ROUNDOFF[dtype] * spread).reshape(b - a, heads * D).numpy()
    assert_half_close(got, want, dtype, floor=floor + 1e-6)


def _packed_qkv(lengths, heads, kv_heads, seed, device, dtype="fp16"):
    rng = np.random.default_rng(seed)
    D = 128
    width = (heads + 2 * kv_heads) * D
    total = int(sum(lengths))
    qkv = rng.standard_normal((total, width)).astype(np.float32)
    qkv_d = _half_tensor(qkv, device, dtype)
    offsets = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    return qkv_d, _to_np(qkv_d), offsets


@pytest.mark.parametrize("kernel", ["tcgen05", "mma"])
@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("heads,kv_heads,lengths,window", [
    (28, 4, [1, 200, 777], 0),
    (32, 8, [129, 64, 300], 0),
    (28, 4, [500], 96),
    (28, 4, [940, 1240, 256, 128, 1], 0),
    (4, 4, [385, 17], 200),
])
def test_causal_attention(cuda, heads, kv_heads, lengths, window, dtype, kernel):
    """Both attention kernels (tcgen05/TMEM and mma.sync) against the oracle's exact softmax."""
    import torch
    from oracle import forward as F
    native = _lib()
    qkv_d, qkv, offsets = _packed_qkv(lengths, heads, kv_heads, sum(lengths), cuda, dtype)
    total = int(offsets[-1])
    out = torch.zeros((total, heads * 128), dtype=_torch_dtype(dtype), device=cuda)
    lse = torch.zeros((total, heads), dtype=torch.float32, device=cuda)
    offsets_d = torch.from_numpy(offsets).to(cuda)
    host_offsets = np.ascontiguousarray(offsets)
    entry = native.lib.ar_causal_attention if kernel == "tcgen05" else native.lib.ar_causal_attention_mma
    native.check(entry(_ptr(qkv_d), _ptr(out), _ptr(lse), host_offsets.ctypes.data, _ptr(offsets_d), len(lengths),
                       heads, kv_heads, 128, window, _code(dtype), _stream()))
    torch.cuda.synchronize()
    want_out, want_lse, probs = F.op_attention(qkv, offsets, heads, kv_heads, 128, window)
    np.testing.assert_allclose(_to_np(lse), want_lse, atol=2e-3, rtol=0)
    assert_attention_close(_to_np(out), want_out, qkv, offsets, probs, heads, kv_heads, dtype)


@pytest.mark.parametrize("kernel", ["tcgen05", "mma"])
@pytest.mark.parametrize("dtype", DTYPES)
def test_causal_attention_rescale_on_some_rows(cuda, dtype, kernel):
    """Rows of one 32-row group whose running max jumps at a later key tile while their
    neighbours' does not: even query rows >= 260 align with keys 260..270, which score
    ~12 log2 units above everything before them; odd rows see ordinary scores. The tcgen05
    kernel rescales its TMEM accumulator for some rows of a warp only (a warp-collective step),
    and both kernels must still match the exact softmax."""
    import torch
    from oracle import forward as F
    native = _lib()
    heads, kv_heads, D, T = 4, 1, 128, 700
    width = (heads + 2 * kv_heads) * D
    rng = np.random.default_rng(11)
    qkv = rng.standard_normal((T, width)).astype(np.float32)
    direction = np.full(D, 1.0 / np.sqrt(D), dtype=np.float32)
    k_col = heads * D
    qkv[260:271, k_col:k_col + D] = 12.0 * direction
    for h in range(heads):
        qkv[260::2, h * D:(h + 1) * D] = 12.0 * direction
    qkv_d = _half_tensor(qkv, cuda, dtype)
    exact = _to_np(qkv_d)
    offsets = np.array([0, T], dtype=np.int32)
    out = torch.zeros((T, heads * D), dtype=_torch_dtype(dtype), device=cuda)
    lse = torch.zeros((T, heads), dtype=torch.float32, device=cuda)
    offsets_d = torch.from_numpy(offsets).to(cuda)
    entry = native.lib.ar_causal_attention if kernel == "tcgen05" else native.lib.ar_causal_attention_mma
    native.check(entry(_ptr(qkv_d), _ptr(out), _ptr(lse), offsets.ctypes.data, _ptr(offsets_d), 1, heads, kv_heads,
                       D, 0, _code(dtype), _stream()))
    torch.cuda.synchronize()
    want_out, want_lse, probs = F.op_attention(exact, offsets, heads, kv_heads, D, 0)
    np.testing.assert_allclose(_to_np(lse), want_lse, atol=2e-3, rtol=0)
    assert_attention_close(_to_np(out), want_out, exact, offsets, probs, heads, kv_heads, dtype)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("heads,kv_heads,lengths,queries,normalize", [
    (28, 4, [940, 700], 40, False),
    (32, 8, [1200], 64, True),
    (28, 4, [130, 300, 9], 5, False),
])
def test_document_mass(cuda, heads, kv_heads, lengths, queries, normalize, dtype):
    """The tcgen05 mass kernel against span sums of the oracle's softmax rows."""
    import torch
    from oracle import forward as F
    native = _lib()
    qkv_d, qkv, offsets = _packed_qkv(lengths, heads, kv_heads, 7 + sum(lengths), cuda, dtype)
    total = int(offsets[-1])
    out = torch.zeros((total, heads * 128), dtype=_torch_dtype(dtype), device=cuda)
    lse = torch.zeros((total, heads), dtype=torch.float32, device=cuda)
    offsets_d = torch.from_numpy(offsets).to(cuda)
    native.check(native.lib.ar_causal_attention(_ptr(qkv_d), _ptr(out), _ptr(lse), offsets.ctypes.data,
                                                _ptr(offsets_d), len(lengths), heads, kv_heads, 128, 0, _code(dtype),
                                                _stream()))
    rng = np.random.default_rng(len(lengths))
    span_count = 5
    query_spans, spans, prompts = [], [], []
    for T in lengths:
        q = min(queries, T)
        qb = T - q
        cuts = np.sort(rng.integers(0, max(qb, 1), size=span_count * 2)).reshape(span_count, 2)
        cuts[0, 0] = 0  # a span at the very start
        doc = [(int(a), int(b)) for a, b in cuts]
        query_spans.append((qb, T))
        spans.extend(doc)
        prompts.append(F.Prompt(tokens=np.zeros(T, np.int32), query_span=(qb, T), spans=doc))
    qs = np.ascontiguousarray(np.array(query_spans, dtype=np.int32).reshape(-1))
    sp = np.ascontiguousarray(np.array(spans, dtype=np.int32).reshape(-1))
    mass = np.zeros((len(lengths), span_count), dtype=np.float64)
    native.check(native.lib.ar_document_attention_mass(_ptr(qkv_d), total, _ptr(lse), offsets.ctypes.data, len(lengths),
                                                       qs.ctypes.data, sp.ctypes.data, span_count, heads, kv_heads, 128,
                                                       0, 512, int(normalize), mass.ctypes.data, _code(dtype),
                                                       _stream()))
    _, _, probs = F.op_attention(qkv, offsets, heads, kv_heads, 128, 0)
    for p, prompt in enumerate(prompts):
        raw = F.document_mass(probs[p], prompt, 512, normalize)
        T = len(prompt.tokens)
        observations = (prompt.query_span[1] - prompt.query_span[0]) * heads
        want = raw / observations
        np.testing.assert_allclose(mass[p], want, rtol=MASS_REL, atol=1e-9)

"""A device wait that runs out ends in an error, not a hang, and the device stays usable.

ar_bounded_wait_selftest makes CTAs wait on the persistent decode step's grid barrier for a counter
value that nothing writes (no fault is involved: the flag is simply never set). The wait gives up
after its poll limit, the kernel records the wait-timeout status and returns, and the call reports
AR_ERR_DEVICE. An engine on the same device then probes and generates as usual.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_a_wait_that_runs_out_reports_an_error_and_the_device_stays_usable(cuda):
    import torch

    import attnrank as ar
    from attnrank import _native, synthetic
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for ctas, limit in [(1, 1 << 10), (8, 1 << 14), (148, 1 << 12)]:
        start = time.monotonic()
        status = _native.lib.ar_bounded_wait_selftest(ctas, limit, stream)
        elapsed = time.monotonic() - start
        assert status == _native.AR_ERR_DEVICE, status
        message = _native.lib.ar_last_error().decode()
        assert "wait timeout" in message, message
        assert elapsed < 5.0, elapsed  # the limit is at most 16K polls of about 64 ns each
    assert _native.lib.ar_bounded_wait_selftest(0, 16, stream) == _native.AR_ERR_INVALID
    assert _native.lib.ar_bounded_wait_selftest(4, (1 << 22) + 1, stream) == _native.AR_ERR_INVALID

    # the context is intact: a small engine probes and generates on the same device
    config = ar.LlamaConfig(hidden_size=512, intermediate_size=1024, num_hidden_layers=2, num_attention_heads=4,
                            num_key_value_heads=2, vocab_size=2000, max_position_embeddings=4096, rms_norm_eps=1e-6,
                            rope_theta=1e6, attention_bias=True, tie_word_embeddings=True)
    engine = ar.Engine.synthetic(config, seed=0, options=ar.RuntimeOptions(device_index=0, max_sequence_length=512))
    shape = synthetic.PromptShape(documents=5, document_min=20, document_max=60, question=8)
    prompts = synthetic.prompts(2, config.vocab_size, shape, seed=5)
    engine.config.eos_token_id = -1  # a fixed number of new tokens
    rows, _ = engine.probe_rows(prompts)
    assert np.all(np.isfinite(rows[0])) and np.allclose(rows[0].sum(axis=1), 1.0)
    assert len(engine.generate(prompts[0].tokens, max_new_tokens=3).generated_tokens) == 3
    engine.close()

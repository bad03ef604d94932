"""GPU: the bounded-wait error path, exercised without any fault.

``tk_attn_selftest_wait_timeout`` launches a one-CTA kernel waiting on an
mbarrier that nothing arrives at; the wait gives up after the limit and the
kernel records TK_ERR_DEVICE_TIMEOUT in the device status word.  The context
must stay usable: a normal attention call afterwards succeeds and reports OK.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from tklab import _native
from tklab.harness.tolerances import assert_relative_frobenius
from tklab.kernels.flash_attention import attention_causal, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]


def test_wait_timeout_is_reported_and_context_survives() -> None:
    lib = _native.load()
    stream = torch.cuda.current_stream().cuda_stream
    assert _native.device_status(stream) == 0
    _native.check(lib.tk_attn_selftest_wait_timeout(20_000_000, stream), "selftest")
    status = _native.device_status(stream)
    assert status & 0xFF == _native.TK_ERR_DEVICE_TIMEOUT
    assert status >> 8 == 15  # the self-test's wait site
    with pytest.raises(RuntimeError, match="device wait timed out"):
        _native.check(status, "selftest")
    assert _native.device_status(stream) == 0  # read clears

    q, k, v = (torch.randn(1, 2, 256, 64, device="cuda", dtype=torch.float16) for _ in range(3))
    out = attention_causal(q, k, v)
    check_device_status()
    assert_relative_frobenius(out, F.scaled_dot_product_attention(q, k, v, is_causal=True), max_relative_error=2e-2)

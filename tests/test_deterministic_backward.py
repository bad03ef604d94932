"""GPU: the deterministic backward (``tk_attn_bwd_deterministic``).

dQ comes from a query-stationary kernel that sums the key tiles in one fixed
order without atomics; dK and dV come from the fused kernel with its dQ path
compiled out.  Checked against the fp32 algebra of the oracle, for bitwise
reproducibility, and against the default (atomic-reduction) path.
"""

from __future__ import annotations

import pytest
import torch

from oracle.attention_oracle import manual_backward
from tklab.harness.tolerances import assert_relative_frobenius, relative_frobenius_error
from tklab.kernels.flash_attention import _launch_backward, _launch_forward, attention_causal, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]


def _forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], dtype=torch.float32, device=q.device)
    _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
    return o, lse


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [32, 64, 96, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sequence_length", [1, 129, 384])
def test_deterministic_backward_matches_manual_algebra(
    dtype: torch.dtype, head_dim: int, causal: bool, sequence_length: int
) -> None:
    torch.manual_seed(17 * sequence_length + head_dim + int(causal))
    shape = (1, 3, sequence_length, head_dim)
    q, k, v, do = (torch.randn(shape, device="cuda", dtype=dtype) for _ in range(4))
    o, lse = _forward(q, k, v, causal)
    dq, dk, dv = _launch_backward(q, k, v, o, lse, do, causal=causal, deterministic=True)
    expected = manual_backward(q, k, v, do, causal=causal)
    for name, grad, reference_grad in zip(("dq", "dk", "dv"), (dq, dk, dv), expected, strict=True):
        grad = grad.float().cpu()
        assert torch.isfinite(grad).all(), name
        assert (grad - reference_grad).abs().max().item() <= 5e-2, name
        if sequence_length == 1 and name in ("dq", "dk"):
            # One key: dS = dP - delta == 0 exactly; dQ and dK are rounding noise on both sides.
            assert grad.abs().max().item() <= 1e-5
            continue
        assert_relative_frobenius(grad, reference_grad, max_relative_error=3e-2)
    check_device_status()


@pytest.mark.parametrize("causal", [False, True])
def test_deterministic_backward_is_bitwise_reproducible(causal: bool) -> None:
    torch.manual_seed(3 + int(causal))
    shape = (2, 4, 1000, 128)
    q, k, v, do = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o, lse = _forward(q, k, v, causal)
    first = _launch_backward(q, k, v, o, lse, do, causal=causal, deterministic=True)
    for _ in range(3):
        again = _launch_backward(q, k, v, o, lse, do, causal=causal, deterministic=True)
        for a, b in zip(first, again, strict=True):
            assert torch.equal(a, b)
    check_device_status()


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_deterministic_dk_dv_equal_the_fused_kernels(causal: bool, head_dim: int) -> None:
    """dK and dV come from the same products in the same order as the default path."""
    torch.manual_seed(29 + head_dim + int(causal))
    shape = (2, 3, 777, head_dim)
    q, k, v, do = (torch.randn(shape, device="cuda", dtype=torch.float16) for _ in range(4))
    o, lse = _forward(q, k, v, causal)
    dq_d, dk_d, dv_d = _launch_backward(q, k, v, o, lse, do, causal=causal, deterministic=True)
    dq_a, dk_a, dv_a = _launch_backward(q, k, v, o, lse, do, causal=causal, deterministic=False)
    assert torch.equal(dk_d, dk_a)
    assert torch.equal(dv_d, dv_a)
    # dQ differs only by the order of the fp32 additions before the final rounding.
    assert relative_frobenius_error(dq_d.float(), dq_a.float()) < 2e-3
    check_device_status()


def test_deterministic_mode_follows_torch_flag() -> None:
    torch.manual_seed(0)
    shape = (1, 2, 300, 64)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.float16, requires_grad=True) for _ in range(3))
    do = torch.randn(shape, device="cuda", dtype=torch.float16)
    previous = torch.are_deterministic_algorithms_enabled()
    try:
        torch.use_deterministic_algorithms(True)
        grads = [torch.autograd.grad(attention_causal(q, k, v), (q, k, v), grad_outputs=do) for _ in range(2)]
    finally:
        torch.use_deterministic_algorithms(previous)
    for a, b in zip(*grads, strict=True):
        assert torch.equal(a, b)
    check_device_status()


def test_deterministic_backward_c3_slabs() -> None:
    """C3 shape (bf16, S=4096, D=128, causal) on 16 slabs against the default path."""
    torch.manual_seed(0)
    shape = (1, 16, 4096, 128)
    q, k, v, do = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o, lse = _forward(q, k, v, True)
    det = _launch_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
    ref = _launch_backward(q, k, v, o, lse, do, causal=True, deterministic=False)
    assert torch.equal(det[1], ref[1]) and torch.equal(det[2], ref[2])
    assert torch.isfinite(det[0]).all()
    assert relative_frobenius_error(det[0].float(), ref[0].float()) < 2e-3
    check_device_status()


def test_deterministic_backward_repeated_long_sequences() -> None:
    """Many back-to-back deterministic backwards over long sequences (K/V tile loads
    that keep the dQ kernel's MMA warp waiting while its compute warps run ahead):
    no bounded wait may expire (the device status stays clean) and every call returns
    the same dQ bit for bit.  Guards the hand-over of dS between the compute warps and
    the MMA warp, whose barrier once fell two phases behind in exactly this situation."""
    torch.manual_seed(3)
    shape = (2, 32, 4096, 128)
    q, k, v, do = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(4))
    o, lse = _forward(q, k, v, True)
    first = _launch_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
    for _ in range(24):
        again = _launch_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
        assert torch.equal(again[0], first[0])
    check_device_status()

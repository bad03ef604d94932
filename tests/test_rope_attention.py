"""Fused rotate-half RoPE attention (``tklab.kernels.rope_attention``).

CPU: the validation contract.  GPU: the fused forward and the rotate-back
backward against the reference's own rope -> attention chain (golden
fixtures made by its Triton kernels), against the oracle on a sweep of
shapes, and against this library's plain attention on explicitly rotated
inputs (bit-identical: the rotation is the same arithmetic in shared memory
as in device memory).
"""

from __future__ import annotations

import pytest
import torch
from conftest import golden_cases, load_golden

from oracle import attention_oracle as orc
from tklab.harness.tolerances import assert_relative_frobenius, relative_frobenius_error
from tklab.kernels import rope_attention as ra
from tklab.kernels.flash_attention import _launch_forward, attention_noncausal, check_device_status

gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required")


# ---------------------------------------------------------------- CPU contract
def test_rope_requires_head_dim_64_or_128() -> None:
    q = torch.zeros(1, 1, 8, 32, dtype=torch.float16)
    cos = sin = torch.zeros(8, 16)
    with pytest.raises(ValueError, match="head_dim 64 or 128"):
        ra.attention_rope(q, q, q, cos, sin)


def test_rope_table_shape_is_checked() -> None:
    q = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(ValueError, match=r"shape \(seq_len, head_dim // 2\)"):
        ra.attention_rope(q, q, q, torch.zeros(8, 64), torch.zeros(8, 64))
    with pytest.raises(ValueError, match="2D angle tables"):
        ra.attention_rope(q, q, q, torch.zeros(8, 32, 1), torch.zeros(8, 32, 1))


def test_rope_tables_and_torch_rope_match_the_oracle() -> None:
    cos, sin = ra.rope_tables(33, 64)
    assert cos.shape == (33, 32) and cos.dtype == torch.float32
    assert torch.allclose(cos[0], torch.ones(32)) and torch.allclose(sin[0], torch.zeros(32))
    x = torch.randn(2, 3, 33, 64)
    assert torch.allclose(ra.torch_rope(x, cos, sin), orc.rope_rotate(x, cos, sin))
    back = orc.rope_rotate(orc.rope_rotate(x, cos, sin), cos, sin, transpose=True)
    assert torch.allclose(back, x, atol=1e-5)


# ---------------------------------------------------------------- GPU
@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("name", golden_cases(rope=True))
def test_rope_attention_matches_reference_chain(name: str) -> None:
    """The reference's rope kernels + attention kernels (interpreter) on the same inputs."""
    case = load_golden(name)
    q, k, v, do = (case[key].cuda().requires_grad_(key != "do") for key in ("q", "k", "v", "do"))
    cos, sin = case["cos"].float().cuda(), case["sin"].float().cuda()
    o = ra.attention_rope(q, k, v, cos, sin, causal=case["causal"])
    assert relative_frobenius_error(o.float().cpu(), case["ref_o"].float()) < 2e-3
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), grad_outputs=do)
    for got, key in ((dq, "ref_dq"), (dk, "ref_dk"), (dv, "ref_dv")):
        assert relative_frobenius_error(got.float().cpu(), case[key].float()) < 3e-3, key
    for got, key in ((dq, "man_dq"), (dk, "man_dk"), (dv, "man_dv")):
        assert relative_frobenius_error(got.float().cpu(), case[key]) < 3e-3, key
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("seq", [1, 7, 129, 384, 1000])
def test_rope_attention_forward_matches_oracle(dtype: torch.dtype, head_dim: int, causal: bool, seq: int) -> None:
    torch.manual_seed(seq * 7 + head_dim + int(causal))
    shape = (2, 3, seq, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=dtype) for _ in range(3))
    cos, sin = ra.rope_tables(seq, head_dim, device="cuda")
    o = ra.attention_rope(q, k, v, cos, sin, causal=causal).float().cpu()
    expected = orc.rope_attention_forward(q.cpu(), k.cpu(), v.cpu(), cos.cpu(), sin.cpu(), causal=causal)
    assert torch.isfinite(o).all()
    assert (o - expected).abs().max().item() <= 2e-2
    assert_relative_frobenius(o, expected, max_relative_error=2e-2)
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("seq", [7, 129, 384])
def test_rope_attention_backward_matches_oracle(dtype: torch.dtype, head_dim: int, causal: bool, seq: int) -> None:
    torch.manual_seed(seq * 5 + head_dim + int(causal))
    shape = (1, 3, seq, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=dtype, requires_grad=True) for _ in range(3))
    do = torch.randn(shape, device="cuda", dtype=dtype)
    cos, sin = ra.rope_tables(seq, head_dim, device="cuda")
    o = ra.attention_rope(q, k, v, cos, sin, causal=causal)
    grads = torch.autograd.grad(o, (q, k, v), grad_outputs=do)
    expected = orc.rope_attention_backward(
        q.detach().cpu(), k.detach().cpu(), v.detach().cpu(), do.cpu(), cos.cpu(), sin.cpu(), causal=causal
    )
    for name, got, want in zip(("dq", "dk", "dv"), grads, expected, strict=True):
        got = got.float().cpu()
        assert torch.isfinite(got).all(), name
        assert (got - want).abs().max().item() <= 5e-2, name
        assert_relative_frobenius(got, want, max_relative_error=3e-2)
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("shape", [(1, 3, 1000, 64), (2, 2, 777, 128), (1, 64, 4096, 128)])
@pytest.mark.parametrize("causal", [False, True])
def test_fused_rotation_equals_rotated_inputs(shape: tuple[int, int, int, int], causal: bool) -> None:
    """Same output bits as plain attention on R q, R k (rotated in device memory).

    (1, 64, 4096, 128) causal runs the persistent forward schedule.
    """
    torch.manual_seed(11)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    cos, sin = ra.rope_tables(shape[2], shape[3], device="cuda")
    fused = ra.attention_rope(q, k, v, cos, sin, causal=causal)
    q_r, k_r = ra.rotate(q, cos, sin), ra.rotate(k, cos, sin)
    plain = torch.empty_like(q)
    _launch_forward(q_r, k_r, v, plain, plain, causal=causal, store_lse=False)
    assert torch.equal(fused, plain)
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_rotate_kernel_matches_oracle_and_inverts(dtype: torch.dtype) -> None:
    torch.manual_seed(5)
    x = torch.randn(2, 3, 300, 128, device="cuda", dtype=dtype)
    cos, sin = ra.rope_tables(300, 128, device="cuda")
    got = ra.rotate(x, cos, sin)
    want = orc.rope_rotate(x.cpu(), cos.cpu(), sin.cpu())
    ulp = (got.cpu().view(torch.int16).int() - want.view(torch.int16).int()).abs()
    assert int(ulp.max()) <= 1
    back = ra.rotate(got, cos, sin, transpose=True)
    assert_relative_frobenius(back.float(), x.float(), max_relative_error=1e-2)
    inplace = x.clone()
    ra.rotate(inplace, cos, sin, out=inplace)
    assert torch.equal(inplace, got)
    check_device_status()


@pytest.mark.gpu
@gpu
def test_inference_and_training_forward_agree() -> None:
    torch.manual_seed(2)
    shape = (1, 4, 513, 128)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.float16) for _ in range(3))
    cos, sin = ra.rope_tables(513, 128, device="cuda")
    with torch.no_grad():
        inference = ra.attention_rope_causal(q, k, v, cos, sin)
    training = ra.attention_rope_causal(q.requires_grad_(), k, v, cos, sin)
    assert torch.equal(inference, training.detach())
    # Identity tables (angle 0) make it plain attention.
    ones, zeros = torch.ones_like(cos), torch.zeros_like(sin)
    with torch.no_grad():
        assert torch.equal(ra.attention_rope_noncausal(q, k, v, ones, zeros), attention_noncausal(q, k, v))
    check_device_status()

"""GPU: head dims 136..256.

The forward (persistent 192- and 256-column kernels, 64-key tiles) and the
backward (two CTAs per 128-key tile, one head-dim half each) against the
CPU fp32 oracle (``manual_forward_lse`` / ``manual_backward``, the
reference's ``tests/test_flash_attention_backward.py:32-64`` algebra) at
the north-star bounds, including ragged lengths, several key tiles per head, a
long causal problem checked on sampled slabs, the public autograd path, and
deterministic mode (no deterministic kernel at these widths: it raises, or
warns under ``warn_only``).
"""

from __future__ import annotations

import pytest
import torch

from oracle.attention_oracle import chunked_reference, manual_backward, manual_forward_lse
from tklab.harness.tolerances import assert_relative_frobenius, relative_frobenius_error
from tklab.kernels.flash_attention import (
    _launch_backward,
    _launch_forward,
    attention_causal,
    attention_noncausal,
    check_device_status,
)

gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required")


def test_head_dim_above_256_rejected_before_device_work() -> None:
    q = torch.zeros(1, 1, 4, 264, dtype=torch.float16)
    with pytest.raises(ValueError):
        attention_causal(q, q, q)


def _oracle(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """The CPU fp32 oracle (O, base-2 LSE), on the GPU tensors' values."""
    o, lse = manual_forward_lse(q.cpu(), k.cpu(), v.cpu(), causal=causal)
    return o, lse


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [136, 192, 200, 256])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("seq", [1, 7, 64, 65, 129, 1000])
def test_wide_head_forward_matches_sdpa(dtype: torch.dtype, head_dim: int, causal: bool, seq: int) -> None:
    torch.manual_seed(13 * head_dim + seq + int(causal))
    shape = (2, 3, seq, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=dtype) for _ in range(3))
    output = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:3], float("nan"), device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference, expected = _oracle(q, k, v, causal)
    assert torch.isfinite(output).all()
    assert_relative_frobenius(output.float().cpu(), reference, max_relative_error=2e-2)
    assert (output.float().cpu() - reference).abs().max().item() <= 2e-2
    assert (lse.cpu() - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("head_dim", [176, 256])
@pytest.mark.parametrize("causal", [False, True])
def test_wide_head_forward_many_units_per_cta(head_dim: int, causal: bool) -> None:
    """Enough (batch, head) slabs that every persistent CTA walks several work units, with an odd
    number of query tiles (1100 rows: 9 tiles, the middle one an unpaired causal unit)."""
    torch.manual_seed(17 + head_dim + int(causal))
    shape = (2, 48, 1100, head_dim)
    q, k, v = (torch.randn(shape, device="cuda", dtype=torch.bfloat16) for _ in range(3))
    output = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:3], float("nan"), device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference, expected = _oracle(q, k, v, causal)
    assert torch.isfinite(output).all()
    assert_relative_frobenius(output.float().cpu(), reference, max_relative_error=2e-2)
    assert (output.float().cpu() - reference).abs().max().item() <= 3e-2
    assert (lse.cpu() - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    again = torch.empty_like(q)
    _launch_forward(q, k, v, again, lse, causal=causal, store_lse=True)
    assert torch.equal(again, output)
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("causal", [False, True])
def test_wide_head_forward_growing_scores(causal: bool) -> None:
    """Scores that grow along the keys move every row's running maximum many times (the O rescale
    path), with a spread of 2^10 in base 2 across a row."""
    torch.manual_seed(5)
    seq, head_dim = 777, 256
    q = torch.randn(1, 2, seq, head_dim, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(1, 2, seq, head_dim, device="cuda", dtype=torch.bfloat16)
    ramp = torch.linspace(0.2, 3.0, seq, device="cuda")[None, None, :, None]
    k = (k.float() * ramp).to(torch.bfloat16)
    v = torch.randn(1, 2, seq, head_dim, device="cuda", dtype=torch.bfloat16)
    output = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device="cuda")
    _launch_forward(q, k, v, output, lse, causal=causal, store_lse=True)
    reference, expected = _oracle(q, k, v, causal)
    assert_relative_frobenius(output.float().cpu(), reference, max_relative_error=2e-2)
    assert (output.float().cpu() - reference).abs().max().item() <= 3e-2
    assert (lse.cpu() - expected).abs().max().item() <= 1e-3 * max(1.0, expected.abs().max().item())
    check_device_status()


@pytest.mark.gpu
@gpu
def test_wide_head_public_api_inference_and_backward() -> None:
    gen = torch.Generator().manual_seed(2)
    q, k, v, do = (torch.randn(2, 4, 300, 256, generator=gen).to(torch.float16) for _ in range(4))
    qd, kd, vd = (t.cuda() for t in (q, k, v))
    with torch.no_grad():
        out_c = attention_causal(qd, kd, vd)
        out_n = attention_noncausal(qd, kd, vd)
    for out, causal in ((out_c, True), (out_n, False)):
        ref, _ = _oracle(qd, kd, vd, causal)
        assert_relative_frobenius(out.float().cpu(), ref, max_relative_error=2e-2)
    # Bitwise reproducible.
    with torch.no_grad():
        assert torch.equal(attention_causal(qd, kd, vd), out_c)
    # Training: forward under autograd, then the wide-head backward.
    qg, kg, vg = (t.clone().requires_grad_(True) for t in (qd, kd, vd))
    out = attention_causal(qg, kg, vg)
    assert torch.equal(out.detach(), out_c)
    grads = torch.autograd.grad(out, (qg, kg, vg), grad_outputs=do.cuda())
    check_device_status()
    for got, want in zip(grads, manual_backward(q, k, v, do, causal=True), strict=True):
        assert torch.isfinite(got).all()
        assert (got.float().cpu() - want).abs().max().item() <= 5e-2
        assert relative_frobenius_error(got.float().cpu(), want) < 2e-2


def _wide_backward(q, k, v, do, causal):
    qd, kd, vd, dod = (t.cuda() for t in (q, k, v, do))
    b, h, s, _ = q.shape
    o = torch.full_like(qd, float("nan"))
    lse = torch.full((b, h, s), float("nan"), device="cuda")
    _launch_forward(qd, kd, vd, o, lse, causal=causal, store_lse=True)
    grads = _launch_backward(qd, kd, vd, o, lse, dod, causal=causal, deterministic=False)
    check_device_status()
    return [g.float().cpu() for g in grads]


def _check_grads(got, want, seq) -> None:
    for name, g, w in zip(("dq", "dk", "dv"), got, want, strict=True):
        assert torch.isfinite(g).all(), name
        if seq == 1 and name in ("dq", "dk"):
            # One key: dS is identically zero, so dQ and dK are exactly zero.
            assert g.abs().max().item() <= 1e-3, name
            continue
        assert (g - w).abs().max().item() <= 5e-2, name
        assert relative_frobenius_error(g, w) < 2e-2, name


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [136, 192, 200, 256])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("seq", [1, 7, 63, 64, 65, 127, 128, 129, 300])
def test_wide_head_backward_matches_oracle(dtype: torch.dtype, head_dim: int, causal: bool, seq: int) -> None:
    gen = torch.Generator().manual_seed(1000 + 7 * head_dim + seq + int(causal))
    shape = (2, 3, seq, head_dim)
    q, k, v, do = (torch.randn(shape, generator=gen).to(dtype) for _ in range(4))
    got = _wide_backward(q, k, v, do, causal)
    _check_grads(got, manual_backward(q, k, v, do, causal=causal), seq)


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize(("head_dim", "causal", "seq"), [(256, True, 1000), (256, False, 1000), (176, True, 777)])
def test_wide_head_backward_several_key_tiles(head_dim: int, causal: bool, seq: int) -> None:
    gen = torch.Generator().manual_seed(head_dim + seq)
    shape = (1, 4, seq, head_dim)
    q, k, v, do = (torch.randn(shape, generator=gen).to(torch.bfloat16) for _ in range(4))
    got = _wide_backward(q, k, v, do, causal)
    _check_grads(got, manual_backward(q, k, v, do, causal=causal), seq)


@pytest.mark.gpu
@gpu
def test_wide_head_backward_long_causal_sampled_slabs() -> None:
    """(1, 16, 4096, 256) causal bf16: the whole problem on the GPU, three slabs against the chunked oracle."""
    shape = (1, 16, 4096, 256)
    gen = torch.Generator(device="cuda").manual_seed(0)
    q, k, v, do = (torch.randn(shape, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(4))
    o = torch.full_like(q, float("nan"))
    lse = torch.full(shape[:3], float("nan"), device="cuda")
    _launch_forward(q, k, v, o, lse, causal=True, store_lse=True)
    dq, dk, dv = _launch_backward(q, k, v, o, lse, do, causal=True, deterministic=False)
    check_device_status()
    for t in (dq, dk, dv):
        assert torch.isfinite(t).all()
    for i in (0, 7, 15):
        sl = [t[:, i : i + 1].cpu() for t in (q, k, v, do)]
        _, _, rdq, rdk, rdv = chunked_reference(*sl, causal=True, chunk=1024)
        for g, w in ((dq, rdq), (dk, rdk), (dv, rdv)):
            got = g[:, i : i + 1].float().cpu()
            assert (got - w).abs().max().item() <= 5e-2
            assert relative_frobenius_error(got, w) < 2e-2


@pytest.mark.gpu
@gpu
def test_wide_head_deterministic_mode_has_no_kernel() -> None:
    gen = torch.Generator().manual_seed(3)
    q, k, v, do = (torch.randn(1, 2, 130, 192, generator=gen).to(torch.bfloat16).cuda() for _ in range(4))
    o = torch.empty_like(q)
    lse = torch.empty(q.shape[:3], device="cuda")
    _launch_forward(q, k, v, o, lse, causal=True, store_lse=True)
    with pytest.raises(RuntimeError, match="does not have a deterministic implementation"):
        _launch_backward(q, k, v, o, lse, do, causal=True, deterministic=True)
    previous = (torch.are_deterministic_algorithms_enabled(), torch.is_deterministic_algorithms_warn_only_enabled())
    try:
        torch.use_deterministic_algorithms(True, warn_only=True)
        with pytest.warns(UserWarning, match="does not have a deterministic implementation"):
            grads = _launch_backward(q, k, v, o, lse, do, causal=True)
    finally:
        torch.use_deterministic_algorithms(previous[0], warn_only=previous[1])
    check_device_status()
    assert all(torch.isfinite(g).all() for g in grads)

"""Flash attention with rotate-half RoPE fused into the Q tile loads (B200).

``attention_rope(q, k, v, cos, sin, causal=...)`` computes
``attention(rope(q), rope(k), v)`` where ``rope`` is the reference's
rotate-half rotary embedding (``src/tklab/kernels/rope.py:27-74`` and its
public ``rope`` at ``:310-316``): for position p and half width h,
``out[:h] = x[:h] cos[p] - x[h:] sin[p]``, ``out[h:] = x[h:] cos[p] + x[:h]
sin[p]``, in fp32, rounded to the input dtype.  In the reference, RoPE is a
separate 2-D op run before attention; here the forward kernel rotates each
Q tile in shared memory right after its TMA load (the rotated Q never
exists in device memory), and K is rotated once into a workspace by an
elementwise pass: every CTA streams every K tile, so rotating K inside the
kernel would repeat the rotation once per query tile (measured 3x slower
than this split).

Tables ``cos`` and ``sin`` are ``(seq_len, head_dim // 2)`` (any float
dtype; converted to contiguous fp32), indexed by the position only and
shared by every batch and head.  head_dim must be 64 or 128.  They are
treated as constants: no gradient flows to them (the reference's ``rope``
returns table gradients; its attention has no RoPE).

Backward: the rotated Q is materialised (``tk_rope_rotate``; the forward's
rotated K is reused), the fused backward runs on them, and the gradients
are rotated back with the transpose rotation (``tk_attn_dq_convert_rope``
for dQ, in place on dK), exactly the chain rule of ``attention(R q, R k,
v)``.
"""

from __future__ import annotations

import math
from functools import partial
from typing import Any, cast

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from tklab import _native
from tklab.harness.addressing import assert_int32_addressable
from tklab.harness.tolerances import assert_relative_frobenius
from tklab.kernels.flash_attention import (
    MAX_HEAD_DIM,
    _BATCH,
    _HEADS,
    _NATIVE_DTYPE,
    _after_launch,
    _flops_factory,
    _metadata_factory,
    _on_device,
    _stream,
    _validate,
)
from tklab.registry import BenchmarkCall, BenchmarkCallFactory, KernelSpec, LaunchFn, TensorArgs, TensorFn, register

ROPE_HEAD_DIMS = (64, 128)
_ROPE_HEAD_DIM = 64  # registered benchmark problem: the reference attention shape


def _validate_rope(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor]:
    """Validate the RoPE-attention contract; return the tables as contiguous fp32."""
    if q.ndim == 4 and q.shape[-1] not in ROPE_HEAD_DIMS:
        raise ValueError("attention with RoPE requires head_dim 64 or 128")
    if cos.ndim != 2 or sin.ndim != 2:
        raise ValueError("rope expects 2D angle tables")
    if q.ndim == 4:
        expected = (q.shape[2], q.shape[3] // 2)
        if tuple(cos.shape) != expected or tuple(sin.shape) != expected:
            raise ValueError("cos and sin must have shape (seq_len, head_dim // 2)")
    if not (cos.is_floating_point() and sin.is_floating_point()):
        raise ValueError("cos and sin must be floating-point tables")
    _validate(q, k, v, max_head_dim=MAX_HEAD_DIM)
    if cos.device != q.device or sin.device != q.device:
        raise ValueError("q, cos, and sin must be on the same device")
    cos32 = cos.detach().to(torch.float32).contiguous()
    sin32 = sin.detach().to(torch.float32).contiguous()
    for name, tensor in (("cos", cos32), ("sin", sin32)):
        assert_int32_addressable(tensor, name=name)
    return cos32, sin32


def _launch_forward_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos32: torch.Tensor,
    sin32: torch.Tensor,
    output: torch.Tensor,
    softmax_lse: torch.Tensor | None,
    k_rot: torch.Tensor,
    *,
    causal: bool,
) -> None:
    """Launch the RoPE forward into preallocated buffers (LSE when given); ``k_rot`` receives R k."""
    batch, heads, n_ctx, head_dim = q.shape
    if output.shape != q.shape or output.dtype != q.dtype or not output.is_contiguous():
        raise ValueError("attention output metadata must match Q")
    if k_rot.shape != k.shape or k_rot.dtype != k.dtype or not k_rot.is_contiguous():
        raise ValueError("rotated-K workspace metadata must match K")
    lib = _native.load()
    with _on_device(q.device):
        status = lib.tk_attn_fwd_rope(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), cos32.data_ptr(), sin32.data_ptr(), k_rot.data_ptr(),
            output.data_ptr(), None if softmax_lse is None else softmax_lse.data_ptr(),
            batch, heads, n_ctx, head_dim, _NATIVE_DTYPE[q.dtype], int(bool(causal)),
            1.0 / math.sqrt(head_dim), _stream(q),
        )
    _native.check(status, "tk_attn_fwd_rope")
    _after_launch(q.device)


def rotate(
    x: torch.Tensor, cos32: torch.Tensor, sin32: torch.Tensor, *, transpose: bool = False,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """``R x`` (or ``R^T x``) for a contiguous (batch, heads, seq, head_dim) tensor, on the GPU."""
    batch, heads, n_ctx, head_dim = x.shape
    result = torch.empty_like(x) if out is None else out
    lib = _native.load()
    with _on_device(x.device):
        status = lib.tk_rope_rotate(
            x.data_ptr(), result.data_ptr(), cos32.data_ptr(), sin32.data_ptr(),
            batch, heads, n_ctx, head_dim, _NATIVE_DTYPE[x.dtype], int(transpose), _stream(x),
        )
    _native.check(status, "tk_rope_rotate")
    return result


def _launch_backward_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    softmax_lse: torch.Tensor,
    do: torch.Tensor,
    cos32: torch.Tensor,
    sin32: torch.Tensor,
    *,
    causal: bool,
    k_rot: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of ``attention(R q, R k, v)``: the fused backward on (R q, R k), then R^T.

    ``k_rot`` (R k, kept from the forward) saves rotating K again."""
    if do.shape != q.shape or do.device != q.device or do.dtype != q.dtype:
        raise ValueError("attention upstream gradient metadata must match Q")
    do = do.contiguous()
    batch, heads, n_ctx, head_dim = q.shape
    q_rot = rotate(q, cos32, sin32)
    if k_rot is None:
        k_rot = rotate(k, cos32, sin32)
    delta = torch.empty((batch, heads, n_ctx), dtype=torch.float32, device=q.device)
    dq_accum = torch.empty((batch, heads, n_ctx, head_dim), dtype=torch.float32, device=q.device)
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    dtype = _NATIVE_DTYPE[q.dtype]
    lib = _native.load()
    with _on_device(q.device):
        stream = _stream(q)
        status = lib.tk_attn_bwd_pre(
            output.data_ptr(), do.data_ptr(), delta.data_ptr(), dq_accum.data_ptr(),
            batch, heads, n_ctx, head_dim, dtype, stream,
        )
        _native.check(status, "tk_attn_bwd_pre")
        status = lib.tk_attn_bwd_fused(
            q_rot.data_ptr(), k_rot.data_ptr(), v.data_ptr(), do.data_ptr(), softmax_lse.data_ptr(),
            delta.data_ptr(), dq_accum.data_ptr(), dk.data_ptr(), dv.data_ptr(),
            batch, heads, n_ctx, head_dim, dtype, int(bool(causal)), 1.0 / math.sqrt(head_dim), stream,
        )
        _native.check(status, "tk_attn_bwd_fused")
        status = lib.tk_attn_dq_convert_rope(
            dq_accum.data_ptr(), dq.data_ptr(), cos32.data_ptr(), sin32.data_ptr(),
            batch, heads, n_ctx, head_dim, dtype, stream,
        )
        _native.check(status, "tk_attn_dq_convert_rope")
    rotate(dk, cos32, sin32, transpose=True, out=dk)
    _after_launch(q.device)
    return dq, dk, dv


class _RopeAttentionFunction(torch.autograd.Function):
    """Autograd bridge: forward saves Q/K/V, O, the LSE and the tables."""

    @staticmethod
    def forward(
        ctx: Any,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        cos: torch.Tensor,
        sin: torch.Tensor,
        causal: bool,
    ) -> torch.Tensor:
        """Fused RoPE forward with the statistic stored for the backward."""
        cos32, sin32 = _validate_rope(q, k, v, cos, sin)
        output = torch.empty_like(q)
        batch, heads, n_ctx, _ = q.shape
        softmax_lse = torch.empty((batch, heads, n_ctx), dtype=torch.float32, device=q.device)
        k_rot = torch.empty_like(k)
        _launch_forward_rope(q, k, v, cos32, sin32, output, softmax_lse, k_rot, causal=causal)
        ctx.save_for_backward(q, k, v, output, softmax_lse, cos32, sin32, k_rot)
        ctx.causal = causal
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx: Any, do: torch.Tensor) -> tuple[Any, ...]:
        """Q, K and V gradients; the tables are constants."""
        q, k, v, output, softmax_lse, cos32, sin32, k_rot = ctx.saved_tensors
        dq, dk, dv = _launch_backward_rope(
            q, k, v, output, softmax_lse, do, cos32, sin32, causal=ctx.causal, k_rot=k_rot
        )
        return dq, dk, dv, None, None, None


def attention_rope(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    causal: bool = False,
) -> torch.Tensor:
    """``attention(rope(q), rope(k), v)`` with RoPE fused into the kernel's Q/K loads."""
    cos32, sin32 = _validate_rope(q, k, v, cos, sin)
    needs_grad = torch.is_grad_enabled() and any(t.requires_grad for t in (q, k, v))
    if not needs_grad:
        output = torch.empty_like(q)
        _launch_forward_rope(q, k, v, cos32, sin32, output, None, torch.empty_like(k), causal=causal)
        return output
    return cast(torch.Tensor, _RopeAttentionFunction.apply(q, k, v, cos, sin, causal))


def attention_rope_noncausal(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> torch.Tensor:
    """Non-causal attention with fused rotate-half RoPE on Q and K."""
    return attention_rope(q, k, v, cos, sin, causal=False)


def attention_rope_causal(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
) -> torch.Tensor:
    """Causal attention with fused rotate-half RoPE on Q and K."""
    return attention_rope(q, k, v, cos, sin, causal=True)


def rope_tables(
    sequence_length: int, head_dim: int, *, base: float = 10000.0, device: torch.device | str = "cpu"
) -> tuple[torch.Tensor, torch.Tensor]:
    """Standard rotary tables: angle[p][i] = p * base^(-2i / head_dim), fp32."""
    inv_freq = base ** (-torch.arange(0, head_dim // 2, dtype=torch.float64, device=device) * 2.0 / head_dim)
    angles = torch.arange(sequence_length, dtype=torch.float64, device=device)[:, None] * inv_freq[None, :]
    return torch.cos(angles).to(torch.float32), torch.sin(angles).to(torch.float32)


def torch_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE in PyTorch over the last dim (the reference's ``_torch_rope``, ``rope.py:319-331``)."""
    first, second = x.chunk(2, dim=-1)
    return torch.cat((first * cos - second * sin, second * cos + first * sin), dim=-1)


def _reference_factory(*, causal: bool) -> TensorFn:
    """RoPE in fp32 rounded to the input dtype, then PyTorch SDPA: the reference's two-op pipeline."""

    def reference(
        q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor
    ) -> torch.Tensor:
        """Rotate Q and K, then call scaled-dot-product attention."""
        q_r = torch_rope(q.float(), cos.float(), sin.float()).to(q.dtype)
        k_r = torch_rope(k.float(), cos.float(), sin.float()).to(k.dtype)
        return F.scaled_dot_product_attention(q_r, k_r, v, is_causal=causal)

    return reference


def _make_inputs(sequence_length: int, device: torch.device, dtype: torch.dtype) -> TensorArgs:
    """Registered-shape inputs plus standard rotary tables."""
    shape = (_BATCH, _HEADS, sequence_length, _ROPE_HEAD_DIM)
    cos, sin = rope_tables(sequence_length, _ROPE_HEAD_DIM, device=device)
    return (
        torch.randn(shape, device=device, dtype=dtype),
        torch.randn(shape, device=device, dtype=dtype),
        torch.randn(shape, device=device, dtype=dtype),
        cos,
        sin,
    )


def _make_adversarial(device: torch.device) -> TensorArgs:
    """A sequence length that is not a tile multiple: partial query and key tiles."""
    return _make_inputs(1000, device, torch.float16)


def _make_output(args: TensorArgs) -> torch.Tensor:
    return torch.empty_like(args[0])


def _launch_factory(*, causal: bool) -> LaunchFn:
    """Inference launcher (no LSE) for one masking mode."""

    def launch(args: TensorArgs, output: torch.Tensor) -> None:
        q, k, v, cos, sin = args
        cos32, sin32 = _validate_rope(q, k, v, cos, sin)
        _launch_forward_rope(q, k, v, cos32, sin32, output, None, torch.empty_like(k), causal=causal)

    return launch


def _benchmark_call_factory(*, causal: bool) -> BenchmarkCallFactory:
    """Benchmark call with the tables converted and the K workspace allocated up front."""

    def factory(args: TensorArgs, output: torch.Tensor) -> BenchmarkCall:
        q, k, v, cos, sin = args
        cos32, sin32 = _validate_rope(q, k, v, cos, sin)
        k_rot = torch.empty_like(k)
        return partial(_launch_forward_rope, q, k, v, cos32, sin32, output, None, k_rot, causal=causal)

    return factory


def _assert_rope_attention(output: torch.Tensor, reference: torch.Tensor) -> None:
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)


_SIZES = (512, 1024, 2048, 4096, 8192)

ATTENTION_ROPE_NONCAUSAL = register(
    KernelSpec(
        name="attention_rope_noncausal",
        description="Flash Attention forward (sm_100a) with rotate-half RoPE: Q rotated in the tile loads, K once.",
        triton_fn=attention_rope_noncausal,
        launch_fn=_launch_factory(causal=False),
        ref_fn=_reference_factory(causal=False),
        make_inputs=_make_inputs,
        make_output=_make_output,
        make_adversarial=_make_adversarial,
        sizes=_SIZES,
        correctness_sizes=(128, 512),
        bound="compute",
        flops=_flops_factory(causal=False),
        dtypes=(torch.float16, torch.bfloat16),
        assert_fn=_assert_rope_attention,
        benchmark_metadata=_metadata_factory(causal=False),
        benchmark_call_factory=_benchmark_call_factory(causal=False),
        compute_mode="attention_fp16_fp32acc",
        supports_interpreter=False,
    )
)

ATTENTION_ROPE_CAUSAL = register(
    KernelSpec(
        name="attention_rope_causal",
        description="Causal Flash Attention forward (sm_100a) with rotate-half RoPE: Q rotated in the tile loads, K once.",
        triton_fn=attention_rope_causal,
        launch_fn=_launch_factory(causal=True),
        ref_fn=_reference_factory(causal=True),
        make_inputs=_make_inputs,
        make_output=_make_output,
        make_adversarial=_make_adversarial,
        sizes=_SIZES,
        correctness_sizes=(128, 512),
        bound="compute",
        flops=_flops_factory(causal=True),
        dtypes=(torch.float16, torch.bfloat16),
        assert_fn=_assert_rope_attention,
        benchmark_metadata=_metadata_factory(causal=True),
        benchmark_call_factory=_benchmark_call_factory(causal=True),
        compute_mode="attention_fp16_fp32acc",
        supports_interpreter=False,
    )
)

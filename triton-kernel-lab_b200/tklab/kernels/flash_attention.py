"""Flash attention forward and backward on B200 (sm_100a), behind the
reference module's interface.

This module keeps every public and test-facing name of the reference's
``src/tklab/kernels/flash_attention.py`` (``attention_noncausal``,
``attention_causal``, ``_launch_forward``, ``_launch_backward``,
``_FlashAttentionFunction``, ``_validate``, the ``ATTENTION_*`` registry
entries ...) with the same signatures, error messages and launch semantics,
but the work is done by hand-written CUDA kernels for sm_100a in
``libtklab_attn.so`` (TMA + tcgen05 + TMEM), reached through its C ABI.
There is no Triton and no CPU fallback: without the library every call
raises.

Contract differences from the reference, all widenings:
* dtypes float16 and bfloat16 (reference: float16 only, ``:281-282``);
* head_dim any multiple of 8 from 8 to 128 (reference: 64 only,
  ``:283-284``); widths below 64 / 128 run the 64- / 128-column kernels with
  the tensor maps declaring the true width;
* head_dim 136 to 256 (multiples of 8): the forward on a 192-column
  (136..192) or 256-column (200..256) kernel (one 128-row query tile per CTA
  against 64-key tiles), the backward on a 256-column kernel (two CTAs per
  128-key tile, one head-dim half of dK/dV/dQ each, 64-query steps).  The
  deterministic backward covers head_dim up to 128; for wider heads
  deterministic mode raises (or warns, under ``warn_only``) as torch does
  for ops without a deterministic implementation.
"""

from __future__ import annotations

import functools
import math
import os
import warnings
from typing import Any, cast

import torch
import torch.nn.functional as F
from torch.autograd.function import once_differentiable

from tklab import _native
from tklab.harness.addressing import assert_int32_addressable
from tklab.harness.tolerances import assert_relative_frobenius
from tklab.registry import (
    BenchmarkMetadataFn,
    BenchmarkScalar,
    CostFn,
    KernelSpec,
    LaunchFn,
    TensorArgs,
    TensorFn,
    register,
)

# Registered benchmark problem (kept equal to the reference so the FLOP model
# and result files line up, src/tklab/kernels/flash_attention.py:27-29).
_BATCH = 1
_HEADS = 16
_HEAD_DIM = 64

# Head dims the kernels accept: multiples of 8 (16-byte rows for TMA) up to
# 256, forward and backward.  64, 128 and 256 are the kernels' native widths
# (the forward also has a 192-column one); the deterministic backward stops
# at 128.
MAX_HEAD_DIM = 256
SUPPORTED_HEAD_DIMS = tuple(range(8, MAX_HEAD_DIM + 1, 8))
MAX_FWD_HEAD_DIM = MAX_HEAD_DIM
SUPPORTED_FWD_HEAD_DIMS = SUPPORTED_HEAD_DIMS
MAX_DETERMINISTIC_HEAD_DIM = 128
_NATIVE_DTYPE = {torch.float16: _native.TK_DTYPE_F16, torch.bfloat16: _native.TK_DTYPE_BF16}

# Tile shape of the sm_100a kernels: 128 query rows x 128 keys per MMA tile;
# a forward CTA runs one query tile at head_dim <= 64 (8 warps, two CTAs per
# SM) and two at head_dim <= 128 (12 warps); backward CTA = 16 warps; K/V
# ring depth 2.
_BLOCK_M = 128
_BLOCK_N = 128
_BWD_WARPS = 16


def _fwd_warps(head_dim: int) -> int:
    return 8 if head_dim <= 64 else 12


def _fwd_stages(head_dim: int) -> int:
    return 2


# Set TKLAB_CHECK_DEVICE_STATUS=1 to synchronise after every launch and raise
# on a device-side error (bounded wait that ran out).  Off by default so
# launches stay asynchronous like the reference's Triton launches.
_CHECK_STATUS = os.environ.get("TKLAB_CHECK_DEVICE_STATUS", "0") == "1"
# TKLAB_DETERMINISTIC_BWD=1 makes the backward use the deterministic path
# (no floating-point atomics) even when torch's deterministic mode is off.
_DETERMINISTIC_ENV = os.environ.get("TKLAB_DETERMINISTIC_BWD", "0") == "1"


def _validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, max_head_dim: int = MAX_FWD_HEAD_DIM) -> None:
    """Validate the dense self-attention contract (same order as the reference, ``:267-288``).

    ``max_head_dim`` is the widest head the calling path has a kernel for
    (256 for the forward and the backward).
    """
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise ValueError("attention expects Q, K, and V shaped (batch, heads, sequence, dim)")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError("Q, K, and V must have identical shapes")
    if 0 in q.shape:
        raise ValueError("attention does not support empty dimensions")
    if q.device != k.device or q.device != v.device:
        raise ValueError("Q, K, and V must be on the same device")
    if q.device.type != "cuda":
        raise ValueError("attention requires CUDA tensors")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("Q, K, and V must have the same dtype")
    if q.dtype not in _NATIVE_DTYPE:
        raise ValueError("attention currently supports float16 and bfloat16 inputs only")
    if q.shape[-1] % 8 or not 8 <= q.shape[-1] <= MAX_FWD_HEAD_DIM:
        raise ValueError(f"attention currently requires head_dim to be a multiple of 8 from 8 to {MAX_FWD_HEAD_DIM}")
    if q.shape[-1] > max_head_dim:
        raise NotImplementedError(
            f"attention backward supports head_dim up to {max_head_dim}; head_dim {q.shape[-1]} is forward-only"
        )
    for name, tensor in (("Q", q), ("K", k), ("V", v)):
        if not tensor.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        assert_int32_addressable(tensor, name=name)


# torch's raw current-stream query (the handle Triton's launcher also uses)
# costs well under a microsecond; building a torch.cuda.Stream object for
# the same handle costs a few.
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(tensor: torch.Tensor) -> int:
    """The current CUDA stream of ``tensor``'s device, as a raw handle."""
    if _RAW_STREAM is not None:
        return int(_RAW_STREAM(tensor.device.index))
    return int(torch.cuda.current_stream(tensor.device).cuda_stream)


class _on_device:
    """``torch.cuda.device(dev)`` only when ``dev`` is not already current.

    The C ABI launches on the current CUDA device; switching (and switching
    back) costs a few microseconds of host time per call, which at small
    shapes is a visible share of the whole call.
    """

    __slots__ = ("_ctx",)

    def __init__(self, device: torch.device) -> None:
        self._ctx = None if device.index == torch.cuda.current_device() else torch.cuda.device(device)

    def __enter__(self) -> None:
        if self._ctx is not None:
            self._ctx.__enter__()

    def __exit__(self, *exc: object) -> None:
        if self._ctx is not None:
            self._ctx.__exit__(*exc)


def check_device_status(device: torch.device | int | None = None) -> None:
    """Synchronise the current stream of ``device`` and raise if a kernel
    reported a device-side error (a bounded wait that ran out)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        status = _native.device_status(int(torch.cuda.current_stream(dev).cuda_stream))
    _native.check(status, "attention kernel (device status)")


def _after_launch(device: torch.device) -> None:
    if _CHECK_STATUS:
        check_device_status(device)


def _make_output(args: TensorArgs) -> torch.Tensor:
    """Allocate the dense attention output."""
    return torch.empty_like(args[0])


def _launch_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    softmax_lse: torch.Tensor,
    *,
    causal: bool,
    store_lse: bool,
) -> None:
    """Launch online-softmax attention into preallocated buffers.

    ``softmax_lse`` receives the per-query base-2 log-sum-exp (scale
    included) when ``store_lse`` is set; otherwise it is an unused
    placeholder, exactly as in the reference launcher (``:296-347``).
    """
    _validate(q, k, v)
    _forward_checked(q, k, v, output, softmax_lse, causal=causal, store_lse=store_lse)


def _forward_checked(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    softmax_lse: torch.Tensor,
    *,
    causal: bool,
    store_lse: bool,
) -> None:
    """``_launch_forward`` after ``_validate(q, k, v)`` has passed (the buffers are still checked)."""
    if output.shape != q.shape or output.device != q.device or output.dtype != q.dtype:
        raise ValueError("attention output metadata must match Q")
    if not output.is_contiguous():
        raise ValueError("attention output must be contiguous")
    batch, heads, n_ctx, head_dim = q.shape
    lse_ptr = None
    if store_lse:
        if (
            softmax_lse.shape != (batch, heads, n_ctx)
            or softmax_lse.device != q.device
            or softmax_lse.dtype != torch.float32
            or not softmax_lse.is_contiguous()
        ):
            raise ValueError("attention log-sum-exp buffer must be contiguous float32 BxHxN")
        assert_int32_addressable(softmax_lse, name="log-sum-exp buffer")
        lse_ptr = softmax_lse.data_ptr()
    # Launches into caller buffers allocate nothing, as the reference's
    # launcher: no key-split scratch on this path.
    _forward_launch(q, k, v, output, lse_ptr, causal=causal, key_split=False)


@functools.lru_cache(maxsize=512)
def _forward_workspace_bytes(lib, device_index, batch, heads, n_ctx, head_dim, dtype_code, causal) -> int:
    """Scratch bytes of the key-split forward schedule for this shape on this device (0: not split)."""
    return int(lib.tk_attn_fwd_workspace_bytes(batch, heads, n_ctx, head_dim, dtype_code, int(causal)))


def _forward_launch(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    lse_ptr: int | None,
    *,
    causal: bool,
    key_split: bool,
) -> None:
    """The library call itself, for a validated Q/K/V and buffers whose metadata is known to match.

    ``_forward_checked`` reaches it after checking caller-supplied buffers
    (``key_split=False``: allocation-free, like the reference's launcher);
    ``_attention`` and the autograd forward call it directly with buffers
    they allocated themselves (``empty_like(q)`` and a float32 BxHxN LSE),
    and with ``key_split=True``: problems with too few query tiles for the
    device then run as key-range chunks merged by a second kernel, with
    scratch from torch's caching allocator.
    """
    batch, heads, n_ctx, head_dim = q.shape
    lib = _native.load()
    with _on_device(q.device):
        # Scratch of the key-split schedule, from torch's caching allocator
        # (stream-ordered, so it is freed safely); 0 when the problem fills
        # the device or the caller wants no allocation.
        ws_bytes = 0
        if key_split:
            ws_bytes = _forward_workspace_bytes(lib, q.device.index, batch, heads, n_ctx, head_dim,
                                                _NATIVE_DTYPE[q.dtype], bool(causal))
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
        status = lib.tk_attn_fwd_ws(
            q.data_ptr(),
            k.data_ptr(),
            v.data_ptr(),
            output.data_ptr(),
            lse_ptr,
            batch,
            heads,
            n_ctx,
            head_dim,
            _NATIVE_DTYPE[q.dtype],
            int(bool(causal)),
            1.0 / math.sqrt(head_dim),
            None if workspace is None else workspace.data_ptr(),
            ws_bytes,
            _stream(q),
        )
    _native.check(status, "tk_attn_fwd_ws")
    _after_launch(q.device)


def _launch_factory(*, causal: bool) -> LaunchFn:
    """Create an allocation-free, inference-only launcher for one masking mode."""

    def launch(args: TensorArgs, output: torch.Tensor) -> None:
        """Launch forward attention without saving backward statistics."""
        q, k, v = args
        _launch_forward(q, k, v, output, output, causal=causal, store_lse=False)

    return launch


_launch_noncausal = _launch_factory(causal=False)
_launch_causal = _launch_factory(causal=True)


def _launch_backward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    softmax_lse: torch.Tensor,
    do: torch.Tensor,
    *,
    causal: bool,
    deterministic: bool | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Run the recompute backward and return ``(dQ, dK, dV)`` (reference ``:536-607``).

    Default: two library calls, ``tk_attn_bwd_pre`` (delta = rowsum(dO * O)
    and a cleared fp32 dQ accumulator) and ``tk_attn_bwd`` (the fused tcgen05
    kernel for dK, dV and dQ, dQ added across key tiles by TMA reduce-add,
    then the dQ conversion).  ``deterministic`` (default: on when
    ``torch.are_deterministic_algorithms_enabled()`` or the environment sets
    ``TKLAB_DETERMINISTIC_BWD=1``) runs ``tk_attn_bwd_deterministic``
    instead: dK/dV from the fused kernel without its dQ path and dQ from a
    query-stationary kernel that sums the key tiles in one fixed order, so
    repeated calls return bitwise identical gradients.  That path covers
    head_dim up to 128; a wider head under deterministic mode raises
    ``RuntimeError`` (a warning and the default path under torch's
    ``warn_only``).
    """
    if do.shape != q.shape or do.device != q.device or do.dtype != q.dtype:
        raise ValueError("attention upstream gradient metadata must match Q")
    _validate(q, k, v, max_head_dim=MAX_HEAD_DIM)
    return _backward_checked(q, k, v, output, softmax_lse, do, causal=causal, deterministic=deterministic)


def _backward_checked(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    softmax_lse: torch.Tensor,
    do: torch.Tensor,
    *,
    causal: bool,
    deterministic: bool | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """``_launch_backward`` after ``do``'s metadata and ``_validate(q, k, v)`` have passed."""
    do = do.contiguous()
    batch, heads, n_ctx, head_dim = q.shape
    if (
        softmax_lse.shape != (batch, heads, n_ctx)
        or softmax_lse.dtype != torch.float32
        or not softmax_lse.is_contiguous()
    ):
        raise ValueError("attention log-sum-exp buffer must be contiguous float32 BxHxN")
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled() or _DETERMINISTIC_ENV
    if deterministic and head_dim > MAX_DETERMINISTIC_HEAD_DIM:
        message = (
            f"attention backward with head_dim {head_dim} does not have a deterministic implementation "
            f"(the deterministic backward covers head_dim up to {MAX_DETERMINISTIC_HEAD_DIM})"
        )
        if torch.is_deterministic_algorithms_warn_only_enabled() and not _DETERMINISTIC_ENV:
            warnings.warn(message, stacklevel=2)
            deterministic = False
        else:
            raise RuntimeError(message)
    # delta and (default path) the fp32 dQ accumulator share one allocation:
    # the accumulator first (16-byte aligned), delta after it (4 * n_acc
    # bytes in, a multiple of 32 because head_dim is a multiple of 8).  The
    # kernels take raw pointers, so no views are built.
    n_acc = 0 if deterministic else batch * heads * n_ctx * head_dim
    workspace = torch.empty(n_acc + batch * heads * n_ctx, dtype=torch.float32, device=q.device)
    dq_accum_ptr = workspace.data_ptr()
    delta_ptr = dq_accum_ptr + 4 * n_acc
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    lib = _native.load()
    dtype = _NATIVE_DTYPE[q.dtype]
    if deterministic:
        with _on_device(q.device):
            status = lib.tk_attn_bwd_deterministic(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), output.data_ptr(), do.data_ptr(),
                softmax_lse.data_ptr(), delta_ptr, dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
                batch, heads, n_ctx, head_dim, dtype, int(bool(causal)), 1.0 / math.sqrt(head_dim), _stream(q),
            )
            _native.check(status, "tk_attn_bwd_deterministic")
        _after_launch(q.device)
        return dq, dk, dv
    with _on_device(q.device):
        stream = _stream(q)
        status = lib.tk_attn_bwd_pre(
            output.data_ptr(), do.data_ptr(), delta_ptr, dq_accum_ptr,
            batch, heads, n_ctx, head_dim, dtype, stream,
        )
        _native.check(status, "tk_attn_bwd_pre")
        status = lib.tk_attn_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), do.data_ptr(),
            softmax_lse.data_ptr(), delta_ptr, dq_accum_ptr,
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
            batch, heads, n_ctx, head_dim, dtype, int(bool(causal)),
            1.0 / math.sqrt(head_dim), stream,
        )
        _native.check(status, "tk_attn_bwd")
    _after_launch(q.device)
    return dq, dk, dv


class _FlashAttentionFunction(torch.autograd.Function):
    """Autograd bridge: forward saves Q/K/V, O and the base-2 LSE; backward recomputes P."""

    @staticmethod
    def forward(
        ctx: Any,
        q: torch.Tensor,
        k: torch.Tensor,
        v: torch.Tensor,
        causal: bool,
    ) -> torch.Tensor:
        """Run the forward kernel with the statistic stored for the backward.

        Q, K and V were validated by ``_attention`` (the only caller).
        """
        output = torch.empty_like(q)
        batch, heads, n_ctx, _ = q.shape
        softmax_lse = torch.empty((batch, heads, n_ctx), dtype=torch.float32, device=q.device)
        _forward_launch(q, k, v, output, softmax_lse.data_ptr(), causal=causal, key_split=True)
        ctx.save_for_backward(q, k, v, output, softmax_lse)
        ctx.causal = causal
        return output

    @staticmethod
    @once_differentiable
    def backward(
        ctx: Any,
        do: torch.Tensor,
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, None]:
        """Compute Q, K and V gradients with the recompute backward."""
        q, k, v, output, softmax_lse = ctx.saved_tensors
        if do.shape != q.shape or do.device != q.device or do.dtype != q.dtype:
            raise ValueError("attention upstream gradient metadata must match Q")
        # Q, K and V passed _validate in the forward and are unchanged.
        dq, dk, dv = _backward_checked(q, k, v, output, softmax_lse, do, causal=ctx.causal)
        return dq, dk, dv, None


def _attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool,
) -> torch.Tensor:
    """Inference without saved statistics; training through autograd (reference ``:663-686``)."""
    _validate(q, k, v)
    needs_grad = torch.is_grad_enabled() and any(tensor.requires_grad for tensor in (q, k, v))
    if not needs_grad:
        output = torch.empty_like(q)
        _forward_launch(q, k, v, output, None, causal=causal, key_split=True)
        return output
    result = _FlashAttentionFunction.apply(q, k, v, causal)
    return cast(torch.Tensor, result)


def attention_noncausal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Compute dense non-causal scaled dot-product attention with autograd."""
    return _attention(q, k, v, causal=False)


def attention_causal(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """Compute dense causal scaled dot-product attention with autograd."""
    return _attention(q, k, v, causal=True)


def _reference_factory(*, causal: bool) -> TensorFn:
    """PyTorch SDPA reference for one masking mode (reference ``:699-706``)."""

    def reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """Call PyTorch scaled-dot-product attention."""
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal)

    return reference


_reference_noncausal = _reference_factory(causal=False)
_reference_causal = _reference_factory(causal=True)


def _make_inputs(
    sequence_length: int,
    device: torch.device,
    dtype: torch.dtype,
) -> TensorArgs:
    """Create contiguous self-attention inputs of the registered shape."""
    shape = (_BATCH, _HEADS, sequence_length, _HEAD_DIM)
    return (
        torch.randn(shape, device=device, dtype=dtype),
        torch.randn(shape, device=device, dtype=dtype),
        torch.randn(shape, device=device, dtype=dtype),
    )


def _make_adversarial(device: torch.device) -> TensorArgs:
    """A sequence length that is not a tile multiple: partial query and key tiles."""
    return _make_inputs(1000, device, torch.float16)


def _assert_attention(output: torch.Tensor, reference: torch.Tensor) -> None:
    """Validate attention through aggregate FP32-relative error."""
    assert_relative_frobenius(output, reference, max_relative_error=2e-2)


def attention_pairs(sequence_length: int, *, causal: bool) -> int:
    """Attended (query, key) pairs: S^2, or S(S+1)/2 under the causal mask."""
    return sequence_length * (sequence_length + 1) // 2 if causal else sequence_length**2


def _flops_factory(*, causal: bool) -> CostFn:
    """Two-matmul forward FLOP model of the reference (``:737-747``)."""

    def flops(sequence_length: int, _dtype: torch.dtype) -> int:
        """Count QK-transpose and probability-value multiply-adds."""
        return 4 * _BATCH * _HEADS * attention_pairs(sequence_length, causal=causal) * _HEAD_DIM

    return flops


def _metadata_factory(*, causal: bool) -> BenchmarkMetadataFn:
    """Tile configuration of the sm_100a forward kernel, with the reference's keys (``:750-766``)."""

    def metadata(_size: int, _dtype: torch.dtype) -> dict[str, BenchmarkScalar]:
        """Return the fixed tile shape and problem dimensions."""
        return {
            "block_m": _BLOCK_M,
            "block_n": _BLOCK_N,
            "num_warps": _fwd_warps(_HEAD_DIM),
            "num_stages": _fwd_stages(_HEAD_DIM),
            "heads": _HEADS,
            "head_dim": _HEAD_DIM,
            "causal": causal,
        }

    return metadata


_SIZES = (512, 1024, 2048, 4096, 8192)

ATTENTION_NONCAUSAL = register(
    KernelSpec(
        name="attention_noncausal",
        description="Flash Attention forward (sm_100a tcgen05) with online softmax and no mask.",
        triton_fn=attention_noncausal,
        launch_fn=_launch_noncausal,
        ref_fn=_reference_noncausal,
        make_inputs=_make_inputs,
        make_output=_make_output,
        make_adversarial=_make_adversarial,
        sizes=_SIZES,
        correctness_sizes=(128, 512),
        bound="compute",
        flops=_flops_factory(causal=False),
        dtypes=(torch.float16, torch.bfloat16),
        assert_fn=_assert_attention,
        benchmark_metadata=_metadata_factory(causal=False),
        compute_mode="attention_fp16_fp32acc",
        supports_interpreter=False,
    )
)

ATTENTION_CAUSAL = register(
    KernelSpec(
        name="attention_causal",
        description="Flash Attention forward (sm_100a tcgen05) with causal tile skipping.",
        triton_fn=attention_causal,
        launch_fn=_launch_causal,
        ref_fn=_reference_causal,
        make_inputs=_make_inputs,
        make_output=_make_output,
        make_adversarial=_make_adversarial,
        sizes=_SIZES,
        correctness_sizes=(128, 512),
        bound="compute",
        flops=_flops_factory(causal=True),
        dtypes=(torch.float16, torch.bfloat16),
        assert_fn=_assert_attention,
        benchmark_metadata=_metadata_factory(causal=True),
        compute_mode="attention_fp16_fp32acc",
        supports_interpreter=False,
    )
)

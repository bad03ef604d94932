"""Grouped-query-attention decode on B200 and its performance model.

The reference specifies contiguous GQA decode only as a model
(``docs/research/gqa_decode_model.md``): one query token per query head,
``Hq = G * Hkv`` query heads, query head ``h`` reading KV head ``h // G``
("Semantic GQA mapping"), a contiguous KV cache ``(B, Hkv, L, Dh)``.
:func:`gqa_decode` is the kernel for that workload (``tk_gqa_decode``:
split-KV with a combine pass; G = 4, 8 or 16 runs on the
tensor cores — 128-key K/V tiles by TMA, S^T = K q^T and O^T = V^T P^T with
tcgen05 — so the CUDA cores only run the softmax; other shapes use 64-key
chunks by bulk copy and CUDA-core products); :func:`decode_model` evaluates the model's
derived quantities (useful FLOPs, unique KV bytes, minimum traffic and the
intensities) so measurements can be reported against it with the model's
vocabulary kept distinct (useful vs executed work, payload-only vs minimum
traffic).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from tklab import _native
from tklab.kernels.flash_attention import _NATIVE_DTYPE, _after_launch, _on_device, _stream

DECODE_GROUPS = (1, 2, 4, 8, 16)
DECODE_HEAD_DIMS = (64, 128)
DECODE_PATHS = {"auto": -1, "cuda_cores": 0}


def set_decode_path(path: str) -> None:
    """Choose the decode kernel for the whole process.

    ``"auto"`` (default): tensor cores for G = 4, 8 or 16, the CUDA-core
    kernel otherwise; ``"cuda_cores"``: always the CUDA-core
    kernel (for A/B measurements and cross-checks).
    """
    if path not in DECODE_PATHS:
        raise ValueError(f"decode path must be one of {tuple(DECODE_PATHS)}")
    _native.check(_native.load().tk_gqa_decode_set_path(DECODE_PATHS[path]), "tk_gqa_decode_set_path")


@dataclass(frozen=True, slots=True)
class DecodeModel:
    """Derived quantities of the decode model for one geometry (all ``[D]`` in its labels)."""

    n_k: int  # N_K = B Hkv L Dh
    n_v: int
    flops_qk_useful: int  # 2 B Hq L Dh
    flops_pv_useful: int
    flops_useful: int  # F_decode_useful = 4 B Hq L Dh
    bytes_kv_unique: float  # 2 sKV B Hkv L Dh
    bytes_q: float  # sQ B Hq Dh
    bytes_o: float  # sO B Hq Dh
    bytes_min: float  # KV unique + Q + O + quantisation metadata
    intensity_kv_ideal: float  # F_useful / Bytes_KV_unique = 2 G / sKV
    intensity_min: float  # F_useful / Bytes_min


def decode_model(
    batch: int,
    q_heads: int,
    kv_heads: int,
    head_dim: int,
    seq_kv: int,
    *,
    kv_bytes: float = 2.0,
    q_bytes: float = 2.0,
    o_bytes: float = 2.0,
    quant_metadata_bytes: float = 0.0,
) -> DecodeModel:
    """The model's quantities (``gqa_decode_model.md`` "Unique compulsory KV payload",
    "Useful and executed work", "Operational intensity").

    Raises:
        ValueError: If ``q_heads`` is not divisible by ``kv_heads`` or a size
            is not positive.
    """
    if min(batch, q_heads, kv_heads, head_dim, seq_kv) <= 0:
        raise ValueError("decode model sizes must be positive")
    if q_heads % kv_heads:
        raise ValueError("the model assumes Hq divisible by Hkv")
    n_k = batch * kv_heads * seq_kv * head_dim
    flops_half = 2 * batch * q_heads * seq_kv * head_dim
    bytes_kv = 2 * kv_bytes * batch * kv_heads * seq_kv * head_dim
    bytes_q = q_bytes * batch * q_heads * head_dim
    bytes_o = o_bytes * batch * q_heads * head_dim
    bytes_min = bytes_kv + bytes_q + bytes_o + quant_metadata_bytes
    flops = 2 * flops_half
    return DecodeModel(
        n_k=n_k,
        n_v=n_k,
        flops_qk_useful=flops_half,
        flops_pv_useful=flops_half,
        flops_useful=flops,
        bytes_kv_unique=bytes_kv,
        bytes_q=bytes_q,
        bytes_o=bytes_o,
        bytes_min=bytes_min,
        intensity_kv_ideal=flops / bytes_kv,
        intensity_min=flops / bytes_min,
    )


def _validate(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_lens: torch.Tensor | None) -> torch.Tensor:
    """Check the decode contract; return q as a contiguous (B, Hq, Dh) view."""
    if k.ndim != 4 or v.ndim != 4 or k.shape != v.shape:
        raise ValueError("K and V caches must be identical (batch, kv_heads, seq_kv, head_dim) tensors")
    if q.ndim == 4:
        if q.shape[2] != 1:
            raise ValueError("decode takes one query token per head")
        q = q[:, :, 0]
    if q.ndim != 3:
        raise ValueError("q must be (batch, q_heads, head_dim) or (batch, q_heads, 1, head_dim)")
    batch, q_heads, head_dim = q.shape
    if k.shape[0] != batch or k.shape[3] != head_dim or 0 in k.shape:
        raise ValueError("q and the KV cache disagree on batch or head_dim")
    if q_heads % k.shape[1]:
        raise ValueError("q_heads must be a multiple of kv_heads")
    if q_heads // k.shape[1] not in DECODE_GROUPS:
        raise ValueError(f"GQA decode supports groups of {DECODE_GROUPS} query heads per KV head")
    if head_dim not in DECODE_HEAD_DIMS:
        raise ValueError("GQA decode supports head_dim 64 or 128")
    if q.dtype != k.dtype or q.dtype != v.dtype or q.dtype not in _NATIVE_DTYPE:
        raise ValueError("q, K and V must share one dtype: float16 or bfloat16")
    if q.device != k.device or q.device != v.device:
        raise ValueError("q, K and V must be on the same device")
    if q.device.type != "cuda":
        raise ValueError("GQA decode requires CUDA tensors")
    if not (k.is_contiguous() and v.is_contiguous()):
        raise ValueError("K and V caches must be contiguous")
    if kv_lens is not None:
        if kv_lens.shape != (batch,) or kv_lens.dtype != torch.int32 or kv_lens.device != q.device:
            raise ValueError("kv_lens must be an int32 tensor of shape (batch,) on the cache's device")
    return q.contiguous()


def gqa_decode(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    kv_lens: torch.Tensor | None = None,
    return_lse: bool = False,
) -> torch.Tensor | tuple[torch.Tensor, torch.Tensor]:
    """``softmax(q . K^T / sqrt(Dh)) V`` per query head over its KV head's first ``kv_lens[b]`` keys.

    Returns ``o`` shaped like ``q`` (and the base-2 log-sum-exp, scale
    included, shaped (batch, q_heads) when ``return_lse``).  A batch with no
    valid key gets ``o = 0`` and ``lse = -inf``.
    """
    q3 = _validate(q, k, v, kv_lens)
    batch, q_heads, head_dim = q3.shape
    kv_heads, seq_kv = k.shape[1], k.shape[2]
    lib = _native.load()
    out = torch.empty_like(q3)
    lse = torch.empty((batch, q_heads), dtype=torch.float32, device=q.device) if return_lse else None
    ws_bytes = int(lib.tk_gqa_decode_workspace_bytes(batch, q_heads, seq_kv, head_dim))
    workspace = torch.empty(max(ws_bytes // 4, 1), dtype=torch.float32, device=q.device)
    with _on_device(q.device):
        status = lib.tk_gqa_decode(
            q3.data_ptr(), k.data_ptr(), v.data_ptr(), None if kv_lens is None else kv_lens.data_ptr(),
            out.data_ptr(), None if lse is None else lse.data_ptr(), workspace.data_ptr(), ws_bytes,
            batch, q_heads, kv_heads, seq_kv, head_dim, _NATIVE_DTYPE[q.dtype], 1.0 / math.sqrt(head_dim),
            _stream(q3),
        )
    _native.check(status, "tk_gqa_decode")
    _after_launch(q.device)
    result = out.view(q.shape)
    return (result, lse) if return_lse else result

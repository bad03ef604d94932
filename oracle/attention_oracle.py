"""CPU oracle for the flash-attention hot path — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
legs may import this module, and only to check or to time the reference's
CPU path.  The product path (``tklab``) never imports it: every attention
call there goes through the sm_100a kernels of ``libtklab_attn.so``.

Three restatements, each citing the reference code it follows (paths inside
the triton-kernel-lab project):

* ``sdpa_forward`` / ``sdpa_backward`` — the repo's own high-precision
  reference: ``F.scaled_dot_product_attention`` on fp32 CPU tensors
  (``src/tklab/kernels/flash_attention.py:699-706``, called with ``.float()``
  inputs as in ``tests/test_correctness.py:40``) and its autograd gradient
  (``tests/test_flash_attention_backward.py:66-76``).
* ``manual_forward_lse`` / ``manual_backward`` — the explicit fp32 algebra of
  ``tests/test_flash_attention_backward.py:32-64`` and the base-2 LSE of
  ``tests/test_flash_attention.py:70-82``.
* ``streaming_forward`` / ``streaming_backward`` — a numpy restatement of the
  reference kernels' blocked algorithm: online softmax in base 2 with
  ``scale*log2(e)`` folded in and P rounded to the input dtype before P.V
  (``flash_attention.py:54-117,120-264``), then delta, dK/dV and dQ passes
  with P = exp2(s*scale*log2(e) - LSE2) and P, dS rounded to the input dtype
  for their products (``:368-533``).  Pure numpy loops over tiles: for small
  cases only.

* ``rope_rotate`` / ``rope_attention_forward`` / ``rope_attention_backward``
  — rotate-half RoPE in fp32 rounded to the element type
  (``src/tklab/kernels/rope.py:27-74``; the transpose of ``:77-160``) and the
  reference's two-op pipeline rope → attention with its chain rule, for the
  fused RoPE attention.

* ``gqa_decode_reference`` — grouped-query decode as the reference's model
  defines it (``docs/research/gqa_decode_model.md``, "Semantic GQA
  mapping": query head h reads KV head h // G), softmax attention of one
  query token in fp32 over each batch's valid keys.

Parity is pinned: ``tests/test_oracle_golden.py`` checks all three against
golden vectors produced by the reference's own Triton kernels (run under the
Triton CPU interpreter) and its SDPA/manual references, committed under
``tests/golden/`` together with the script that made them.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

LOG2E = 1.4426950408889634


def _causal_mask(n: int, device: torch.device | None = None) -> torch.Tensor:
    """Upper triangle (key > query) that the causal mask removes."""
    return torch.triu(torch.ones(n, n, dtype=torch.bool, device=device), diagonal=1)


def sdpa_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool) -> torch.Tensor:
    """fp32 SDPA on CPU: the reference's ``ref_fn``."""
    return F.scaled_dot_product_attention(
        q.detach().float().cpu(), k.detach().float().cpu(), v.detach().float().cpu(), is_causal=causal
    )


def sdpa_backward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, do: torch.Tensor, *, causal: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """fp32 SDPA forward + autograd backward on CPU: returns (O, dQ, dK, dV)."""
    qf, kf, vf = (t.detach().float().cpu().requires_grad_(True) for t in (q, k, v))
    out = F.scaled_dot_product_attention(qf, kf, vf, is_causal=causal)
    dq, dk, dv = torch.autograd.grad(out, (qf, kf, vf), grad_outputs=do.detach().float().cpu())
    return out.detach(), dq, dk, dv


def manual_forward_lse(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool
) -> tuple[torch.Tensor, torch.Tensor]:
    """Explicit fp32 softmax attention: returns (O, base-2 LSE incl. the scale)."""
    qf, kf, vf = (t.detach().float().cpu() for t in (q, k, v))
    scale = q.shape[-1] ** -0.5
    scores = (qf @ kf.transpose(-2, -1)) * scale
    if causal:
        scores = scores.masked_fill(_causal_mask(q.shape[-2]), -torch.inf)
    lse2 = torch.logsumexp(scores, dim=-1) * math.log2(math.e)
    return torch.softmax(scores, dim=-1) @ vf, lse2


def manual_backward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, do: torch.Tensor, *, causal: bool
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Attention gradient algebra evaluated directly in fp32 (dQ, dK, dV)."""
    qf, kf, vf, dof = (t.detach().float().cpu() for t in (q, k, v, do))
    scale = q.shape[-1] ** -0.5
    scores = (qf @ kf.transpose(-2, -1)) * scale
    if causal:
        scores = scores.masked_fill(_causal_mask(q.shape[-2]), -torch.inf)
    probs = torch.softmax(scores, dim=-1)
    out = probs @ vf
    dv = probs.transpose(-2, -1) @ dof
    dprobs = dof @ vf.transpose(-2, -1)
    delta = torch.sum(dof * out, dim=-1, keepdim=True)
    dscores = probs * (dprobs - delta)
    dq = (dscores @ kf) * scale
    dk = (dscores.transpose(-2, -1) @ qf) * scale
    return dq, dk, dv


def _round(x: np.ndarray, dtype: torch.dtype) -> np.ndarray:
    """Round fp32 values to a 16-bit dtype and back (the P / dS cast before an MMA)."""
    if dtype == torch.float32:
        return x
    return torch.from_numpy(np.ascontiguousarray(x)).to(dtype).float().numpy()


def streaming_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool,
    block_m: int = 64,
    block_n: int = 32,
) -> tuple[np.ndarray, np.ndarray]:
    """Blocked online-softmax forward of the reference kernel, in numpy.

    Returns (O in fp32, base-2 LSE).  Per query block: causal runs the
    unmasked keys below the diagonal block, then the diagonal block with
    ``m >= n``; non-causal runs every key block; keys ``>= S`` are masked.
    """
    b, h, s, d = q.shape
    p_dtype = q.dtype
    qn, kn, vn = (t.detach().float().cpu().numpy() for t in (q, k, v))
    scale_log2 = np.float32((1.0 / math.sqrt(d)) * LOG2E)
    out = np.zeros((b, h, s, d), dtype=np.float32)
    lse = np.zeros((b, h, s), dtype=np.float32)
    for bi in range(b):
        for hi in range(h):
            for m0 in range(0, s, block_m):
                rows = np.arange(m0, m0 + block_m)
                qb = np.zeros((block_m, d), np.float32)
                valid_rows = rows < s
                qb[valid_rows] = qn[bi, hi, rows[valid_rows]]
                acc = np.zeros((block_m, d), np.float32)
                row_sum = np.zeros(block_m, np.float32)
                row_max = np.full(block_m, -np.inf, np.float32)
                if causal:
                    stages = [(0, m0, False), (m0, m0 + block_m, True)]
                else:
                    stages = [(0, s, False)]
                for lo, hi_n, diag in stages:
                    for n0 in range(lo, hi_n, block_n):
                        cols = np.arange(n0, n0 + block_n)
                        key_ok = cols < s
                        kb = np.zeros((block_n, d), np.float32)
                        vb = np.zeros((block_n, d), np.float32)
                        kb[key_ok] = kn[bi, hi, cols[key_ok]]
                        vb[key_ok] = vn[bi, hi, cols[key_ok]]
                        scores = (qb @ kb.T).astype(np.float32) * scale_log2
                        mask = np.broadcast_to(key_ok[None, :], scores.shape)
                        if diag:
                            mask = mask & (rows[:, None] >= cols[None, :])
                        scores = np.where(mask, scores, -np.inf).astype(np.float32)
                        new_max = np.maximum(row_max, scores.max(axis=1))
                        with np.errstate(invalid="ignore"):
                            probs = np.exp2(scores - new_max[:, None]).astype(np.float32)
                            corr = np.exp2(row_max - new_max).astype(np.float32)
                        probs = np.nan_to_num(probs, nan=0.0)
                        corr = np.nan_to_num(corr, nan=0.0)
                        acc = acc * corr[:, None] + _round(probs, p_dtype) @ vb
                        row_sum = row_sum * corr + probs.sum(axis=1)
                        row_max = new_max
                res = acc / row_sum[:, None]
                out[bi, hi, rows[valid_rows]] = res[valid_rows]
                lse[bi, hi, rows[valid_rows]] = (row_max + np.log2(row_sum))[valid_rows]
    return out, lse


def streaming_backward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    o: torch.Tensor,
    lse: np.ndarray,
    do: torch.Tensor,
    *,
    causal: bool,
    block: int = 64,
) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Blocked recompute backward of the reference kernels, in numpy: (dQ, dK, dV) in fp32."""
    b, h, s, d = q.shape
    p_dtype = q.dtype
    qn, kn, vn, on, don = (t.detach().float().cpu().numpy() for t in (q, k, v, o, do))
    scale = np.float32(1.0 / math.sqrt(d))
    scale_log2 = np.float32(scale * LOG2E)
    delta = np.sum(on * don, axis=-1).astype(np.float32)
    dq = np.zeros_like(qn)
    dk = np.zeros_like(kn)
    dv = np.zeros_like(vn)
    for bi in range(b):
        for hi in range(h):
            for n0 in range(0, s, block):
                cols = np.arange(n0, n0 + block)
                key_ok = cols < s
                start = (n0 // block) * block if causal else 0
                for m0 in range(start, s, block):
                    rows = np.arange(m0, m0 + block)
                    q_ok = rows < s
                    qb = np.zeros((block, d), np.float32)
                    dob = np.zeros((block, d), np.float32)
                    qb[q_ok] = qn[bi, hi, rows[q_ok]]
                    dob[q_ok] = don[bi, hi, rows[q_ok]]
                    kb = np.zeros((block, d), np.float32)
                    vb = np.zeros((block, d), np.float32)
                    kb[key_ok] = kn[bi, hi, cols[key_ok]]
                    vb[key_ok] = vn[bi, hi, cols[key_ok]]
                    lse_b = np.zeros(block, np.float32)
                    del_b = np.zeros(block, np.float32)
                    lse_b[q_ok] = lse[bi, hi, rows[q_ok]]
                    del_b[q_ok] = delta[bi, hi, rows[q_ok]]
                    scores = (qb @ kb.T) * scale_log2
                    probs = np.exp2(scores - lse_b[:, None]).astype(np.float32)
                    valid = q_ok[:, None] & key_ok[None, :]
                    if causal:
                        valid = valid & (rows[:, None] >= cols[None, :])
                    probs = np.where(valid, probs, 0.0).astype(np.float32)
                    dp = dob @ vb.T
                    ds = (probs * (dp - del_b[:, None])).astype(np.float32)
                    dv_blk = _round(probs, p_dtype).T @ dob
                    dk_blk = _round(ds, p_dtype).T @ qb
                    dq_blk = _round(ds, p_dtype) @ kb
                    dv[bi, hi, cols[key_ok]] += dv_blk[key_ok]
                    dk[bi, hi, cols[key_ok]] += dk_blk[key_ok]
                    dq[bi, hi, rows[q_ok]] += dq_blk[q_ok]
    return dq * scale, dk * scale, dv


def chunked_reference(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    do: torch.Tensor,
    *,
    causal: bool,
    chunk: int = 1024,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """The manual fp32 algebra above, evaluated one query chunk at a time.

    Same mathematics as ``manual_forward_lse`` + ``manual_backward`` but the
    score matrix never exceeds ``chunk x S`` per (batch, head), so long
    sequences (S = 16384) can be checked on the host.  Returns
    (O, base-2 LSE, dQ, dK, dV) in fp32.
    """
    qf, kf, vf, dof = (t.detach().float().cpu() for t in (q, k, v, do))
    s = q.shape[-2]
    scale = q.shape[-1] ** -0.5
    out = torch.empty_like(qf)
    lse = torch.empty(qf.shape[:-1])
    dq = torch.empty_like(qf)
    dk = torch.zeros_like(kf)
    dv = torch.zeros_like(vf)
    for m0 in range(0, s, chunk):
        m1 = min(s, m0 + chunk)
        scores = (qf[..., m0:m1, :] @ kf.transpose(-2, -1)) * scale
        if causal:
            rows = torch.arange(m0, m1)[:, None]
            cols = torch.arange(s)[None, :]
            scores = scores.masked_fill(cols > rows, -torch.inf)
        lse_nat = torch.logsumexp(scores, dim=-1)
        probs = torch.exp(scores - lse_nat[..., None])
        o_c = probs @ vf
        out[..., m0:m1, :] = o_c
        lse[..., m0:m1] = lse_nat * math.log2(math.e)
        do_c = dof[..., m0:m1, :]
        dv += probs.transpose(-2, -1) @ do_c
        dprobs = do_c @ vf.transpose(-2, -1)
        delta = torch.sum(do_c * o_c, dim=-1, keepdim=True)
        dscores = probs * (dprobs - delta)
        dq[..., m0:m1, :] = (dscores @ kf) * scale
        dk += (dscores.transpose(-2, -1) @ qf[..., m0:m1, :]) * scale
    return out, lse, dq, dk, dv


# ---------------------------------------------------------------------------
# Rotate-half RoPE (reference src/tklab/kernels/rope.py:27-74 forward,
# :77-160 backward = transpose rotation) and the rope -> attention pipeline.
# ---------------------------------------------------------------------------
def rope_rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, transpose: bool = False) -> torch.Tensor:
    """R x (or R^T x) over the last dim in fp32, rounded to x's dtype.

    ``cos``/``sin`` are (seq, dim/2) tables broadcast over the leading dims
    of ``x`` (positions along dim -2), as the fused kernel indexes them.
    """
    xf = x.float()
    half = xf.shape[-1] // 2
    first, second = xf[..., :half], xf[..., half:]
    c, s = cos.float(), sin.float()
    if transpose:
        s = -s
    out = torch.cat((first * c - second * s, second * c + first * s), dim=-1)
    return out.to(x.dtype)


def rope_attention_forward(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, *, causal: bool
) -> torch.Tensor:
    """fp32 attention of the dtype-rounded rotated Q and K (the reference's rope output feeds attention)."""
    return sdpa_forward(rope_rotate(q, cos, sin), rope_rotate(k, cos, sin), v, causal=causal)


def rope_attention_backward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    do: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    causal: bool,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """fp32 gradients: manual attention algebra on (R q, R k), then R^T on dQ and dK."""
    q_r, k_r = rope_rotate(q, cos, sin), rope_rotate(k, cos, sin)
    dq_r, dk, dv = manual_backward(q_r, k_r, v, do, causal=causal)
    dq = rope_rotate(dq_r, cos, sin, transpose=True)
    dk = rope_rotate(dk, cos, sin, transpose=True)
    return dq, dk, dv


def gqa_decode_reference(
    q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, kv_lens: torch.Tensor | None = None
) -> tuple[torch.Tensor, torch.Tensor]:
    """(o, base-2 lse) of one-token GQA decode in fp32 on the CPU.

    q (B, Hq, D), k/v (B, Hkv, L, D); a batch with no valid key gets o = 0
    and lse = -inf.
    """
    qf, kf, vf = (t.detach().float().cpu() for t in (q, k, v))
    batch, q_heads, dim = qf.shape
    kv_heads, seq = kf.shape[1], kf.shape[2]
    group = q_heads // kv_heads
    scale = dim ** -0.5
    out = torch.zeros(batch, q_heads, dim)
    lse = torch.full((batch, q_heads), -torch.inf)
    for b in range(batch):
        n = seq if kv_lens is None else max(0, min(int(kv_lens[b]), seq))
        if n == 0:
            continue
        for h in range(q_heads):
            kh, vh = kf[b, h // group, :n], vf[b, h // group, :n]
            scores = (kh @ qf[b, h]) * scale
            probs = torch.softmax(scores, dim=0)
            out[b, h] = probs @ vh
            lse[b, h] = torch.logsumexp(scores, dim=0) / math.log(2.0)
    return out, lse

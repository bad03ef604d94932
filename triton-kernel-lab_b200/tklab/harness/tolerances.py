"""Numerical acceptance policy (same thresholds as the reference harness).

Defaults per dtype follow ``src/tklab/harness/tolerances.py:7-11`` and the
relative-Frobenius rule follows ``:47-85`` of the same file.
"""

from __future__ import annotations

import torch

_TOLERANCES: dict[torch.dtype, tuple[float, float]] = {
    torch.float16: (1e-2, 1e-2),
    torch.bfloat16: (1.6e-2, 1e-2),
    torch.float32: (1e-4, 1e-5),
}


def assert_close(
    output: torch.Tensor,
    reference: torch.Tensor,
    *,
    rtol: float | None = None,
    atol: float | None = None,
) -> None:
    """Elementwise check with dtype-aware default tolerances.

    Raises ``ValueError`` for a dtype without a default and ``AssertionError``
    for non-finite output or a mismatch.
    """
    if output.dtype not in _TOLERANCES:
        raise ValueError(f"no default tolerance configured for {output.dtype}")
    if not bool(torch.isfinite(output).all()):
        raise AssertionError("output contains non-finite values")
    default_rtol, default_atol = _TOLERANCES[output.dtype]
    torch.testing.assert_close(
        output,
        reference.to(output.dtype),
        rtol=default_rtol if rtol is None else rtol,
        atol=default_atol if atol is None else atol,
    )


def relative_frobenius_error(output: torch.Tensor, reference: torch.Tensor) -> float:
    """``||output - reference|| / ||reference||`` in fp32 (absolute if the reference is 0)."""
    diff = torch.linalg.vector_norm(output.detach().float() - reference.detach().float())
    ref = torch.linalg.vector_norm(reference.detach().float())
    return float(diff if float(ref) == 0.0 else diff / ref)


def assert_relative_frobenius(
    output: torch.Tensor,
    reference: torch.Tensor,
    *,
    max_relative_error: float,
) -> None:
    """Aggregate check for large reductions: relative Frobenius error below a bound.

    Raises ``ValueError`` for a non-positive bound and ``AssertionError`` for
    non-finite tensors or an error at or above ``max_relative_error``.
    """
    if max_relative_error <= 0:
        raise ValueError("max_relative_error must be positive")
    output_float = output.float()
    reference_float = reference.float()
    if not bool(torch.isfinite(output_float).all()):
        raise AssertionError("output contains non-finite values")
    if not bool(torch.isfinite(reference_float).all()):
        raise AssertionError("reference contains non-finite values")
    error = relative_frobenius_error(output_float, reference_float)
    if error != error or error in (float("inf"), float("-inf")):
        raise AssertionError("relative Frobenius error is non-finite")
    if error >= max_relative_error:
        raise AssertionError(f"relative Frobenius error {error:.6g} exceeds {max_relative_error:.6g}")

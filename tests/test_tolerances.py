"""CPU: the numerical policy helpers (reference ``tests/test_tolerances.py``)."""

from __future__ import annotations

import pytest
import torch

from tklab.harness.addressing import assert_int32_addressable, max_relative_offset
from tklab.harness.tolerances import assert_close, assert_relative_frobenius


def test_assert_close_uses_dtype_defaults() -> None:
    x = torch.ones(4, dtype=torch.float16)
    assert_close(x, x.float() * (1 + 5e-3))
    with pytest.raises(AssertionError):
        assert_close(x, x.float() * 1.1)


def test_assert_close_rejects_unknown_dtype_and_non_finite() -> None:
    with pytest.raises(ValueError, match="no default tolerance"):
        assert_close(torch.ones(2, dtype=torch.int32), torch.ones(2))
    with pytest.raises(AssertionError, match="non-finite"):
        assert_close(torch.tensor([float("nan")]), torch.zeros(1))


def test_relative_frobenius() -> None:
    ref = torch.ones(100)
    assert_relative_frobenius(ref * 1.001, ref, max_relative_error=2e-3)
    with pytest.raises(AssertionError, match="exceeds"):
        assert_relative_frobenius(ref * 1.01, ref, max_relative_error=2e-3)
    with pytest.raises(ValueError, match="positive"):
        assert_relative_frobenius(ref, ref, max_relative_error=0.0)
    with pytest.raises(AssertionError, match="reference contains non-finite"):
        assert_relative_frobenius(ref, ref * float("inf"), max_relative_error=1.0)


def test_int32_guard() -> None:
    big = torch.empty_strided((2, 2), (2**31, 1), dtype=torch.float16, device="meta")
    assert max_relative_offset(big) == 2**31 + 1
    with pytest.raises(ValueError, match="int32 offset"):
        assert_int32_addressable(big, name="X")
    assert_int32_addressable(torch.empty(4, 4, device="meta"), name="X")

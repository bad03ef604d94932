"""CPU: pin the oracle against the reference's own outputs (golden fixtures).

The fixtures hold the reference Triton kernels' results (run by the Triton
CPU interpreter), its fp32 SDPA reference and its manual fp32 gradient
algebra, for the same seeded inputs.  Every oracle restatement must agree
with them before it is trusted as the checker of the sm_100a kernels.
"""

from __future__ import annotations

import pytest
import torch
from conftest import golden_cases, load_golden

from oracle import attention_oracle as orc
from tklab.harness.tolerances import relative_frobenius_error

CASES = golden_cases()


def test_fixture_set_is_complete() -> None:
    assert len(CASES) >= 8
    assert "c1_fp32_s256_d64_noncausal" in CASES


@pytest.mark.parametrize("name", CASES)
def test_sdpa_and_manual_oracles_match_reference_outputs(name: str) -> None:
    case = load_golden(name)
    q, k, v, do, causal = case["q"], case["k"], case["v"], case["do"], case["causal"]
    o = orc.sdpa_forward(q, k, v, causal=causal)
    assert relative_frobenius_error(o, case["sdpa_o"]) < 1e-6
    o_man, lse = orc.manual_forward_lse(q, k, v, causal=causal)
    assert relative_frobenius_error(o_man, case["sdpa_o"]) < 1e-5
    if "sdpa_dq" in case:
        _, dq, dk, dv = orc.sdpa_backward(q, k, v, do, causal=causal)
        expected = (case["sdpa_dq"], case["sdpa_dk"], case["sdpa_dv"])
        for got, want in zip((dq, dk, dv), expected, strict=True):
            assert relative_frobenius_error(got, want) < 1e-6
    else:
        grads = orc.manual_backward(q, k, v, do, causal=causal)
        expected = (case["man_dq"], case["man_dk"], case["man_dv"])
        for got, want in zip(grads, expected, strict=True):
            assert relative_frobenius_error(got, want) < 1e-6
    if "ref_lse" in case:
        assert relative_frobenius_error(lse, case["ref_lse"]) < 1e-5


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("f16_")])
def test_streaming_oracle_matches_reference_kernels(name: str) -> None:
    """The blocked restatement reproduces the reference Triton kernels' outputs."""
    case = load_golden(name)
    q, k, v, do, causal = case["q"], case["k"], case["v"], case["do"], case["causal"]
    o, lse = orc.streaming_forward(q, k, v, causal=causal)
    assert relative_frobenius_error(torch.from_numpy(o), case["ref_o"]) < 1e-3
    assert relative_frobenius_error(torch.from_numpy(lse), case["ref_lse"]) < 1e-5
    dq, dk, dv = orc.streaming_backward(q, k, v, case["ref_o"], case["ref_lse"].numpy(), do, causal=causal)
    for got, key in ((dq, "ref_dq"), (dk, "ref_dk"), (dv, "ref_dv")):
        assert relative_frobenius_error(torch.from_numpy(got), case[key]) < 2e-3, key


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("f16_")])
def test_reference_kernels_meet_the_repo_tolerances(name: str) -> None:
    """Sanity of the fixtures themselves: the reference kernels pass the reference's own bars."""
    case = load_golden(name)
    assert relative_frobenius_error(case["ref_o"], case["sdpa_o"]) < 2e-2
    for key in ("dq", "dk", "dv"):
        assert relative_frobenius_error(case[f"ref_{key}"], case[f"man_{key}"]) < 3e-2


def test_chunked_reference_matches_manual_algebra() -> None:
    gen = torch.Generator().manual_seed(11)
    shape = (1, 2, 300, 64)
    q, k, v, do = (torch.randn(shape, generator=gen) for _ in range(4))
    for causal in (False, True):
        o, lse, dq, dk, dv = orc.chunked_reference(q, k, v, do, causal=causal, chunk=64)
        o_man, lse_man = orc.manual_forward_lse(q, k, v, causal=causal)
        grads = orc.manual_backward(q, k, v, do, causal=causal)
        assert relative_frobenius_error(o, o_man) < 1e-5
        assert relative_frobenius_error(lse, lse_man) < 1e-5
        for got, want in zip((dq, dk, dv), grads, strict=True):
            assert relative_frobenius_error(got, want) < 1e-5


ROPE_CASES = golden_cases(rope=True)


def test_rope_fixture_set() -> None:
    assert ROPE_CASES == ["rope_f16_s129_d64_causal", "rope_f16_s200_d64_noncausal"]


@pytest.mark.parametrize("name", ROPE_CASES)
def test_rope_oracle_matches_reference_rope_kernel(name: str) -> None:
    """rope_rotate reproduces the reference rotate-half kernel's fp16 output.

    Both evaluate x1*c - x2*s / x2*c + x1*s in fp32 and round to fp16; the
    only freedom is whether the products are fused, which can move a result
    by one fp16 ulp on rare ties.
    """
    case = load_golden(name)
    cos, sin = case["cos"].float(), case["sin"].float()
    for src, key in (("q", "ref_qrot"), ("k", "ref_krot")):
        got = orc.rope_rotate(case[src], cos, sin)
        want = case[key]
        assert got.dtype == want.dtype == torch.float16
        bits_got = got.view(torch.int16).int()
        bits_want = want.view(torch.int16).int()
        ulp = (bits_got - bits_want).abs()
        assert int(ulp.max()) <= 1
        assert float((ulp > 0).float().mean()) < 1e-3


@pytest.mark.parametrize("name", ROPE_CASES)
def test_rope_attention_oracle_matches_reference_chain(name: str) -> None:
    """Oracle gradients of attention(R q, R k, v) equal the reference's rope -> attention chain in fp32."""
    case = load_golden(name)
    cos, sin = case["cos"].float(), case["sin"].float()
    dq, dk, dv = orc.rope_attention_backward(
        case["q"], case["k"], case["v"], case["do"], cos, sin, causal=case["causal"]
    )
    for got, key in ((dq, "man_dq"), (dk, "man_dk"), (dv, "man_dv")):
        assert relative_frobenius_error(got, case[key]) < 1e-5, key
    o = orc.rope_attention_forward(case["q"], case["k"], case["v"], cos, sin, causal=case["causal"])
    assert relative_frobenius_error(o, case["ref_o"]) < 2e-3

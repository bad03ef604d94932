"""GQA decode (``tklab.kernels.gqa_decode``): the model's derived quantities
(CPU, against the reference specification's own numerical point) and the
``tk_gqa_decode`` kernel against the fp32 oracle (GPU).
"""

from __future__ import annotations

import math

import pytest
import torch

from oracle import attention_oracle as orc
from tklab.kernels.flash_attention import check_device_status
from tklab.kernels.gqa_decode import decode_model, gqa_decode, set_decode_path

gpu = pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required")


def test_model_reference_numerical_point() -> None:
    """B=1, Hq=32, Hkv=8, G=4, Dh=128, L=4096 (gqa_decode_model.md, "Reference numerical point")."""
    m = decode_model(1, 32, 8, 128, 4096)
    assert m.n_k == m.n_v == 4_194_304
    assert m.flops_qk_useful == m.flops_pv_useful == 33_554_432
    assert m.flops_useful == 67_108_864
    assert m.bytes_kv_unique == 16_777_216
    assert m.bytes_min == 16_793_600
    assert m.intensity_min == pytest.approx(67_108_864 / 16_793_600)
    assert m.intensity_min == pytest.approx(3.9961, abs=1e-4)
    assert m.intensity_kv_ideal == pytest.approx(4.0)  # 2 G / sKV
    fp8 = decode_model(1, 32, 8, 128, 4096, kv_bytes=1.0)
    assert fp8.bytes_kv_unique == 8_388_608
    assert fp8.bytes_min == 8_404_992
    assert fp8.intensity_min == pytest.approx(7.9844, abs=1e-4)
    assert fp8.intensity_kv_ideal == pytest.approx(8.0)


def test_model_rejects_bad_geometry() -> None:
    with pytest.raises(ValueError, match="divisible"):
        decode_model(1, 30, 8, 128, 16)
    with pytest.raises(ValueError, match="positive"):
        decode_model(0, 32, 8, 128, 16)


def test_decode_validation_on_cpu() -> None:
    q = torch.zeros(1, 8, 128, dtype=torch.float16)
    k = torch.zeros(1, 2, 16, 128, dtype=torch.float16)
    with pytest.raises(ValueError, match="one query token"):
        gqa_decode(torch.zeros(1, 8, 2, 128, dtype=torch.float16), k, k)
    with pytest.raises(ValueError, match="multiple of kv_heads"):
        gqa_decode(torch.zeros(1, 7, 128, dtype=torch.float16), k, k)
    with pytest.raises(ValueError, match="groups of"):
        gqa_decode(torch.zeros(1, 6, 128, dtype=torch.float16), k, k)
    small = torch.zeros(1, 2, 16, 32, dtype=torch.float16)
    with pytest.raises(ValueError, match="head_dim 64 or 128"):
        gqa_decode(torch.zeros(1, 8, 32, dtype=torch.float16), small, small)
    with pytest.raises(ValueError, match="CUDA"):
        gqa_decode(q, k, k)


@pytest.fixture(params=["auto", "cuda_cores"])
def decode_path(request: pytest.FixtureRequest):
    """Run a test on both decode kernels (tensor cores where "auto" selects them)."""
    set_decode_path(request.param)
    yield request.param
    set_decode_path("auto")


def test_decode_path_validation() -> None:
    with pytest.raises(ValueError, match="decode path"):
        set_decode_path("tensor")


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("group", [1, 2, 4, 8, 16])
@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("seq", [1, 63, 64, 65, 127, 128, 129, 1000, 4096])
def test_decode_matches_oracle(decode_path: str, dtype: torch.dtype, group: int, head_dim: int, seq: int) -> None:
    torch.manual_seed(seq + 3 * group + head_dim)
    batch, kv_heads = 2, 2
    q = torch.randn(batch, kv_heads * group, head_dim, device="cuda", dtype=dtype)
    k = torch.randn(batch, kv_heads, seq, head_dim, device="cuda", dtype=dtype)
    v = torch.randn(batch, kv_heads, seq, head_dim, device="cuda", dtype=dtype)
    o, lse = gqa_decode(q, k, v, return_lse=True)
    ref_o, ref_lse = orc.gqa_decode_reference(q, k, v)
    assert o.shape == q.shape and o.dtype == dtype
    assert (o.float().cpu() - ref_o).abs().max().item() <= 1e-2
    assert torch.allclose(lse.cpu(), ref_lse, atol=1e-3, rtol=1e-4)
    check_device_status()


@pytest.mark.gpu
@gpu
def test_decode_ragged_lengths_and_4d_query(decode_path: str) -> None:
    torch.manual_seed(9)
    batch, kv_heads, group, seq, dim = 5, 8, 4, 777, 128
    q = torch.randn(batch, kv_heads * group, 1, dim, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(batch, kv_heads, seq, dim, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(batch, kv_heads, seq, dim, device="cuda", dtype=torch.bfloat16)
    lens = torch.tensor([777, 1, 0, 64, 500], dtype=torch.int32, device="cuda")
    o, lse = gqa_decode(q, k, v, kv_lens=lens, return_lse=True)
    assert o.shape == q.shape
    ref_o, ref_lse = orc.gqa_decode_reference(q[:, :, 0], k, v, lens.cpu())
    assert (o[:, :, 0].float().cpu() - ref_o).abs().max().item() <= 1e-2
    assert torch.equal(o[2].float().cpu(), torch.zeros_like(o[2].float().cpu()))
    assert torch.isinf(lse[2]).all() and (lse[2] < 0).all()
    finite = torch.isfinite(ref_lse)
    assert torch.allclose(lse.cpu()[finite], ref_lse[finite], atol=1e-3, rtol=1e-4)
    # Bitwise reproducible, and keys past a batch's length do not matter.
    assert torch.equal(gqa_decode(q, k, v, kv_lens=lens), o)
    k2 = k.clone()
    k2[3, :, 64:] = 1e4
    assert torch.equal(gqa_decode(q, k2, v, kv_lens=lens), o)
    check_device_status()


@pytest.mark.gpu
@gpu
@pytest.mark.parametrize("group", [4, 16])
def test_decode_tensor_core_path_agrees_with_cuda_cores(group: int) -> None:
    """The two kernels on the same inputs (a long cache with many splits, growing scores so the
    running maxima move often): equal to within the 16-bit rounding of P."""
    torch.manual_seed(21 + group)
    batch, kv_heads, seq, dim = 3, 4, 5000, 128
    q = torch.randn(batch, kv_heads * group, dim, device="cuda", dtype=torch.bfloat16)
    ramp = torch.linspace(0.1, 2.5, seq, device="cuda")[None, None, :, None]
    k = (torch.randn(batch, kv_heads, seq, dim, device="cuda") * ramp).to(torch.bfloat16)
    v = torch.randn(batch, kv_heads, seq, dim, device="cuda", dtype=torch.bfloat16)
    try:
        set_decode_path("cuda_cores")
        o_cc, lse_cc = gqa_decode(q, k, v, return_lse=True)
        set_decode_path("auto")
        o_tc, lse_tc = gqa_decode(q, k, v, return_lse=True)
        assert torch.equal(gqa_decode(q, k, v), o_tc)
    finally:
        set_decode_path("auto")
    ref_o, ref_lse = orc.gqa_decode_reference(q, k, v)
    assert (o_tc.float().cpu() - ref_o).abs().max().item() <= 1e-2
    assert (o_tc.float() - o_cc.float()).abs().max().item() <= 1e-2
    assert torch.allclose(lse_tc.cpu(), ref_lse, atol=1e-3, rtol=1e-4)
    assert torch.allclose(lse_tc, lse_cc, atol=1e-3, rtol=1e-4)
    check_device_status()


@pytest.mark.gpu
@gpu
def test_decode_equals_single_token_attention() -> None:
    """G = 1, one token: the same as SDPA of one query against the whole cache."""
    torch.manual_seed(4)
    q = torch.randn(3, 4, 64, device="cuda", dtype=torch.float16)
    k = torch.randn(3, 4, 300, 64, device="cuda", dtype=torch.float16)
    v = torch.randn(3, 4, 300, 64, device="cuda", dtype=torch.float16)
    o = gqa_decode(q, k, v)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float()[:, :, None], k.float(), v.float())[:, :, 0]
    assert (o.float() - ref).abs().max().item() <= 1e-2
    assert math.isfinite(float(o.float().abs().max()))
    check_device_status()

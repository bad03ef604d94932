"""GPU: parity at the BASELINE configurations' full sizes.

The full problems are too large for the CPU oracle to redo entirely, so each
test runs the whole problem on the GPU, then
* checks a few sampled (batch, head) slabs against the chunked fp32 oracle
  (same inputs, copied back bit-exactly),
* checks size-independent properties over the whole output: everything
  finite, the causal first row equal to V's first row, and linearity of
  attention in V (attn(q,k,v1+v2) = attn(q,k,v1) + attn(q,k,v2) up to
  rounding).
Configurations (synthetic, seeded): C2 fp16 (4,16,1024,64) non-causal;
C3 bf16 (8,32,4096,128) causal; C4 bf16 (1,32,16384,128) causal with Q and K
drawn with standard deviation 1.5.
"""

from __future__ import annotations

import pytest
import torch

from oracle.attention_oracle import chunked_reference
from tklab.harness.tolerances import relative_frobenius_error
from tklab.kernels.flash_attention import _launch_backward, _launch_forward, check_device_status

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="CUDA GPU is required"),
]

CONFIGS = {
    "c2": ((4, 16, 1024, 64), torch.float16, False, 1.0, (0, 37, 63)),
    "c3": ((8, 32, 4096, 128), torch.bfloat16, True, 1.0, (0, 131, 255)),
    "c4": ((1, 32, 16384, 128), torch.bfloat16, True, 1.5, (7,)),
}


def _inputs(shape, dtype, qk_std, seed=0):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    q = (torch.randn(shape, generator=gen, device="cuda") * qk_std).to(dtype)
    k = (torch.randn(shape, generator=gen, device="cuda") * qk_std).to(dtype)
    v = torch.randn(shape, generator=gen, device="cuda").to(dtype)
    do = torch.randn(shape, generator=gen, device="cuda").to(dtype)
    return q, k, v, do


def _slab(t: torch.Tensor, i: int) -> torch.Tensor:
    return t.reshape(-1, *t.shape[2:])[i].unsqueeze(0).unsqueeze(0).cpu()


@pytest.mark.parametrize("name", list(CONFIGS))
def test_full_size_forward_backward(name: str) -> None:
    shape, dtype, causal, qk_std, slabs = CONFIGS[name]
    q, k, v, do = _inputs(shape, dtype, qk_std)
    b, h, s, _ = shape
    o = torch.full_like(q, float("nan"))
    lse = torch.full((b, h, s), float("nan"), device="cuda")
    _launch_forward(q, k, v, o, lse, causal=causal, store_lse=True)
    dq, dk, dv = _launch_backward(q, k, v, o, lse, do, causal=causal)
    check_device_status()
    for t in (o, lse, dq, dk, dv):
        assert torch.isfinite(t).all()
    chunk = 1024 if s <= 4096 else 512
    for i in slabs:
        ro, rl, rdq, rdk, rdv = chunked_reference(
            _slab(q, i), _slab(k, i), _slab(v, i), _slab(do, i), causal=causal, chunk=chunk
        )
        got_o = _slab(o, i).float()
        assert (got_o - ro).abs().max().item() <= 2e-2, i
        assert relative_frobenius_error(got_o, ro) < 2e-2
        got_l = lse.reshape(-1, s)[i].cpu()
        assert (got_l - rl.reshape(-1)).abs().max().item() <= 1e-3 * max(1.0, rl.abs().max().item())
        for label, got, want in (("dq", dq, rdq), ("dk", dk, rdk), ("dv", dv, rdv)):
            g = _slab(got, i).float()
            assert (g - want).abs().max().item() <= 5e-2, (i, label)
            assert relative_frobenius_error(g, want) < 2e-2, (i, label)
    if causal:
        assert torch.equal(o[:, :, 0, :], v[:, :, 0, :])


@pytest.mark.parametrize("name", ["c3", "c4"])
def test_full_size_linearity_in_v(name: str) -> None:
    shape, dtype, causal, qk_std, _ = CONFIGS[name]
    q, k, v1, v2 = _inputs(shape, dtype, qk_std, seed=1)
    outs = []
    for v in (v1, v2, (v1.float() + v2.float()).to(dtype)):
        o = torch.empty_like(q)
        _launch_forward(q, k, v, o, o, causal=causal, store_lse=False)
        outs.append(o.float())
    check_device_status()
    # v1 + v2 is rounded to the input dtype once; the bound covers that
    # rounding plus the three outputs' own rounding.
    assert relative_frobenius_error(outs[2], outs[0] + outs[1]) < 1e-2

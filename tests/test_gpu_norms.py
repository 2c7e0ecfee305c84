"""The native RMSNorm kernels against the reference module's eager arithmetic on the GPU.

Reference: RMSNorm.forward (training/model.py:161-172), evaluated with torch ops in float32
statistics. The kernels reduce the sum of squares in another order, so with 16-bit inputs
an output may differ by up to two rounding steps of the input dtype (at least 99% of the
elements identical); f32 inputs agree to 1e-5 relative. Input gradients are compared with
torch's autograd of the same expression (relative Frobenius 5e-3 in 16-bit, 1e-5 in f32).
"""

from __future__ import annotations

import pytest
import torch

from moss_image_b200.norms import rms_norm

pytestmark = pytest.mark.gpu


def _reference(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    normalized = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + eps)
    return normalized.to(x.dtype) * weight


def _ulp(t: torch.Tensor) -> torch.Tensor:
    bits = {torch.bfloat16: 8, torch.float16: 11, torch.float32: 24}[t.dtype]
    mag = t.float().abs().clamp_min(torch.finfo(t.dtype).tiny)
    return torch.exp2(torch.floor(torch.log2(mag)) - (bits - 1))


CASES = [  # rows, dim, x dtype, weight dtype
    (4099, 128, torch.bfloat16, torch.bfloat16),   # per-head q/k norm (4 lanes per row)
    (300, 3072, torch.bfloat16, torch.bfloat16),   # block norm (one CTA per row)
    (5000, 3072, torch.bfloat16, torch.bfloat16),  # more rows than resident CTAs: next row prefetched
    (3000, 2048, torch.float16, torch.float16),    # two chunks per thread, prefetched
    (2000, 4096, torch.float32, torch.float32),    # f32 rows, four chunks per thread
    (257, 64, torch.float16, torch.float16),       # 2 lanes per row
    (129, 24, torch.bfloat16, torch.bfloat16),     # 1 lane per row
    (41, 1024, torch.bfloat16, torch.bfloat16),    # a full warp per row
    (130, 16384, torch.bfloat16, torch.bfloat16),  # longer than the register budget: re-read
    (77, 3072, torch.bfloat16, torch.float32),     # f32 gain: f32 output
    (64, 256, torch.float32, torch.float32),
    (33, 100, torch.bfloat16, torch.bfloat16),     # element path (dim % 8 != 0)
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_rmsnorm_matches_the_reference_module(cuda_device, case):
    rows, dim, dtype, w_dtype = CASES[case]
    gen = torch.Generator(device=cuda_device).manual_seed(case)
    x = (torch.randn(rows, dim, device=cuda_device, generator=gen) * 3).to(dtype).requires_grad_(True)
    weight = (1 + 0.1 * torch.randn(dim, device=cuda_device, generator=gen)).to(w_dtype)
    y = rms_norm(x, weight)
    ref_x = x.detach().clone().requires_grad_(True)
    expected = _reference(ref_x, weight)
    assert y.dtype == expected.dtype and y.shape == expected.shape
    diff = (y.float() - expected.float()).abs()
    if dtype == torch.float32:
        torch.testing.assert_close(y, expected, rtol=1e-5, atol=1e-6)
    else:
        # the rsqrt may differ in its last f32 bits: one step of the normalised value, which
        # the gain can turn into two steps of the output
        step = torch.maximum(_ulp(expected.detach().to(dtype)), _ulp(y.detach().to(dtype)))  # steps of x's dtype
        ulps = (diff / step).max().item()
        assert ulps <= 2, ulps
        assert (diff == 0).float().mean().item() >= 0.99
    dy = torch.randn(y.shape, device=cuda_device, generator=gen).to(y.dtype)
    y.backward(dy)
    expected.backward(dy)
    tol = 1e-5 if dtype == torch.float32 else 5e-3
    err = (x.grad.float() - ref_x.grad.float()).norm() / ref_x.grad.float().norm()
    assert err.item() <= tol


def test_rmsnorm_trainable_gain_and_edge_cases(cuda_device):
    x = torch.randn(5, 4, 128, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    weight = torch.ones(128, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    y = rms_norm(x, weight)
    assert y.shape == x.shape
    y.float().sum().backward()
    ref_w = weight.detach().clone().requires_grad_(True)
    _reference(x.detach(), ref_w).float().sum().backward()
    torch.testing.assert_close(weight.grad.float(), ref_w.grad.float(), rtol=2e-2, atol=2e-2)
    empty = torch.empty(0, 64, device=cuda_device, dtype=torch.bfloat16)
    assert rms_norm(empty, torch.ones(64, device=cuda_device, dtype=torch.bfloat16)).shape == (0, 64)
    zeros = torch.zeros(3, 64, device=cuda_device, dtype=torch.bfloat16)
    assert torch.equal(rms_norm(zeros, torch.ones(64, device=cuda_device, dtype=torch.bfloat16)), zeros)
    with pytest.raises(ValueError, match="weight"):
        rms_norm(x, torch.ones(64, device=cuda_device, dtype=torch.bfloat16))

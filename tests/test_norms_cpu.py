"""RMSNorm without a GPU: the native entry points' argument checks, the module's CPU
arithmetic (the reference's expression), and the loud failure of the CUDA-only op."""

from __future__ import annotations

import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200.dit import RMSNorm
from moss_image_b200.norms import rms_norm


def test_rmsnorm_entry_points_validate_arguments():
    lib = _lib.library()
    assert lib.moss_rmsnorm_fwd(None, 1, 0, 64, None, 1, 1e-6, None, None, None) == _lib.MOSS_OK
    assert lib.moss_rmsnorm_fwd(None, 1, 4, 64, None, 1, 1e-6, None, None, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_rmsnorm_fwd(None, 1, 4, 0, None, 1, 1e-6, None, None, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_rmsnorm_fwd(None, 5, 4, 64, None, 1, 1e-6, None, None, None) == _lib.MOSS_ERR_UNSUPPORTED
    assert lib.moss_rmsnorm_bwd(None, None, 1, 4, 64, None, 1, None, None, None) == _lib.MOSS_ERR_INVALID_ARGUMENT


def test_module_cpu_arithmetic_is_the_reference_expression():
    torch.manual_seed(2)
    norm = RMSNorm(48)
    with torch.no_grad():
        norm.weight.normal_(1.0, 0.1)
    x = torch.randn(3, 5, 48).to(torch.bfloat16)
    norm = norm.to(torch.bfloat16)
    expected = (x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + 1e-6)).to(x.dtype) * norm.weight
    assert torch.equal(norm(x), expected)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        rms_norm(x, norm.weight)

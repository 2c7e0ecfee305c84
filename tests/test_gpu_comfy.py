"""Comfy int8_tensorwise checkpoints loaded straight into the int8 GEMM modules, on the GPU.

The directly loaded modules run the sm_100a kernels on the stored codes: outputs meet the GEMM
bar (relative Frobenius 5e-3) against the oracle on the same codes, and ConvRot storage
reproduces the dense decoded layer. Re-quantising the dense decode, as a reference pipeline
does, moves codes; the direct load keeps every one.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn
from torch.nn import functional as F

from golden.comfy_cases import comfy_codes, comfy_marker
from moss_image_b200.comfy_weights import decode_comfy_state, load_comfy_quantized
from moss_image_b200.convrot import FrozenConvRotLinear
from moss_image_b200.quantization import FrozenInt8Linear
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def test_direct_modules_run_the_kernels_on_the_stored_codes(cuda_device):
    codes, scale = comfy_codes(1280, 3072, seed=11)
    rot_codes, rot_scale = comfy_codes(768, 1024, seed=12)
    state = {"a.weight": codes, "a.weight_scale": scale, "a.bias": torch.randn(1280),
             "a.comfy_quant": comfy_marker({"format": "int8_tensorwise"}),
             "b.weight": rot_codes, "b.weight_scale": rot_scale,
             "b.comfy_quant": comfy_marker({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256})}
    model = nn.ModuleDict({"a": nn.Linear(3072, 1280), "b": nn.Linear(1024, 768, bias=False)}).to(cuda_device)
    assert load_comfy_quantized(model, state, dtype=torch.bfloat16) == ["a", "b"]
    assert model["a"].weight_int8.is_cuda and isinstance(model["b"], FrozenConvRotLinear)
    x = torch.randn(77, 3072, device=cuda_device, dtype=torch.bfloat16)
    y = model["a"](x)
    torch.cuda.synchronize()
    expected = O.gemm_fwd(_np(x), codes.numpy(), scale[:, 0].numpy(), w_kind=O.BF16, v_kind=O.BF16,
                          bias=O.round_kind(state["a.bias"].numpy(), O.BF16))
    assert O.rel_fro(_np(y), expected) <= 5e-3
    # ConvRot storage: the layer equals the dense decoded linear
    xr = torch.randn(3, 41, 1024, device=cuda_device, dtype=torch.bfloat16)
    dense = decode_comfy_state({k: v for k, v in state.items() if k.startswith("b.")}, torch.float32)["b.weight"]
    reference = F.linear(xr.float(), dense.to(cuda_device))
    assert O.rel_fro(_np(model["b"](xr)), _np(reference)) <= 1e-2


def test_requantising_the_dense_decode_moves_codes_and_the_direct_load_does_not(cuda_device):
    """BASELINE-width weight (3072 x 3072): decode to bf16 and quantise again, as a pipeline that
    only decodes must, then compare with the stored codes."""
    codes, scale = comfy_codes(3072, 3072, seed=13)
    marker = comfy_marker({"format": "int8_tensorwise"})
    dense = decode_comfy_state({"w.weight": codes, "w.weight_scale": scale, "w.comfy_quant": marker},
                               torch.bfloat16)["w.weight"]
    linear = nn.Linear(3072, 3072, bias=False, dtype=torch.bfloat16).requires_grad_(False).to(cuda_device)
    with torch.no_grad():
        linear.weight.copy_(dense.to(cuda_device))
    requantized = FrozenInt8Linear(linear)
    direct = FrozenInt8Linear.from_codes(codes.to(cuda_device), scale[:, 0].to(cuda_device), dtype=torch.bfloat16)
    moved = (requantized.weight_int8.cpu() != codes).float().mean().item()
    assert moved > 0.0
    assert torch.equal(direct.weight_int8.cpu(), codes)
    truth = codes.double() * scale.double()
    err_requant = (requantized.weight_int8.cpu().double() * requantized.weight_scale.cpu().double()[:, None] - truth)
    err_direct = direct.weight_int8.cpu().double() * direct.weight_scale.cpu().double()[:, None] - truth
    assert err_direct.abs().max().item() == 0.0 and err_requant.abs().max().item() > 0.0

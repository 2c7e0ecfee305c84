"""GPU tests of the drop-in torch API: FrozenInt8Linear, converters, fused LoRA.

Ports the reference's module tests (training/tests/test_quantization.py:12-85,
training/tests/test_quant_kernels.py:61-129) to CUDA, where this implementation runs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
from torch import nn
from torch.nn import functional as F

from moss_image_b200 import _lib
from moss_image_b200 import quant_kernels as qk
from moss_image_b200.lora import LoRALinear
from moss_image_b200.quantization import FrozenInt8Linear, configure_quantized_backend, quantize_frozen_linears
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


def test_forward_backward_and_saved_storage(cuda_device):
    """test_quantization.py:12-33 on CUDA (bf16 module: the kernels compute in 16-bit)."""
    torch.manual_seed(7)
    base = nn.Linear(64, 32).to(cuda_device, torch.bfloat16).requires_grad_(False)
    with torch.no_grad():
        base.weight[0].zero_()
    quantized = FrozenInt8Linear(base)
    tokens = torch.randn(2, 3, 64, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    reference = tokens.detach().clone().requires_grad_(True)
    saved = []
    with torch.autograd.graph.saved_tensors_hooks(lambda t: saved.append(t) or t, lambda t: t):
        actual = quantized(tokens)
    expected = F.linear(reference.float(), quantized.weight.float(), quantized.bias.float())
    torch.testing.assert_close(actual.float(), expected, atol=2e-2, rtol=2e-2)
    gradient = torch.randn_like(actual)
    actual.backward(gradient)
    expected.backward(gradient.float())
    torch.testing.assert_close(tokens.grad.float(), reference.grad.float(), atol=2e-2, rtol=2e-2)
    assert len(saved) == 2
    assert saved[0].dtype == torch.int8
    assert saved[1].shape == (32,)
    assert not list(quantized.parameters())
    assert quantized.weight_scale[0] == 1.0 and not quantized.weight_int8[0].any()


@pytest.mark.parametrize("name", ["lin_70x37_bf16", "lin_256x320_bf16", "lin_160x96_f16"])
def test_module_matches_reference_eager_goldens(cuda_device, golden_arrays, golden_meta, name):
    """Same codes, same inputs: outputs within the reference's own 2e-2 parity bar and 5e-3 Frobenius."""
    case = golden_meta["cases"][name]
    dtype = getattr(torch, case["dtype"])
    q = torch.from_numpy(golden_arrays[f"{name}.q"])
    in_f, out_f = q.shape[1], q.shape[0]
    lin = nn.Linear(in_f, out_f, bias=case["bias"]).to(cuda_device, dtype).requires_grad_(False)
    module = FrozenInt8Linear(lin)
    with torch.no_grad():
        module.weight_int8.copy_(q)
        module.weight_scale.copy_(torch.from_numpy(golden_arrays[f"{name}.s"]))
        if case["bias"]:
            module.bias.copy_(torch.from_numpy(golden_arrays[f"{name}.bias"]))
    x = torch.from_numpy(golden_arrays[f"{name}.x"]).to(cuda_device, dtype).requires_grad_()
    y = module(x)
    y.backward(torch.from_numpy(golden_arrays[f"{name}.dy"]).to(cuda_device, dtype))
    y_ref = golden_arrays[f"{name}.y"]
    dx_ref = golden_arrays[f"{name}.dx"]
    np.testing.assert_allclose(_np(y), y_ref, atol=2e-2, rtol=2e-2)
    np.testing.assert_allclose(_np(x.grad), dx_ref, atol=2e-2, rtol=2e-2)
    assert O.rel_fro(_np(y), y_ref) < 5e-3
    assert O.rel_fro(_np(x.grad), dx_ref) < 5e-3


@pytest.mark.parametrize("base_dtype", ["bfloat16", "float32"])
def test_bit_exact_decode_and_bias_rounding_kat(cuda_device, golden_arrays, golden_meta, base_dtype):
    """test_quant_kernels.py:85-129: atol = rtol = 0 against the reference eager outputs."""
    name = f"kat_{base_dtype}"
    dtype = getattr(torch, base_dtype)
    lin = nn.Linear(70, 37, bias=True).to(cuda_device, dtype).requires_grad_(False)
    module = FrozenInt8Linear(lin)
    with torch.no_grad():
        module.weight_int8.copy_(torch.from_numpy(golden_arrays[f"{name}.q"]))
        module.weight_scale.copy_(torch.from_numpy(golden_arrays[f"{name}.s"]))
        module.bias.copy_(torch.from_numpy(golden_arrays[f"{name}.bias"]))
    tokens = torch.from_numpy(golden_arrays[f"{name}.x"]).to(cuda_device, dtype).requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16):
        actual = module(tokens)
    grad = torch.from_numpy(golden_arrays[f"{name}.dy"]).to(cuda_device, actual.dtype)
    actual.backward(grad)
    assert actual.dtype == torch.bfloat16
    np.testing.assert_array_equal(_np(actual), golden_arrays[f"{name}.y"])
    assert tokens.grad.dtype == dtype
    np.testing.assert_array_equal(_np(tokens.grad), golden_arrays[f"{name}.dx"])


def test_dtype_moves_and_state_roundtrip(cuda_device):
    base = nn.Linear(16, 8).to(cuda_device).requires_grad_(False)
    quantized = FrozenInt8Linear(base)
    original_scale = quantized.weight_scale.clone()
    quantized.to(dtype=torch.bfloat16)
    assert quantized.compute_dtype == torch.bfloat16
    assert quantized.weight_int8.dtype == torch.int8
    torch.testing.assert_close(quantized.weight_scale, original_scale, rtol=0, atol=0)
    tokens = torch.randn(2, 16, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    quantized(tokens).float().sum().backward()
    assert tokens.grad.dtype == torch.bfloat16
    restored = FrozenInt8Linear(base).to(dtype=torch.bfloat16)
    restored.load_state_dict(quantized.state_dict())
    torch.testing.assert_close(restored(tokens), quantized(tokens), rtol=0, atol=0)
    assert set(quantized.state_dict()) == {"weight_int8", "weight_scale", "bias"}


def test_module_quantises_cpu_weights_identically(cuda_device):
    torch.manual_seed(3)
    base = nn.Linear(40, 24).requires_grad_(False)
    module = FrozenInt8Linear(base)
    assert module.weight_int8.device.type == "cpu"
    q, s, _ = O.quantize(base.weight.detach().numpy())
    np.testing.assert_array_equal(module.weight_int8.numpy(), q)
    np.testing.assert_array_equal(module.weight_scale.numpy().view(np.uint32), s.view(np.uint32))


def test_non_finite_weights_are_rejected(cuda_device):
    base = nn.Linear(8, 4).to(cuda_device).requires_grad_(False)
    with torch.no_grad():
        base.weight[1, 2] = float("inf")
    with pytest.raises(ValueError, match="non-finite"):
        FrozenInt8Linear(base)


def test_weight_accessor_decodes_in_module_dtype(cuda_device):
    base = nn.Linear(70, 37).to(cuda_device, torch.bfloat16).requires_grad_(False)
    module = FrozenInt8Linear(base)
    w = module.weight
    assert w.dtype == torch.bfloat16
    expected = O.dequantize(module.weight_int8.cpu().numpy(), module.weight_scale.cpu().numpy(), O.BF16)
    np.testing.assert_array_equal(_np(w), expected)


def test_converters_and_backend_strings(cuda_device):
    model = nn.Sequential(nn.Linear(16, 8), nn.GELU(), nn.Linear(8, 4)).to(cuda_device, torch.bfloat16)
    model[2].requires_grad_(False)
    assert quantize_frozen_linears(model) == ["2"]
    assert isinstance(model[2], FrozenInt8Linear) and isinstance(model[0], nn.Linear)
    assert configure_quantized_backend(model, "triton") == ["2"]
    for backend in ("auto", "eager", "triton"):
        model[2].set_quantized_backend(backend)
        out = model(torch.randn(3, 16, device=cuda_device, dtype=torch.bfloat16))
        assert out.shape == (3, 4)
    with pytest.raises(ValueError, match="auto, eager or triton"):
        model[2].quantized_backend = "cuda"


def test_float32_compute_dtype_fails_loudly(cuda_device):
    module = FrozenInt8Linear(nn.Linear(16, 8).to(cuda_device).requires_grad_(False))
    with pytest.raises(RuntimeError, match="float32"):
        module(torch.randn(2, 16, device=cuda_device))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        out = module(torch.randn(2, 16, device=cuda_device))
    assert out.dtype == torch.bfloat16


def test_cpu_tensors_fail_loudly():
    module = FrozenInt8Linear(nn.Linear(8, 5).requires_grad_(False), backend="triton")
    with pytest.raises(RuntimeError, match="unavailable.*not on CUDA"):
        module(torch.randn(2, 8, dtype=torch.bfloat16))


def test_fused_lora_matches_reference_composition(cuda_device):
    """LoRALinear over an int8 base: fused single-GEMM path vs the reference composition."""
    torch.manual_seed(5)
    base = nn.Linear(256, 384, bias=True).to(cuda_device, torch.bfloat16).requires_grad_(False)
    fused = LoRALinear(FrozenInt8Linear(base), rank=32, alpha=16).to(cuda_device)
    with torch.no_grad():
        fused.lora_B.normal_(std=0.05)
    ref_A = fused.lora_A.detach().clone().requires_grad_()
    ref_B = fused.lora_B.detach().clone().requires_grad_()
    x = torch.randn(3, 70, 256, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    xr = x.detach().clone().requires_grad_()
    g = torch.randn(3, 70, 384, device=cuda_device, dtype=torch.bfloat16)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = fused(x)
        # reference composition (training/lora.py:70-86) with the same int8 base
        result = fused.base(xr)
        update = F.linear(F.linear(xr.to(torch.bfloat16), ref_A.to(torch.bfloat16)), ref_B.to(torch.bfloat16))
        y_ref = result + update.to(result.dtype) * fused.scale
    y.backward(g)
    y_ref.backward(g)
    assert O.rel_fro(_np(y), _np(y_ref)) < 5e-3
    assert O.rel_fro(_np(x.grad), _np(xr.grad)) < 5e-3
    assert O.rel_fro(_np(fused.lora_A.grad), _np(ref_A.grad)) < 2e-2
    assert O.rel_fro(_np(fused.lora_B.grad), _np(ref_B.grad)) < 2e-2
    assert fused.lora_A.grad.dtype == torch.float32
    torch.cuda.synchronize()
    assert qk.check_device_status(cuda_device) & _lib.STATUS_TIMEOUT_MASK == 0

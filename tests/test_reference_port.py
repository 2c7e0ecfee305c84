"""The reference's own module tests, run against this drop-in.

Ports training/tests/test_quant_kernels.py:16-153 and training/tests/test_quantization.py:
12-85. Each test keeps the reference's construction, inputs, assertions and tolerances; the
"expected" side that the reference computes with its eager backend is computed here with the
reference's eager formula written out in torch (dequantise with
``q.to(dtype) * scale.to(dtype)[:, None]``, then ``F.linear`` / ``matmul``,
training/quantization.py:23-24,43,61-64), because every backend string of this library runs
the sm_100a kernels.

The deliberate differences are tested as such (the module raises the reference's
"Triton quantized backend is unavailable" RuntimeError instead of computing):

* CPU tensors, for every backend string (the reference runs ``auto``/``eager`` eagerly on
  CPU, test_quant_kernels.py:16-33);
* a float32 compute dtype outside autocast (the reference's fp32 eager/Triton path,
  test_quantization.py:12-33 and :66-77 run in fp32 on CPU). Those tests run here in bf16
  on CUDA, the precision the trainer uses, with the reference's tolerances.

The ConvRot workspace bound is this library's own (test_convrot_workspace_is_bounded_...).
"""

from __future__ import annotations

import pytest
import torch
from torch import nn
from torch.nn import functional as F

from moss_image_b200.convrot import FrozenConvRotLinear, rotate_hadamard
from moss_image_b200.lora import LoRALinear
from moss_image_b200.quant_kernels import convrot_workspace_bound_bytes
from moss_image_b200.quantization import FrozenInt8Linear, configure_quantized_backend, quantize_frozen_linears

gpu = pytest.mark.gpu


def _eager_dequantize(module: FrozenInt8Linear, dtype: torch.dtype) -> torch.Tensor:
    """training/quantization.py:23-24."""
    return module.weight_int8.to(dtype) * module.weight_scale.to(dtype)[:, None]


# ------------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("backend", ["triton", "auto", "eager"])
def test_explicit_triton_fails_clearly_on_cpu(backend):
    """test_quant_kernels.py:46-49 (``triton``); ``auto``/``eager`` raise too (no CPU path)."""
    codes = torch.randint(-127, 128, (5, 8), dtype=torch.int8)
    module = FrozenInt8Linear.from_codes(codes, torch.full((5,), 0.01), dtype=torch.float32, backend=backend)
    with pytest.raises(RuntimeError, match="Triton quantized backend is unavailable.*not on CUDA"):
        module(torch.randn(2, 8))


def test_convrot_workspace_is_bounded_independently_of_token_count():
    """test_quant_kernels.py:52-56, with this library's bound.

    Deliberate difference: the reference rotates chunks of 256 Ki elements through two stage
    buffers (2 x 256 Ki elements); here one rotated chunk of up to 32 Mi elements exists (the
    rotation runs on chip, so there is no second buffer). A 256 Ki-element chunk is 85 rows at
    width 3072: every chunk would re-stream the whole int8 weight through the GEMM.
    """
    expected = 32 * 1024 * 1024 * torch.empty((), dtype=torch.bfloat16).element_size()
    assert convrot_workspace_bound_bytes(64, torch.bfloat16) == expected
    assert convrot_workspace_bound_bytes(4096, torch.bfloat16) == expected
    assert convrot_workspace_bound_bytes(3072, torch.bfloat16) <= expected


def test_trainable_base_is_rejected_and_skipped():
    """test_quantization.py:59-63."""
    with pytest.raises(ValueError, match="Freeze"):
        FrozenInt8Linear(nn.Linear(4, 4))
    model = nn.Sequential(nn.Linear(4, 4))
    assert quantize_frozen_linears(model) == []


# ------------------------------------------------------------------------------- GPU
@gpu
def test_backend_selection_is_explicit_and_auto_preserves_eager_results(cuda_device):
    """test_quant_kernels.py:16-33 on CUDA in bf16: ``auto`` and ``eager`` give identical results."""
    torch.manual_seed(12)
    base = nn.Linear(11, 7).to(cuda_device, torch.bfloat16).requires_grad_(False)
    eager = FrozenInt8Linear(base)
    automatic = FrozenInt8Linear(base, backend="auto")
    automatic.load_state_dict(eager.state_dict())
    assert eager.quantized_backend == "eager"
    assert automatic.quantized_backend == "auto"
    tokens = torch.randn(2, 3, 11, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    reference = tokens.detach().clone().requires_grad_(True)
    output = automatic(tokens)
    expected = eager(reference)
    gradient = torch.randn_like(output)
    output.backward(gradient)
    expected.backward(gradient)
    torch.testing.assert_close(output, expected)
    torch.testing.assert_close(tokens.grad, reference.grad)


@gpu
def test_module_backend_configuration_and_validation(cuda_device):
    """test_quant_kernels.py:36-43."""
    model = nn.Sequential(
        FrozenInt8Linear(nn.Linear(8, 5).to(cuda_device).requires_grad_(False)),
        FrozenConvRotLinear(nn.Linear(5, 3).to(cuda_device).requires_grad_(False), group_size=4),
    )
    assert configure_quantized_backend(model, "auto") == ["0", "1"]
    assert all(layer.quantized_backend == "auto" for layer in model)
    model[0].set_quantized_backend("eager")
    assert model[0].quantized_backend == "eager"
    with pytest.raises(ValueError, match="auto, eager or triton"):
        model[0].quantized_backend = "cuda"


@gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_int8_uneven_output_and_input_gradient_parity(cuda_device, dtype):
    """test_quant_kernels.py:61-82: 70 -> 37, tokens [2, 3, 70], 2e-2 against eager."""
    torch.manual_seed(73)
    base = nn.Linear(70, 37, device=cuda_device, dtype=dtype).requires_grad_(False)
    fused = FrozenInt8Linear(base, backend="triton")
    tokens = torch.randn(2, 3, 70, device=cuda_device, dtype=dtype, requires_grad=True)
    reference = tokens.detach().clone().requires_grad_(True)
    actual = fused(tokens)
    expected = F.linear(reference, _eager_dequantize(fused, dtype), fused.bias)
    gradient = torch.randn_like(actual)
    actual.backward(gradient)
    expected.backward(gradient)
    torch.testing.assert_close(actual, expected, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(tokens.grad, reference.grad, atol=2e-2, rtol=2e-2)


@gpu
@pytest.mark.parametrize("base_dtype", [torch.bfloat16, torch.float32])
def test_bf16_autocast_preserves_eager_decode_rounding(cuda_device, base_dtype):
    """test_quant_kernels.py:85-129, bit-exact (atol = rtol = 0) against the eager formula."""
    base = nn.Linear(70, 37, bias=True, device=cuda_device, dtype=base_dtype).requires_grad_(False)
    fused = FrozenInt8Linear(base, backend="triton")
    scale = 0.0002928110350837356  # separates BF16(scale) * BF16(q) from BF16(FP32(scale * q))
    with torch.no_grad():
        fused.weight_int8.zero_()
        fused.weight_int8[0, 0] = 83
        fused.weight_int8[1, 1] = -83
        fused.weight_scale.fill_(scale)
        fused.weight_int8[2:6, 2] = 1
        fused.weight_scale[2:6] = 1
        fused.bias.zero_()
        fused.bias[0] = 0.08285745223138713  # FP32 and BF16 bias land on opposite sides of a rounding boundary
    tokens = torch.zeros(1, 70, device=cuda_device, dtype=base_dtype, requires_grad=True)
    with torch.no_grad():
        tokens[0, :2] = 1
    reference = tokens.detach().clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        actual = fused(tokens)
        expected = F.linear(reference.to(base_dtype), _eager_dequantize(fused, base_dtype), fused.bias)
    gradient = torch.zeros_like(actual)
    gradient[0, :2] = 1
    # these four BF16 terms sum to a non-BF16 value: fp32 inputs must get eager's BF16 output rounding
    gradient[0, 2:6] = torch.tensor([-0.1962890625, -2.265625, -0.52734375, 1.546875], device=cuda_device,
                                    dtype=torch.bfloat16)
    actual.backward(gradient)
    with torch.autocast("cuda", enabled=False):
        # the eager backward, training/quantization.py:61-64
        grad_expected = gradient.to(expected.dtype).matmul(
            _eager_dequantize(fused, base_dtype).to(expected.dtype)).to(reference.dtype)
    assert actual.dtype == expected.dtype == torch.bfloat16
    torch.testing.assert_close(actual, expected, atol=0, rtol=0)
    torch.testing.assert_close(tokens.grad, grad_expected, atol=0, rtol=0)


@gpu
@pytest.mark.parametrize("group_size", [1, 2, 4, 8, 16, 64, 256])
def test_convrot_bf16_uneven_output_and_input_gradient_parity(cuda_device, group_size):
    """test_quant_kernels.py:132-153: 256 -> 37 ConvRot, 3e-2 against the eager rotation + linear."""
    torch.manual_seed(91 + group_size)
    base = nn.Linear(256, 37, device=cuda_device, dtype=torch.bfloat16).requires_grad_(False)
    fused = FrozenConvRotLinear(base, group_size=group_size, backend="triton")
    tokens = torch.randn(2, 3, 256, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    reference = tokens.detach().clone().requires_grad_(True)
    actual = fused(tokens)
    rotated = rotate_hadamard(reference, fused.group_size)
    expected = F.linear(rotated, _eager_dequantize(fused, torch.bfloat16), fused.bias)
    gradient = torch.randn_like(actual)
    actual.backward(gradient)
    expected.backward(gradient)
    torch.testing.assert_close(actual, expected, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(tokens.grad, reference.grad, atol=3e-2, rtol=3e-2)


@gpu
def test_conversion_preserves_adapters_and_gradients(cuda_device):
    """test_quantization.py:36-48 on CUDA (bf16 base, fp32 adapter masters as in the reference)."""
    base = nn.Linear(16, 8).to(cuda_device, torch.bfloat16).requires_grad_(False)
    model = nn.Sequential(LoRALinear(base, rank=3, alpha=3)).to(cuda_device)
    model[0].lora_B.data.normal_()
    adapter_ids = [id(model[0].lora_A), id(model[0].lora_B)]
    assert quantize_frozen_linears(model) == ["0.base"]
    assert isinstance(model[0].base, FrozenInt8Linear)
    assert [id(model[0].lora_A), id(model[0].lora_B)] == adapter_ids
    assert model[0].lora_A.dtype == torch.float32
    tokens = torch.randn(2, 16, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        model(tokens).float().square().mean().backward()
    assert tokens.grad is not None and torch.isfinite(tokens.grad).all()
    assert model[0].lora_A.grad is not None and model[0].lora_B.grad is not None


@gpu
def test_autocast_input_backward_matches_float_linear(cuda_device):
    """test_quantization.py:66-77 with CUDA autocast (bf16 outputs, fp32 input gradient)."""
    quantized = FrozenInt8Linear(nn.Linear(16, 8).to(cuda_device).requires_grad_(False))
    tokens = torch.randn(2, 16, device=cuda_device, requires_grad=True)
    reference = tokens.detach().clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        actual = quantized(tokens)
        expected = F.linear(reference, quantized.weight, quantized.bias)
    gradient = torch.randn_like(actual)
    actual.backward(gradient)
    expected.backward(gradient)
    torch.testing.assert_close(actual, expected)
    torch.testing.assert_close(tokens.grad, reference.grad)


@gpu
def test_float32_compute_outside_autocast_is_refused(cuda_device):
    """Deliberate difference: the reference computes an fp32 module in fp32 outside autocast."""
    quantized = FrozenInt8Linear(nn.Linear(16, 8).to(cuda_device).requires_grad_(False))
    with pytest.raises(RuntimeError, match="Triton quantized backend is unavailable.*float32"):
        quantized(torch.randn(2, 16, device=cuda_device))

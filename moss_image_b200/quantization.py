"""Frozen int8 weight storage for adapter training, executed by the sm_100a kernels.

Drop-in for ``training/quantization.py``: same class and function names, constructor
arguments, state-dict keys (``weight_int8`` int8 ``[out, in]``, ``weight_scale`` f32
``[out]``, ``bias``), non-persistent ``_dtype_anchor``, properties and error messages.
The quantiser, the forward GEMM and the input-gradient GEMM run in ``libmoss_w8.so``.
Neither direction materialises a floating-point copy of the weight.
"""

from __future__ import annotations

import torch
from torch import nn

from .quant_kernels import (
    autocast_compute_dtype,
    dequantize_weight,
    int8_linear_backward,
    int8_linear_forward,
    quantize_weight,
    resolve_quantized_backend,
    validate_quantized_backend,
)


def _dequantize(weight: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Decoded weight ``round_d(q * round_d(s))`` (reference training/quantization.py:23-24)."""
    return dequantize_weight(weight, scale, dtype)


class _FrozenInt8Linear(torch.autograd.Function):
    """Forward ``Y = X dec(W)^T + b``; backward returns only the input gradient.

    Reference: training/quantization.py:27-65. Only ``(weight, scale)`` are saved, so the
    activation offload never sees the input of a frozen linear.
    """

    @staticmethod
    def forward(ctx, tokens, weight, scale, bias, dtype, backend):
        ctx.save_for_backward(weight, scale)
        ctx.input_dtype = tokens.dtype
        ctx.weight_dtype = dtype
        ctx.backend = resolve_quantized_backend(backend, tokens, weight, scale)
        ctx.input_shape = tokens.shape
        output_dtype = autocast_compute_dtype(tokens, dtype)
        result = int8_linear_forward(tokens, weight, scale, bias, output_dtype, dtype)
        ctx.compute_dtype = result.dtype
        return result

    @staticmethod
    def backward(ctx, gradient):
        weight, scale = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            return None, None, None, None, None, None
        grad_input = int8_linear_backward(
            gradient,
            weight,
            scale,
            ctx.input_shape,
            ctx.input_dtype,
            ctx.weight_dtype,
            compute_dtype=ctx.compute_dtype,
        )
        return grad_input, None, None, None, None, None


class FrozenInt8Linear(nn.Module):
    """Per-output-channel symmetric int8 linear with gradients only to its input.

    Reference: training/quantization.py:68-131. ``weight`` is a compatibility accessor that
    allocates a transient decoded tensor; call the module for computation.
    """

    # The module multiplies its input by dec(weight_int8)^T unchanged, so an adapter's
    # update can share its GEMM (subclasses that transform the input set this to False).
    fuses_lora = True

    def __init__(self, linear: nn.Linear, *, backend: str = "eager") -> None:
        super().__init__()
        if linear.weight.requires_grad or (linear.bias is not None and linear.bias.requires_grad):
            raise ValueError("Freeze the base linear before quantizing it (LoRA training only).")
        if linear.weight.device.type == "meta":
            raise ValueError("Load the base weights before quantizing them.")
        self.in_features = linear.in_features
        self.out_features = linear.out_features
        self._quantized_backend = validate_quantized_backend(backend)
        codes, scale = quantize_weight(linear.weight.detach())
        self.register_buffer("weight_int8", codes)
        self.register_buffer("weight_scale", scale)
        self.register_buffer(
            "_dtype_anchor", torch.empty(0, device=linear.weight.device, dtype=linear.weight.dtype), persistent=False
        )
        self.register_buffer("bias", None if linear.bias is None else linear.bias.detach().clone())

    @property
    def compute_dtype(self) -> torch.dtype:
        return self._dtype_anchor.dtype

    @property
    def quantized_backend(self) -> str:
        return self._quantized_backend

    @quantized_backend.setter
    def quantized_backend(self, backend: str) -> None:
        self._quantized_backend = validate_quantized_backend(backend)

    def set_quantized_backend(self, backend: str) -> "FrozenInt8Linear":
        """Select execution for this module and return it for fluent setup."""
        self.quantized_backend = backend
        return self

    @property
    def weight(self) -> torch.Tensor:
        return _dequantize(self.weight_int8, self.weight_scale, self.compute_dtype)

    def _apply(self, fn, recurse=True):
        # Keep scales at fp32 even when model.to(dtype=...) casts other floats.
        scale = self.weight_scale
        result = super()._apply(fn, recurse=recurse)
        self.weight_scale = scale.to(device=self.weight_int8.device, dtype=torch.float32)
        return result

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        return _FrozenInt8Linear.apply(
            tokens,
            self.weight_int8,
            self.weight_scale,
            self.bias,
            self.compute_dtype,
            self.quantized_backend,
        )

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


def configure_quantized_backend(model: nn.Module, backend: str) -> list[str]:
    """Set the backend on every frozen INT8 module and return their paths.

    Reference: training/quantization.py:134-142.
    """
    selected = validate_quantized_backend(backend)
    names = []
    for name, child in model.named_modules():
        if isinstance(child, FrozenInt8Linear):
            child.quantized_backend = selected
            names.append(name)
    return names


def quantize_frozen_linears(model: nn.Module, *, backend: str = "eager") -> list[str]:
    """Replace frozen Linear children, including bases inside existing LoRA wrappers.

    Reference: training/quantization.py:145-162. Trainable linears are left alone.
    Returns the replaced module paths.
    """
    validate_quantized_backend(backend)
    names = []
    for name, child in list(model.named_modules()):
        if not name or not isinstance(child, nn.Linear):
            continue
        if any(parameter.requires_grad for parameter in child.parameters()):
            continue
        parent_name, _, leaf = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, leaf, FrozenInt8Linear(child, backend=backend))
        names.append(name)
    return names

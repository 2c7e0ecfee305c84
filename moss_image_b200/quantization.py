"""Frozen int8 weight storage for adapter training, executed by the sm_100a kernels.

Drop-in for ``training/quantization.py``: same class and function names, constructor
arguments, state-dict keys (``weight_int8`` int8 ``[out, in]``, ``weight_scale`` f32
``[out]``, ``bias``), non-persistent ``_dtype_anchor``, properties and error messages.
The quantiser, the forward GEMM and the input-gradient GEMM run in ``libmoss_w8.so``.
Neither direction materialises a floating-point copy of the weight.
"""

from __future__ import annotations

from typing import Callable

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
        validate_quantized_backend(backend)
        codes, scale = quantize_weight(linear.weight.detach())
        bias = None if linear.bias is None else linear.bias.detach().clone()
        self._set_codes(codes, scale, bias, linear.weight.dtype, backend)

    @classmethod
    def from_codes(cls, codes: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None, *,
                   dtype: torch.dtype = torch.bfloat16, backend: str = "eager") -> "FrozenInt8Linear":
        """Wrap stored codes (int8 ``[out, in]``) and per-row float32 scales (``[out]``) as they
        are - e.g. a quantised checkpoint's - without decoding or re-quantising them.

        ``dtype`` is the compute dtype (what ``.to(dtype)`` would have set).
        """
        if codes.dtype != torch.int8 or codes.ndim != 2:
            raise ValueError("int8 codes must be an int8 [out, in] tensor.")
        if scale.dtype != torch.float32 or tuple(scale.shape) != (codes.shape[0],):
            raise ValueError("weight scales must be float32 [out].")
        if scale.device != codes.device or (bias is not None and bias.device != codes.device):
            raise ValueError("codes, scales and bias must be on one device.")
        if bias is not None and tuple(bias.shape) != (codes.shape[0],):
            raise ValueError("bias must be [out].")
        module = cls.__new__(cls)
        nn.Module.__init__(module)
        module._set_codes(codes.contiguous(), scale.contiguous(), bias, dtype, validate_quantized_backend(backend))
        return module

    def _set_codes(self, codes: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None, dtype: torch.dtype,
                   backend: str) -> None:
        self.in_features = codes.shape[1]
        self.out_features = codes.shape[0]
        self._quantized_backend = backend
        self.register_buffer("weight_int8", codes)
        self.register_buffer("weight_scale", scale)
        self.register_buffer("_dtype_anchor", torch.empty(0, device=codes.device, dtype=dtype), persistent=False)
        self.register_buffer("bias", bias)

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


def replace_frozen_linears(model: nn.Module, make: Callable[[nn.Linear], nn.Module]) -> list[str]:
    """Swap every frozen ``nn.Linear`` below ``model`` (including bases inside LoRA wrappers)
    for ``make(linear)``; trainable linears are left alone. Returns the replaced paths.

    The module walk shared by ``quantize_frozen_linears`` and
    ``convrot.quantize_frozen_convrot_linears`` (reference training/quantization.py:152-162 and
    training/convrot.py:163-172 walk the same way).
    """
    names = []
    for name, child in list(model.named_modules()):
        if not name or not isinstance(child, nn.Linear):
            continue
        if any(parameter.requires_grad for parameter in child.parameters()):
            continue
        parent_name, _, leaf = name.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, leaf, make(child))
        names.append(name)
    return names


def quantize_frozen_linears(model: nn.Module, *, backend: str = "eager") -> list[str]:
    """Replace frozen Linear children, including bases inside existing LoRA wrappers.

    Reference: training/quantization.py:145-162. Trainable linears are left alone.
    Returns the replaced module paths.
    """
    validate_quantized_backend(backend)
    return replace_frozen_linears(model, lambda linear: FrozenInt8Linear(linear, backend=backend))

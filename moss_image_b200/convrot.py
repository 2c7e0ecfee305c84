"""Frozen int8 weights in a grouped, normalised Hadamard basis (weight-only ConvRot).

Drop-in for ``training/convrot.py``: same names, constructor arguments, state-dict keys
(``weight_int8``, ``weight_scale``, ``bias``, ``rotation_group_size``), properties and error
messages. The layer stores int8(W H) and computes (x H) dec(W H)^T; H is block-diagonal with
``group_size`` blocks built from the regular H4 (plus one H2 factor for odd log2(group)),
symmetric and orthonormal, so the input gradient is H (dY dec(W H)).

On CUDA the activation and gradient rotations run in ``moss_hadamard_rotate`` (one on-chip
pass with the reference's per-stage rounding) around the sm_100a int8 GEMMs.
"""

from __future__ import annotations

import math

import torch
from torch import nn

from .quant_kernels import (
    autocast_compute_dtype,
    convrot_backward,
    convrot_forward,
    hadamard_transform,
    validate_quantized_backend,
)
from .quantization import FrozenInt8Linear, replace_frozen_linears


def effective_group_size(in_features: int, group_size: int = 256) -> int:
    """Largest power of two not above ``group_size`` that divides the input width.

    Reference: training/convrot.py:24-33.
    """
    if isinstance(group_size, bool) or not isinstance(group_size, int) or group_size < 1:
        raise ValueError("ConvRot group_size must be a positive integer.")
    if in_features < 1:
        raise ValueError("ConvRot input width must be positive.")
    group = 1 << (group_size.bit_length() - 1)
    while in_features % group:
        group //= 2
    return group


def rotate_hadamard(tokens: torch.Tensor, group_size: int) -> torch.Tensor:
    """Rotate groups of the last dimension by the normalised grouped Hadamard matrix.

    Reference: training/convrot.py:36-63 (eager torch arithmetic in the input dtype, the same
    expressions in the same order, so weights rotated here quantise to the same codes).
    """
    if group_size < 1 or group_size & (group_size - 1):
        raise ValueError("Hadamard group size must be a positive power of two.")
    if tokens.shape[-1] % group_size:
        raise ValueError("Input width must be divisible by Hadamard group size.")
    if group_size == 1:
        return tokens
    shape = tokens.shape
    value = tokens.reshape(-1, group_size)
    stride = 1
    while stride * 4 <= group_size:
        a, b, c, d = value.reshape(-1, group_size // (4 * stride), 4, stride).unbind(dim=-2)
        stacked = torch.stack((a + b + c - d, a + b - c + d, a - b + c + d, -a + b + c + d), dim=-2)
        value = stacked.reshape(-1, group_size) * 0.5
        stride *= 4
    if stride < group_size:
        a, b = value.reshape(-1, 2, stride).unbind(dim=-2)
        value = torch.stack((a + b, a - b), dim=-2).reshape(-1, group_size) / math.sqrt(2)
    return value.reshape(shape)


class _FrozenConvRot(torch.autograd.Function):
    """Forward ``(x H) dec(W H)^T + b``; backward returns only ``H (dY dec(W H))``.

    Reference: training/convrot.py:66-93. Only ``(weight, scale)`` are saved.
    """

    @staticmethod
    def forward(ctx, tokens, weight, scale, bias, dtype, group_size):
        output_dtype = autocast_compute_dtype(tokens, dtype)
        result = convrot_forward(tokens, weight, scale, bias, output_dtype, dtype, group_size)
        ctx.save_for_backward(weight, scale)
        ctx.input_shape = tokens.shape
        ctx.input_dtype = tokens.dtype
        ctx.weight_dtype = dtype
        ctx.group_size = group_size
        return result

    @staticmethod
    def backward(ctx, gradient):
        weight, scale = ctx.saved_tensors
        if not ctx.needs_input_grad[0]:
            return None, None, None, None, None, None
        grad_input = convrot_backward(gradient, weight, scale, ctx.input_shape, ctx.input_dtype, ctx.weight_dtype,
                                      ctx.group_size)
        return grad_input, None, None, None, None, None


class FrozenConvRotLinear(FrozenInt8Linear):
    """Quantise W H and compute (x H)(W H)^T, with frozen base weights.

    Reference: training/convrot.py:96-150.
    """

    # the GEMM sees x H, not x: an adapter's update is added after the rotated product
    fuses_lora = False

    def __init__(self, linear: nn.Linear, group_size: int = 256, *, backend: str = "eager") -> None:
        if any(parameter.requires_grad for parameter in linear.parameters()):
            raise ValueError("Freeze the base linear before ConvRot quantization (LoRA only).")
        if linear.weight.device.type == "meta":
            raise ValueError("Load the base weights before ConvRot quantization.")
        group = effective_group_size(linear.in_features, group_size)
        rotated = nn.Linear(linear.in_features, linear.out_features, bias=linear.bias is not None,
                            device="meta", dtype=torch.float32)
        rotated.weight = nn.Parameter(rotate_hadamard(linear.weight.detach().float(), group), requires_grad=False)
        if linear.bias is not None:
            rotated.bias = nn.Parameter(linear.bias.detach().clone(), requires_grad=False)
        super().__init__(rotated, backend=backend)
        self._dtype_anchor = torch.empty(0, device=linear.weight.device, dtype=linear.weight.dtype)
        self.group_size = group
        self.register_buffer("rotation_group_size", torch.tensor(group, device=linear.weight.device))

    @classmethod
    def from_codes(cls, codes: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None = None,
                   group_size: int = 256, *, dtype: torch.dtype = torch.bfloat16,
                   backend: str = "eager") -> "FrozenConvRotLinear":
        """Wrap stored codes of ``W H`` (int8 ``[out, in]``, per-row float32 scales ``[out]``)
        rotated with ``group_size``, without decoding or re-quantising them."""
        if effective_group_size(codes.shape[1], group_size) != group_size:
            raise ValueError("ConvRot group size must be a power of two that divides the input width.")
        module = super().from_codes(codes, scale, bias, dtype=dtype, backend=backend)
        module.group_size = group_size
        module.register_buffer("rotation_group_size", torch.tensor(group_size, device=codes.device))
        return module

    @property
    def weight(self) -> torch.Tensor:
        """Transient decoded weight in the original, unrotated basis."""
        decoded = super().weight
        if self.group_size == 1:
            return decoded
        return hadamard_transform(decoded.contiguous(), self.group_size)

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        return _FrozenConvRot.apply(tokens, self.weight_int8, self.weight_scale, self.bias, self.compute_dtype,
                                    self.group_size)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        stored_group = state_dict.get(prefix + "rotation_group_size")
        if stored_group is not None and int(stored_group.item()) != self.group_size:
            error_msgs.append(f"{prefix}ConvRot group size differs from the checkpoint; "
                              "construct the module with the checkpoint's group size.")
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)

    def extra_repr(self) -> str:
        return f"{super().extra_repr()}, group_size={self.group_size}"


def quantize_frozen_convrot_linears(model: nn.Module, group_size: int = 256, *, backend: str = "eager") -> list[str]:
    """Replace frozen Linear children (after LoRA injection; adapters stay intact).

    Reference: training/convrot.py:153-172. Returns the replaced module paths.
    """
    effective_group_size(1, group_size)  # validate even when nothing is replaced
    validate_quantized_backend(backend)
    return replace_frozen_linears(model, lambda linear: FrozenConvRotLinear(linear, group_size, backend=backend))

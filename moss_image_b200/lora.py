"""LoRA adapters whose update is fused into the int8 GEMM accumulator.

``LoRALinear`` keeps the reference module's interface (training/lora.py:21-86): same
constructor, parameters ``lora_A [rank, in]`` (Kaiming-uniform) and ``lora_B [out, rank]``
(zeros), ``scale = alpha / rank``, ``lora_compute_dtype``, and ``compute_dtype``/``weight``/
``bias`` accessors. When the frozen base is a :class:`FrozenInt8Linear` and the adapter math
runs in the same 16-bit dtype as the base output (autocast, or an explicit
``lora_compute_dtype``), the forward is one kernel launch:

    y = x dec(W)^T + b + (x A^T) (scale * B)^T          (rank-r block appended to K)

and the input gradient is likewise one launch,

    dx = dy dec(W) + (dy B) (scale * A)                  (rank-r block appended to N)

with the two small rank-r products (``x A^T`` and ``dy B``) and the adapter weight
gradients done as plain library GEMMs. The reference adds the update after rounding the
base output and the update separately (``result + update.to(result.dtype) * scale``); the
fused form rounds once, which stays within the 5e-3 relative-Frobenius bar.

Other cases (fp32 adapter math, non-int8 bases) run the reference composition.
"""

from __future__ import annotations

import math

import torch
from torch import nn
from torch.nn import functional as F

from .quant_kernels import autocast_compute_dtype, int8_linear_backward, int8_linear_forward, resolve_quantized_backend
from .quantization import FrozenInt8Linear


class _FusedLoRAInt8Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, lora_a, lora_b, weight, scale, bias, weight_dtype, backend, lora_scale, compute_dtype):
        resolve_quantized_backend(backend, tokens, weight, scale)
        x = tokens.to(compute_dtype)
        a = lora_a.to(compute_dtype)
        xa = F.linear(x, a)  # [.., r] plain library GEMM (rank r)
        y = int8_linear_forward(x, weight, scale, bias, compute_dtype, weight_dtype, lora_xa=xa, lora_b=lora_b,
                                lora_scale=lora_scale)
        ctx.save_for_backward(x, xa, lora_a, lora_b, weight, scale)
        ctx.input_dtype = tokens.dtype
        ctx.input_shape = tokens.shape
        ctx.weight_dtype = weight_dtype
        ctx.lora_scale = lora_scale
        ctx.compute_dtype = compute_dtype
        return y

    @staticmethod
    def backward(ctx, gradient):
        x, xa, lora_a, lora_b, weight, scale = ctx.saved_tensors
        cd = ctx.compute_dtype
        g = gradient.to(cd)
        g2 = g.reshape(-1, g.shape[-1])
        b = lora_b.to(cd)
        dyb = g2 @ b  # [M, r]
        grad_input = None
        if ctx.needs_input_grad[0]:
            grad_input = int8_linear_backward(g, weight, scale, ctx.input_shape, ctx.input_dtype, ctx.weight_dtype,
                                              compute_dtype=cd, lora_dyb=dyb, lora_a=lora_a,
                                              lora_scale=ctx.lora_scale)
        grad_a = grad_b = None
        s = ctx.lora_scale
        if ctx.needs_input_grad[1]:
            x2 = x.reshape(-1, x.shape[-1])
            grad_a = (dyb.t() @ x2).to(lora_a.dtype).mul_(s)
        if ctx.needs_input_grad[2]:
            xa2 = xa.reshape(-1, xa.shape[-1])
            grad_b = (g2.t() @ xa2).to(lora_b.dtype).mul_(s)
        return grad_input, grad_a, grad_b, None, None, None, None, None, None, None


class LoRALinear(nn.Module):
    """A frozen linear plus a low-rank residual (reference: training/lora.py:21-86)."""

    def __init__(self, base: nn.Module, rank: int, alpha: float) -> None:
        super().__init__()
        if rank < 1:
            raise ValueError("LoRA rank must be positive.")
        self.base = base
        self.rank = rank
        self.alpha = float(alpha)
        self.scale = self.alpha / rank
        in_features = base.in_features
        out_features = base.out_features
        self.lora_A = nn.Parameter(torch.empty(rank, in_features))
        self.lora_B = nn.Parameter(torch.zeros(out_features, rank))
        self.lora_compute_dtype: torch.dtype | None = None
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        for parameter in self.base.parameters():
            parameter.requires_grad_(False)

    @property
    def compute_dtype(self) -> torch.dtype:
        if hasattr(self.base, "compute_dtype"):
            return self.base.compute_dtype
        return self.base.weight.dtype

    @property
    def weight(self) -> torch.Tensor:
        return self.base.weight

    @property
    def bias(self) -> torch.Tensor | None:
        return self.base.bias

    def _adapter_dtype(self, tokens: torch.Tensor) -> torch.dtype | None:
        compute_dtype = self.lora_compute_dtype
        if compute_dtype is None and torch.is_autocast_enabled(tokens.device.type):
            compute_dtype = torch.get_autocast_dtype(tokens.device.type)
        return compute_dtype

    def forward(self, tokens: torch.Tensor) -> torch.Tensor:
        adapter_dtype = self._adapter_dtype(tokens)
        base = self.base
        if (
            isinstance(base, FrozenInt8Linear)
            and base.fuses_lora
            and tokens.device.type == "cuda"
            and adapter_dtype in (torch.float16, torch.bfloat16)
            and autocast_compute_dtype(tokens, base.compute_dtype) == adapter_dtype
        ):
            return _FusedLoRAInt8Linear.apply(
                tokens, self.lora_A, self.lora_B, base.weight_int8, base.weight_scale, base.bias,
                base.compute_dtype, base.quantized_backend, float(self.scale), adapter_dtype,
            )
        # Reference composition (training/lora.py:70-86).
        result = base(tokens)
        if adapter_dtype is None:
            adapter_input = tokens.to(self.lora_A.dtype)
            adapter_a, adapter_b = self.lora_A, self.lora_B
        else:
            adapter_input = tokens.to(adapter_dtype)
            adapter_a, adapter_b = self.lora_A.to(adapter_dtype), self.lora_B.to(adapter_dtype)
        update = F.linear(F.linear(adapter_input, adapter_a), adapter_b)
        return result + update.to(result.dtype) * self.scale

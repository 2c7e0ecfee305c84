"""RMSNorm of the DiT block on the native kernels (``moss_rmsnorm_fwd``/``moss_rmsnorm_bwd``).

Same arithmetic as the reference module (training/model.py:154-172): statistics in f32,
``n = (x * rsqrt(mean(x^2) + eps)).to(x.dtype)``, then ``n * weight`` in torch's promoted
dtype. The kernels keep a row in registers between the two passes and pack several short
rows (the per-head q/k norms) into one warp, so both directions run near the copy bandwidth;
the backward reuses the per-row rsqrt saved by the forward. The sum of squares is reduced in a
different order than torch's, so outputs may differ from the eager module by one rounding of
the result dtype. CUDA tensors only: there is no CPU path.
"""

from __future__ import annotations

import torch

from . import _lib


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, weight, eps):
        rows = tokens.reshape(-1, tokens.shape[-1])
        out_dtype = torch.promote_types(tokens.dtype, weight.dtype)
        out = torch.empty(rows.shape, dtype=out_dtype, device=tokens.device)
        rstd = torch.empty(rows.shape[0], dtype=torch.float32, device=tokens.device)
        _lib.check(_lib.library().moss_rmsnorm_fwd(
            rows.data_ptr(), _lib.dtype_code(rows.dtype), rows.shape[0], rows.shape[1], weight.data_ptr(),
            _lib.dtype_code(weight.dtype), float(eps), out.data_ptr(), rstd.data_ptr(),
            _lib.stream_handle(tokens.device)), "moss_rmsnorm_fwd")
        _lib.count_launch("rmsnorm")
        ctx.save_for_backward(rows, weight, rstd)
        ctx.shape = tokens.shape
        return out.view(ctx.shape)

    @staticmethod
    def backward(ctx, grad):
        rows, weight, rstd = ctx.saved_tensors
        out_dtype = torch.promote_types(rows.dtype, weight.dtype)
        grad = grad.reshape(rows.shape).to(out_dtype).contiguous()
        d_tokens = None
        if ctx.needs_input_grad[0]:
            d_rows = torch.empty_like(rows)
            _lib.check(_lib.library().moss_rmsnorm_bwd(
                grad.data_ptr(), rows.data_ptr(), _lib.dtype_code(rows.dtype), rows.shape[0], rows.shape[1],
                weight.data_ptr(), _lib.dtype_code(weight.dtype), rstd.data_ptr(), d_rows.data_ptr(),
                _lib.stream_handle(rows.device)), "moss_rmsnorm_bwd")
            _lib.count_launch("rmsnorm")
            d_tokens = d_rows.view(ctx.shape)
        d_weight = None
        if ctx.needs_input_grad[1]:  # a trainable gain (not on the frozen-base path): torch ops
            normalized = (rows.float() * rstd[:, None]).to(rows.dtype)
            d_weight = (grad.float() * normalized.float()).sum(0).to(weight.dtype)
        return d_tokens, d_weight, None


def rms_norm(tokens: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """``(x * rsqrt(mean(x^2) + eps)).to(x.dtype) * weight`` over the last dimension."""
    if not tokens.is_cuda:
        raise RuntimeError("rms_norm runs on CUDA tensors only (there is no CPU path).")
    if weight.shape != tokens.shape[-1:] or weight.device != tokens.device:
        raise ValueError("rms_norm: weight must be [dim] on the tokens' device.")
    return _RMSNorm.apply(tokens.contiguous(), weight.contiguous(), eps)

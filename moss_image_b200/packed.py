"""Packed variable-length batches around the int8 GEMMs.

A packed batch concatenates the tokens of samples of different lengths into one
``[1, total, dim]`` stream with cumulative boundaries ``cu_seqlens``, so every linear runs
once over all tokens (the GEMMs see M = total) and attention stays block-diagonal.

Drop-ins:

* ``training/performance.py:90-225`` - :func:`validate_attention_backend`,
  :func:`scaled_attention` and :func:`scaled_attention_varlen` (same backends, checks and
  messages). For ``auto``/``sdpa`` the variable-length attention runs torch's jagged
  (nested) scaled-dot-product attention over the packed rows: a variable-length flash
  kernel on CUDA. It never builds the reference's quadratic block mask.
* ``training/model.py:752-776`` - :func:`modulation_sample_indices`,
  :func:`condition_for_tokens` and :func:`cumulative_lengths`.

Native kernels (``moss_segment_*`` in ``libmoss_w8.so``): :func:`segment_modulate` and
:func:`segment_gate` apply each sequence's adaLN scale/shift and residual gate inside the
packed stream, bit-identical to the reference's ``index_select`` expansion followed by its
elementwise ops, without materialising the expanded ``[total, dim]`` conditions; their
backward passes reduce the condition gradients per sequence.
"""

from __future__ import annotations

import importlib
from functools import lru_cache
from typing import Callable

import torch
import torch.nn.attention
from torch.nn import functional as F

from . import _lib

_ATTENTION_BACKENDS = {"auto", "sdpa", "sdpa_cudnn", "flash_attn_2"}
# Checkpoint recomputation check for blocks that run variable-length attention: the default
# check reads the shape of every saved tensor, which jagged (nested) tensors do not have.
CHECKPOINT_CHECK = "none"
# Packed streams with at most this many sequences run one dense attention call per sequence.
VARLEN_LOOP_MAX_SEQUENCES = 32
_JAGGED_BACKENDS = [torch.nn.attention.SDPBackend.FLASH_ATTENTION, torch.nn.attention.SDPBackend.EFFICIENT_ATTENTION,
                    torch.nn.attention.SDPBackend.MATH]


# ----------------------------------------------------------------------------- attention
def _normalize_attention_backend(backend: str) -> str:
    value = str(backend).strip().lower().replace("-", "_")
    if value not in _ATTENTION_BACKENDS:
        choices = ", ".join(sorted(_ATTENTION_BACKENDS))
        raise ValueError(f"attention backend must be one of: {choices}; got {backend!r}.")
    return value


@lru_cache(maxsize=2)
def _flash_attn_function(name: str) -> Callable[..., torch.Tensor]:
    """FlashAttention-2 entry points, imported on first use (library code)."""
    try:
        package = importlib.import_module("flash_attn")
    except (ImportError, OSError) as exc:
        raise RuntimeError(
            "flash_attn_2 was requested, but flash-attn could not be imported. "
            "Install a wheel matching this Python, PyTorch, and CUDA environment.") from exc
    function = getattr(package, name, None)
    if not callable(function):
        raise RuntimeError(f"The installed flash-attn package does not expose {name}.")
    return function


def validate_attention_backend(backend: str, *, device: torch.device | str | None = None,
                               dtype: torch.dtype | None = None) -> str:
    """Reference: training/performance.py:90-112 (same checks; no CUDA work without a device)."""
    selected = _normalize_attention_backend(backend)
    target = torch.device(device) if device is not None else None
    if selected == "flash_attn_2":
        _flash_attn_function("flash_attn_func")
        if target is not None and target.type != "cuda":
            raise ValueError("flash_attn_2 requires CUDA tensors.")
        if dtype is not None and dtype not in {torch.float16, torch.bfloat16}:
            raise ValueError("flash_attn_2 requires float16 or bfloat16 query/key/value tensors.")
    elif selected == "sdpa_cudnn" and target is not None and target.type != "cuda":
        raise ValueError("sdpa_cudnn requires CUDA tensors and an enabled cuDNN attention kernel.")
    return selected


def _validate_qkv(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> None:
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("attention query, key, and value must be [batch, heads, sequence, head_dim].")
    if query.shape != key.shape or query.shape != value.shape:
        raise ValueError("attention query, key, and value must have identical shapes.")
    if query.device != key.device or query.device != value.device:
        raise ValueError("attention query, key, and value must be on the same device.")


def scaled_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                     backend: str = "auto") -> torch.Tensor:
    """Unmasked, non-causal attention on ``[B, H, N, D]``. Reference: training/performance.py:124-160."""
    _validate_qkv(query, key, value)
    query = query.to(value.dtype)
    key = key.to(value.dtype)
    selected = validate_attention_backend(backend, device=value.device, dtype=value.dtype)
    if selected in {"auto", "sdpa"}:
        return F.scaled_dot_product_attention(query, key, value)
    if selected == "sdpa_cudnn":
        from torch.nn.attention import SDPBackend, sdpa_kernel

        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            return F.scaled_dot_product_attention(query, key, value)
    output = _flash_attn_function("flash_attn_func")(query.transpose(1, 2), key.transpose(1, 2),
                                                     value.transpose(1, 2), dropout_p=0.0, causal=False)
    return output.transpose(1, 2)


def varlen_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, offsets: torch.Tensor,
                     lengths: tuple[int, ...]) -> torch.Tensor:
    """Block-diagonal attention over packed ``[total, heads, head_dim]`` rows.

    ``offsets`` holds the int64 sequence boundaries on the tensors' device and ``lengths`` the
    same boundaries on the host; each sequence attends only to itself, and memory stays linear
    in ``total``. The rows must be contiguous. Up to ``VARLEN_LOOP_MAX_SEQUENCES`` sequences
    run one dense attention call per sequence on views of the packed rows (cuDNN's Blackwell
    kernels; the split's backward writes the packed gradient once). More sequences run torch's
    jagged attention (a variable-length flash kernel) in one call.
    """
    if len(lengths) <= VARLEN_LOOP_MAX_SEQUENCES:
        parts = [F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None],
                                                v.transpose(0, 1)[None])[0].transpose(0, 1)
                 for q, k, v in zip(query.split(lengths), key.split(lengths), value.split(lengths))]
        return torch.cat(parts, 0)
    from torch.nn.attention import sdpa_kernel

    def jagged(tensor: torch.Tensor) -> torch.Tensor:
        return torch.nested.nested_tensor_from_jagged(tensor, offsets=offsets, max_seqlen=max(lengths)).transpose(1, 2)

    # jagged inputs run on the variable-length flash or memory-efficient kernels (math only
    # for what neither supports); cuDNN has no jagged form
    with sdpa_kernel(_JAGGED_BACKENDS):
        output = F.scaled_dot_product_attention(jagged(query), jagged(key), jagged(value))
    return output.transpose(1, 2).values()


def scaled_attention_varlen(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, cu_seqlens: torch.Tensor,
                            backend: str = "auto") -> torch.Tensor:
    """Isolated attention over concatenated sequences of ``[1, H, total, D]``.

    Reference: training/performance.py:163-225 (same checks and messages). ``auto``/``sdpa``
    use :func:`varlen_attention` instead of the reference's ``[total, total]`` boolean mask.
    """
    _validate_qkv(query, key, value)
    query = query.to(value.dtype)
    key = key.to(value.dtype)
    if query.shape[0] != 1:
        raise ValueError("Packed variable-length attention expects a singleton packed batch.")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError("cu_seqlens must be a 1D tensor with at least two entries.")
    lengths = cu_seqlens[1:] - cu_seqlens[:-1]
    if int(cu_seqlens[0]) != 0 or int(cu_seqlens[-1]) != query.shape[2] or bool(torch.any(lengths <= 0)):
        raise ValueError("cu_seqlens must describe positive sequences covering all packed tokens.")
    selected = validate_attention_backend(backend, device=value.device, dtype=value.dtype)
    max_length = int(lengths.max())
    if selected == "flash_attn_2":
        cumulative = cu_seqlens.to(device=value.device, dtype=torch.int32)
        output = _flash_attn_function("flash_attn_varlen_func")(
            query.squeeze(0).transpose(0, 1), key.squeeze(0).transpose(0, 1), value.squeeze(0).transpose(0, 1),
            cumulative, cumulative, max_length, max_length, dropout_p=0.0, causal=False)
        return output.transpose(0, 1).unsqueeze(0)
    if selected == "sdpa_cudnn":
        raise ValueError(
            "sdpa_cudnn does not support packed block-diagonal attention; "
            "use 'sdpa' or 'flash_attn_2' for packed batching.")
    offsets = cu_seqlens.to(device=value.device, dtype=torch.int64)
    rows = [t.squeeze(0).transpose(0, 1).contiguous() for t in (query, key, value)]
    output = varlen_attention(*rows, offsets, tuple(int(n) for n in lengths.tolist()))
    return output.transpose(0, 1).unsqueeze(0)


# ----------------------------------------------------------------------------- sequence bookkeeping
def cumulative_lengths(lengths: list[int], device: torch.device) -> torch.Tensor:
    """``[0, l0, l0 + l1, ...]`` as int64. Reference: training/model.py:774-776."""
    return torch.tensor([0, *lengths], device=device, dtype=torch.int64).cumsum(0)


def modulation_sample_indices(modulation: torch.Tensor, tokens: torch.Tensor,
                              cu_seqlens: torch.Tensor | None) -> torch.Tensor | None:
    """Per-token modulation row of a packed stream. Reference: training/model.py:752-766."""
    if modulation.shape[0] == tokens.shape[0]:
        return None
    if tokens.shape[0] != 1 or cu_seqlens is None or modulation.shape[0] != cu_seqlens.numel() - 1:
        raise ValueError("Packed modulation must contain one row per sequence.")
    lengths = (cu_seqlens[1:] - cu_seqlens[:-1]).to(dtype=torch.long)
    return torch.repeat_interleave(torch.arange(modulation.shape[0], device=modulation.device), lengths,
                                   output_size=tokens.shape[1])


def condition_for_tokens(condition: torch.Tensor, sample_indices: torch.Tensor | None) -> torch.Tensor:
    """Reference: training/model.py:769-772 (the expansion the native kernels avoid)."""
    if sample_indices is None:
        return condition[:, None]
    return condition.index_select(0, sample_indices).unsqueeze(0)


def sequence_lengths(cu_seqlens: torch.Tensor) -> tuple[int, ...]:
    """Sequence lengths of ``cu_seqlens`` on the host: read from the device once per boundaries
    tensor (a packing caller that knows them sets ``cu_seqlens.moss_lengths``)."""
    known = getattr(cu_seqlens, "moss_lengths", None)
    if known is None:
        known = tuple(int(n) for n in (cu_seqlens[1:] - cu_seqlens[:-1]).tolist())
        cu_seqlens.moss_lengths = known
    return known


_batch_offsets: dict[tuple, torch.Tensor] = {}


def batch_offsets(batch: int, length: int, device: torch.device) -> torch.Tensor:
    """Boundaries of ``batch`` equal sequences of ``length`` tokens (cached per device)."""
    key = (batch, length, device.type, device.index)
    offsets = _batch_offsets.get(key)
    if offsets is None:
        offsets = torch.arange(0, (batch + 1) * length, length, device=device, dtype=torch.int64)
        _batch_offsets[key] = offsets
    return offsets


# ----------------------------------------------------------------------------- native conditioning
def _check_stream(tokens: torch.Tensor, condition: torch.Tensor, offsets: torch.Tensor, what: str) -> None:
    if not tokens.is_cuda:
        raise RuntimeError(f"{what} runs on CUDA tensors only (there is no CPU path).")
    if condition.device != tokens.device or offsets.device != tokens.device:
        raise ValueError(f"{what}: tokens, conditions and offsets must share one device.")
    if offsets.dtype != torch.int64 or offsets.ndim != 1 or offsets.numel() != condition.shape[0] + 1:
        raise ValueError(f"{what}: offsets must be int64 [sequences + 1].")
    if condition.ndim != 2 or condition.shape[1] != tokens.shape[-1] or condition.stride(1) != 1:
        raise ValueError(f"{what}: conditions must be [sequences, dim] with contiguous rows.")


def _result_dtype(tokens: torch.Tensor, condition: torch.Tensor) -> torch.dtype:
    return torch.promote_types(tokens.dtype, condition.dtype)


def _shared_rows(first: torch.Tensor, second: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Two condition views with one row stride (the kernel takes a single stride)."""
    if first.stride(0) == second.stride(0) and first.dtype == second.dtype:
        return first, second
    dtype = torch.promote_types(first.dtype, second.dtype)
    return first.to(dtype).contiguous(), second.to(dtype).contiguous()


class _SegmentModulate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, scale, shift, offsets):
        rows = tokens.reshape(-1, tokens.shape[-1])
        out = torch.empty(rows.shape, dtype=_result_dtype(tokens, scale), device=tokens.device)
        stream = _lib.stream_handle(tokens.device)
        _lib.check(_lib.library().moss_segment_modulate(
            rows.data_ptr(), _lib.dtype_code(rows.dtype), rows.shape[0], rows.shape[1], scale.data_ptr(),
            shift.data_ptr(), _lib.dtype_code(scale.dtype), scale.stride(0), offsets.data_ptr(), scale.shape[0],
            out.data_ptr(), stream), "moss_segment_modulate")
        _lib.count_launch("segment")
        ctx.save_for_backward(rows, scale, offsets)
        ctx.shape = tokens.shape
        return out.view(*tokens.shape[:-1], tokens.shape[-1])

    @staticmethod
    def backward(ctx, grad):
        rows, scale, offsets = ctx.saved_tensors
        grad = grad.reshape(rows.shape).to(_result_dtype(rows, scale)).contiguous()
        sequences, dim = scale.shape
        d_rows = torch.empty_like(rows)
        d_scale = torch.zeros(sequences, dim, dtype=torch.float32, device=rows.device) if ctx.needs_input_grad[1] else None
        d_shift = torch.zeros(sequences, dim, dtype=torch.float32, device=rows.device) if ctx.needs_input_grad[2] else None
        _lib.check(_lib.library().moss_segment_modulate_bwd(
            grad.data_ptr(), rows.data_ptr(), _lib.dtype_code(rows.dtype), rows.shape[0], dim, scale.data_ptr(),
            _lib.dtype_code(scale.dtype), scale.stride(0), offsets.data_ptr(), sequences, d_rows.data_ptr(),
            None if d_scale is None else d_scale.data_ptr(), None if d_shift is None else d_shift.data_ptr(),
            _lib.stream_handle(rows.device)), "moss_segment_modulate_bwd")
        _lib.count_launch("segment")
        return (d_rows.view(ctx.shape), None if d_scale is None else d_scale.to(scale.dtype),
                None if d_shift is None else d_shift.to(scale.dtype), None)


class _SegmentGate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, tokens, update, gate, offsets):
        rows = tokens.reshape(-1, tokens.shape[-1])
        branch = update.reshape(rows.shape)
        out = torch.empty(rows.shape, dtype=_result_dtype(tokens, gate), device=tokens.device)
        _lib.check(_lib.library().moss_segment_gate(
            rows.data_ptr(), branch.data_ptr(), _lib.dtype_code(rows.dtype), rows.shape[0], rows.shape[1],
            gate.data_ptr(), _lib.dtype_code(gate.dtype), gate.stride(0), offsets.data_ptr(), gate.shape[0],
            out.data_ptr(), _lib.stream_handle(tokens.device)), "moss_segment_gate")
        _lib.count_launch("segment")
        ctx.save_for_backward(branch, gate, offsets)
        ctx.shape = tokens.shape
        ctx.token_dtype = tokens.dtype
        return out.view(*tokens.shape[:-1], tokens.shape[-1])

    @staticmethod
    def backward(ctx, grad):
        branch, gate, offsets = ctx.saved_tensors
        grad = grad.reshape(branch.shape).to(_result_dtype(branch, gate)).contiguous()
        d_tokens = grad.to(ctx.token_dtype).view(ctx.shape) if ctx.needs_input_grad[0] else None
        d_branch, d_gate = None, None
        if ctx.needs_input_grad[1] or ctx.needs_input_grad[2]:
            d_branch = torch.empty_like(branch)
            if ctx.needs_input_grad[2]:
                d_gate = torch.zeros(gate.shape, dtype=torch.float32, device=branch.device)
            _lib.check(_lib.library().moss_segment_gate_bwd(
                grad.data_ptr(), branch.data_ptr(), _lib.dtype_code(branch.dtype), branch.shape[0], branch.shape[1],
                gate.data_ptr(), _lib.dtype_code(gate.dtype), gate.stride(0), offsets.data_ptr(), gate.shape[0],
                d_branch.data_ptr(), None if d_gate is None else d_gate.data_ptr(),
                _lib.stream_handle(branch.device)), "moss_segment_gate_bwd")
            _lib.count_launch("segment")
            d_branch = d_branch.view(ctx.shape) if ctx.needs_input_grad[1] else None
            d_gate = None if d_gate is None else d_gate.to(gate.dtype)
        return d_tokens, d_branch, d_gate, None


def segment_modulate(tokens: torch.Tensor, scale: torch.Tensor, shift: torch.Tensor,
                     offsets: torch.Tensor) -> torch.Tensor:
    """``tokens * (1 + scale[s]) + shift[s]`` per sequence s of a packed ``[..., dim]`` stream.

    Bit-identical to ``tokens * (1 + condition_for_tokens(scale, idx)) + condition_for_tokens(shift, idx)``
    (training/model.py:291-293, :303-305). ``scale``/``shift``: ``[sequences, dim]`` (strided
    rows allowed); ``offsets``: int64 ``[sequences + 1]`` on the same device.
    """
    _check_stream(tokens, scale, offsets, "segment_modulate")
    scale, shift = _shared_rows(scale, shift)
    return _SegmentModulate.apply(tokens.contiguous(), scale, shift, offsets)


def segment_gate(tokens: torch.Tensor, update: torch.Tensor, gate: torch.Tensor, offsets: torch.Tensor) -> torch.Tensor:
    """``tokens + update * gate[s]`` per sequence s (training/model.py:302, :310-312)."""
    _check_stream(tokens, gate, offsets, "segment_gate")
    if update.shape != tokens.shape or update.dtype != tokens.dtype:
        raise ValueError("segment_gate: update must have the tokens' shape and dtype.")
    return _SegmentGate.apply(tokens.contiguous(), update.contiguous(), gate, offsets)

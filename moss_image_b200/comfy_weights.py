"""Comfy ``int8_tensorwise`` (optionally ConvRot) checkpoints: dense decode and direct int8 load.

Drop-in for ``training/comfy_weights.py``: :func:`decode_comfy_state` and
:func:`load_comfy_state` take the same arguments, accept and reject the same storage with the
same messages and return bit-identical dense tensors (``float(codes) * scale`` per output row in
float32, rotated back by the regular normalised Hadamard when ``convrot`` is set, then cast).

The reference only decodes: a quantised checkpoint becomes dense weights, and a LoRA run then
re-quantises them, which moves codes wherever the dense rounding crosses a rounding boundary.
:func:`load_comfy_quantized` keeps the checkpoint's codes: each quantised linear becomes a
:class:`~moss_image_b200.quantization.FrozenInt8Linear` (or, for ConvRot storage, a
:class:`~moss_image_b200.convrot.FrozenConvRotLinear`, whose stored codes are likewise int8 of
``W H`` with per-row scales) built from the codes and scales as stored - no dense decode, no
re-quantisation, one byte per weight on the way to the device.
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path

import torch
from torch import nn

from .convrot import FrozenConvRotLinear, rotate_hadamard
from .quantization import FrozenInt8Linear

_DENSE_DTYPES = {torch.float16, torch.bfloat16, torch.float32, torch.float64}
_MARKER_FIELDS = {"format", "convrot", "convrot_groupsize", "full_precision_matrix_mult"}
_DECODE_CHUNK_ELEMENTS = 4 * 1024 * 1024


@dataclass(frozen=True)
class ComfyInt8Weight:
    """One quantised weight as stored: ``codes`` int8 ``[out, in]`` (of ``W H`` when ``group > 1``),
    ``scale`` float32 ``[out, 1]``, and the Hadamard group (1 = no rotation)."""

    codes: torch.Tensor
    scale: torch.Tensor
    group: int


def _marker_config(marker: torch.Tensor, name: str) -> dict:
    """Parse and check a ``comfy_quant`` JSON marker. Reference: training/comfy_weights.py:23-39."""
    if marker.dtype != torch.uint8 or marker.ndim != 1:
        raise ValueError(f"{name}: comfy_quant must be a one-dimensional uint8 JSON marker.")
    try:
        config = json.loads(bytes(marker.cpu().tolist()).decode("utf-8"))
    except (ValueError, UnicodeError) as exc:
        raise ValueError(f"{name}: malformed comfy_quant JSON.") from exc
    if not isinstance(config, dict) or config.get("format") != "int8_tensorwise":
        raise ValueError(f"{name}: only Comfy int8_tensorwise storage is supported; packed/GPTQ formats are unsupported.")
    if set(config) - _MARKER_FIELDS:
        raise ValueError(f"{name}: unsupported quantization metadata fields.")
    if not isinstance(config.get("convrot", False), bool):
        raise ValueError(f"{name}: convrot must be a boolean.")
    if "convrot_groupsize" in config and not config.get("convrot", False):
        raise ValueError(f"{name}: rotation group specified without convrot.")
    return config


def _take_quantized(state: dict[str, torch.Tensor], key: str) -> tuple[str, ComfyInt8Weight]:
    """Remove one marker with its weight and scale from ``state`` and check them.

    Reference: training/comfy_weights.py:49-75 (same checks, same order, same messages).
    """
    prefix = key[: -len(".comfy_quant")]
    config = _marker_config(state.pop(key), prefix)
    weight_key, scale_key = prefix + ".weight", prefix + ".weight_scale"
    if weight_key not in state or scale_key not in state:
        raise ValueError(f"{prefix}: quantized weight requires weight, weight_scale and comfy_quant together.")
    codes, scale = state.pop(weight_key), state.pop(scale_key)
    if codes.dtype != torch.int8 or codes.ndim != 2:
        raise ValueError(f"{prefix}: int8_tensorwise weight must be int8 [out, in]; packed tensors are unsupported.")
    if scale.dtype != torch.float32 or tuple(scale.shape) != (codes.shape[0], 1):
        raise ValueError(f"{prefix}: weight_scale must be float32 [out, 1].")
    if not torch.isfinite(scale).all() or not (scale > 0).all():
        raise ValueError(f"{prefix}: weight_scale must be finite and positive.")
    group = 1
    if config.get("convrot", False):
        group = config.get("convrot_groupsize", 256)
        # Comfy's regular Hadamard is a Kronecker power of H4: the group is a power of four
        if (isinstance(group, bool) or not isinstance(group, int) or group < 4
                or group & (group - 1) or (group.bit_length() - 1) % 2):
            raise ValueError(f"{prefix}: Comfy ConvRot group size must be a power of four >= 4.")
        if codes.shape[1] % group:
            raise ValueError(f"{prefix}: input width is not divisible by declared ConvRot group size.")
    return prefix, ComfyInt8Weight(codes, scale, group)


def _check_dense(key: str, value: torch.Tensor) -> None:
    """Reference: training/comfy_weights.py:89-96 (side tensors and non-dense weights)."""
    if key.endswith(".weight_scale") or key.endswith(".input_scale"):
        raise ValueError(f"{key}: unmatched or unsupported quantization side tensor.")
    if key.endswith(".weight") and value.dtype not in _DENSE_DTYPES:
        raise ValueError(f"{key}: integer/packed/float8 weights need a supported comfy_quant marker.")
    if value.is_floating_point() and value.dtype not in _DENSE_DTYPES:
        raise ValueError(f"{key}: unsupported floating-point storage format.")


def decode_weight(weight: ComfyInt8Weight, dtype: torch.dtype) -> torch.Tensor:
    """Dense ``rotate(float(codes) * scale)`` cast to ``dtype``, decoded in row chunks.

    Reference: training/comfy_weights.py:76-86: float32 product, the eager Hadamard (which
    repeats the reference's expressions in order), then one cast; chunks of about 4M values
    keep float32 temporaries small for embedding tables.
    """
    codes, scale = weight.codes, weight.scale
    dense = torch.empty(codes.shape, device=codes.device, dtype=dtype)
    rows = max(1, _DECODE_CHUNK_ELEMENTS // max(1, codes.shape[1]))
    for first in range(0, codes.shape[0], rows):
        decoded = codes[first:first + rows].float() * scale[first:first + rows]
        if weight.group > 1:
            decoded = rotate_hadamard(decoded, weight.group)
        dense[first:first + rows] = decoded.to(dtype=dtype)
    return dense


def split_comfy_state(state: Mapping[str, torch.Tensor]) -> tuple[dict[str, ComfyInt8Weight], dict[str, torch.Tensor]]:
    """Separate quantised weights (by module prefix) from the other tensors, checking both.

    Nothing is decoded or cast; the caller's mapping is not modified.
    """
    remaining = dict(state)
    quantized = dict(_take_quantized(remaining, key) for key in list(remaining) if key.endswith(".comfy_quant"))
    for key, value in remaining.items():
        _check_dense(key, value)
    return quantized, remaining


def _decode(state: dict[str, torch.Tensor], dtype: torch.dtype) -> dict[str, torch.Tensor]:
    """Reference: training/comfy_weights.py:42-98. Consumes ``state`` as it goes."""
    if dtype not in _DENSE_DTYPES:
        raise ValueError("Dense checkpoint output dtype must be float16, bfloat16, float32 or float64.")
    result = {}
    for key in list(state):
        if not key.endswith(".comfy_quant"):
            continue
        prefix, weight = _take_quantized(state, key)
        result[prefix + ".weight"] = decode_weight(weight, dtype)
        del weight
    for key in list(state):
        value = state.pop(key)
        _check_dense(key, value)
        result[key] = value.to(dtype=dtype) if value.is_floating_point() else value
    return result


def decode_comfy_state(state: Mapping[str, torch.Tensor], dtype: torch.dtype = torch.bfloat16) -> dict[str, torch.Tensor]:
    """Decode every supported marker to dense weights without mutating the caller's mapping."""
    return _decode(dict(state), dtype)


def load_comfy_state(path: str | Path, dtype: torch.dtype = torch.bfloat16) -> dict[str, torch.Tensor]:
    """Load a safetensors checkpoint on the CPU and expand quantised rows to dense."""
    from safetensors.torch import load_file

    return _decode(load_file(str(path), device="cpu"), dtype)


def _frozen_from_codes(weight: ComfyInt8Weight, bias: torch.Tensor | None, dtype: torch.dtype,
                       device: torch.device, backend: str) -> FrozenInt8Linear:
    codes = weight.codes.to(device)
    scale = weight.scale.reshape(-1).to(device)
    bias = None if bias is None else bias.to(device=device, dtype=dtype)
    if weight.group > 1:
        return FrozenConvRotLinear.from_codes(codes, scale, bias, weight.group, dtype=dtype, backend=backend)
    return FrozenInt8Linear.from_codes(codes, scale, bias, dtype=dtype, backend=backend)


def load_comfy_quantized(
    model: nn.Module,
    state: Mapping[str, torch.Tensor],
    *,
    dtype: torch.dtype = torch.bfloat16,
    device: torch.device | str | None = None,
    backend: str = "eager",
    strict: bool = True,
) -> list[str]:
    """Load a Comfy checkpoint into ``model`` keeping quantised linears as int8.

    Every ``nn.Linear`` whose prefix carries an ``int8_tensorwise`` marker is replaced by a
    frozen int8 module built from the stored codes and scales (ConvRot storage: a ConvRot
    module with the stored group), placed on ``device`` (default: where the linear was) with
    compute dtype ``dtype``. Other quantised tensors (embedding tables) are decoded exactly as
    :func:`decode_comfy_state` decodes them, and they and the remaining tensors are copied into
    the model's existing parameters and buffers. Returns the replaced module paths.
    """
    if dtype not in _DENSE_DTYPES:
        raise ValueError("Dense checkpoint output dtype must be float16, bfloat16, float32 or float64.")
    quantized, dense = split_comfy_state(state)
    modules = dict(model.named_modules())
    replaced = []
    for prefix, weight in quantized.items():
        module = modules.get(prefix)
        if not isinstance(module, nn.Linear):
            dense[prefix + ".weight"] = decode_weight(weight, dtype)
            continue
        if tuple(weight.codes.shape) != (module.out_features, module.in_features):
            raise ValueError(f"{prefix}: checkpoint weight {tuple(weight.codes.shape)} does not match the module "
                             f"({module.out_features}, {module.in_features}).")
        bias = dense.pop(prefix + ".bias", None)
        if (bias is None) != (module.bias is None):
            raise ValueError(f"{prefix}: checkpoint and module disagree about the bias.")
        target = torch.device(device) if device is not None else module.weight.device
        parent_name, _, leaf = prefix.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, leaf, _frozen_from_codes(weight, bias, dtype, target, backend))
        replaced.append(prefix)
    cast = {key: value.to(dtype=dtype) if value.is_floating_point() else value for key, value in dense.items()}
    result = model.load_state_dict(cast, strict=False)
    missing = [key for key in result.missing_keys if not any(key.startswith(p + ".") for p in replaced)]
    if strict and (missing or result.unexpected_keys):
        raise ValueError(f"Comfy checkpoint does not match the model: missing {missing[:8]}, "
                         f"unexpected {result.unexpected_keys[:8]}")
    return replaced

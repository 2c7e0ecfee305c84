"""Comfy ``int8_tensorwise`` golden cases shared by ``make_golden.py`` and the tests.

Seeded codes and scales, the marker fields of every decode case, and the malformed states
whose reference error messages the fixtures record.
"""

from __future__ import annotations

import json

import torch

# name, rows, cols, marker fields, output dtype
COMFY_CASES = [
    ("comfy.rot4_f32", 2, 4, {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 4}, torch.float32),
    ("comfy.plain_bf16", 19, 96, {"format": "int8_tensorwise"}, torch.bfloat16),
    ("comfy.plain_f32_fpmm", 7, 40, {"format": "int8_tensorwise", "full_precision_matrix_mult": True}, torch.float32),
    ("comfy.rot16_f32", 11, 64, {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 16},
     torch.float32),
    ("comfy.rot64_bf16", 9, 192, {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 64},
     torch.bfloat16),
    ("comfy.rot256_f16", 5, 512, {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256},
     torch.float16),
    ("comfy.rotdefault_f64", 3, 512, {"format": "int8_tensorwise", "convrot": True}, torch.float64),
    ("comfy.rot1024_f32", 3, 2048, {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 1024},
     torch.float32),
]


def comfy_marker(fields: dict) -> torch.Tensor:
    return torch.tensor(list(json.dumps(fields).encode()), dtype=torch.uint8)


def comfy_codes(rows: int, cols: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Seeded int8 codes over the full range and positive float32 row scales ``[rows, 1]``."""
    gen = torch.Generator().manual_seed(seed)
    codes = torch.randint(-128, 128, (rows, cols), generator=gen, dtype=torch.int64).to(torch.int8)
    scale = (torch.rand(rows, 1, generator=gen) * 0.05 + 1e-3).float()
    return codes, scale


def comfy_fixture() -> dict[str, torch.Tensor]:
    """A small valid state: one rotated linear, its bias, and an integer counter."""
    return {"layer.weight": torch.tensor([[1, 2, 3, 4], [-4, -3, -2, -1]], dtype=torch.int8),
            "layer.weight_scale": torch.tensor([[0.25], [0.125]], dtype=torch.float32),
            "layer.comfy_quant": comfy_marker({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 4}),
            "layer.bias": torch.tensor([1.0, 2.0]),
            "vae.num_batches_tracked": torch.tensor(9)}


def _set(key: str, value):
    return lambda state: state.update({key: value() if callable(value) else value})


def comfy_mutations() -> dict:
    """Malformed variants of :func:`comfy_fixture`, by label."""
    rot = {"format": "int8_tensorwise", "convrot": True}
    return {
        "missing_scale": lambda s: s.pop("layer.weight_scale"),
        "missing_marker": lambda s: s.pop("layer.comfy_quant"),
        "gptq_format": _set("layer.comfy_quant", lambda: comfy_marker({**rot, "format": "gptq"})),
        "bad_json": _set("layer.comfy_quant", torch.tensor([255], dtype=torch.uint8)),
        "marker_not_uint8": _set("layer.comfy_quant", torch.tensor([1, 2], dtype=torch.int32)),
        "extra_field": _set("layer.comfy_quant", lambda: comfy_marker({**rot, "convrot_groupsize": 4, "x": 1})),
        "scale_1d": _set("layer.weight_scale", torch.ones(2)),
        "scale_f16": _set("layer.weight_scale", torch.ones(2, 1, dtype=torch.float16)),
        "scale_zero": _set("layer.weight_scale", torch.zeros(2, 1)),
        "scale_nan": _set("layer.weight_scale", torch.full((2, 1), float("nan"))),
        "scale_inf": _set("layer.weight_scale", torch.full((2, 1), float("inf"))),
        "weight_uint8": _set("layer.weight", torch.ones(2, 4, dtype=torch.uint8)),
        "weight_3d": _set("layer.weight", torch.ones(2, 4, 1, dtype=torch.int8)),
        "group_16_width_4": _set("layer.comfy_quant", lambda: comfy_marker({**rot, "convrot_groupsize": 16})),
        "group_8": _set("layer.comfy_quant", lambda: comfy_marker({**rot, "convrot_groupsize": 8})),
        "group_2": _set("layer.comfy_quant", lambda: comfy_marker({**rot, "convrot_groupsize": 2})),
        "group_bool": _set("layer.comfy_quant", lambda: comfy_marker({**rot, "convrot_groupsize": True})),
        "convrot_string": _set("layer.comfy_quant", lambda: comfy_marker({"format": "int8_tensorwise",
                                                                          "convrot": "yes"})),
        "group_without_convrot": _set("layer.comfy_quant", lambda: comfy_marker({"format": "int8_tensorwise",
                                                                                 "convrot_groupsize": 4})),
        "stray_input_scale": _set("other.input_scale", torch.ones(1)),
        "stray_weight_scale": _set("other.weight_scale", torch.ones(2, 1)),
        "int8_weight_unmarked": _set("other.weight", torch.ones(2, 2, dtype=torch.int8)),
        "float8_tensor": _set("other.bias", lambda: torch.zeros(2).to(torch.float8_e4m3fn)),
    }

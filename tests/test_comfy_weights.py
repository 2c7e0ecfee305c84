"""Comfy int8_tensorwise storage on the CPU: the dense decode against the reference's outputs,
the reference's error messages, and the direct int8 load (codes kept as stored).

Golden arrays come from the reference's ``training.comfy_weights.decode_comfy_state``
(tests/golden/make_golden.py); the cases themselves are in tests/golden/comfy_cases.py.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch
from torch import nn
from torch.nn import functional as F

from golden.comfy_cases import COMFY_CASES, comfy_codes, comfy_fixture, comfy_marker, comfy_mutations
from moss_image_b200.comfy_weights import (
    decode_comfy_state,
    load_comfy_quantized,
    load_comfy_state,
    split_comfy_state,
)
from moss_image_b200.convrot import FrozenConvRotLinear, rotate_hadamard
from moss_image_b200.quantization import FrozenInt8Linear


def _state(name, rows, cols, fields, seed):
    codes, scale = comfy_codes(rows, cols, seed=seed)
    return {"layer.weight": codes, "layer.weight_scale": scale, "layer.comfy_quant": comfy_marker(fields),
            "layer.bias": torch.linspace(-1, 1, rows), "norm.num_batches_tracked": torch.tensor(9)}


@pytest.mark.parametrize("index", range(len(COMFY_CASES)))
def test_dense_decode_is_bit_exact_with_the_reference(golden_arrays, golden_meta, index):
    name, rows, cols, fields, dtype = COMFY_CASES[index]
    state = _state(name, rows, cols, fields, 700 + index)
    np.testing.assert_array_equal(state["layer.weight"].numpy(), golden_arrays[f"{name}.codes"])
    dense = decode_comfy_state(state, dtype)
    assert len(state) == 5  # the caller's mapping survives
    expected = golden_meta["comfy"][name]
    assert sorted(dense) == expected["keys"]
    assert dense["layer.weight"].dtype == dtype
    np.testing.assert_array_equal(dense["layer.weight"].to(torch.float64).numpy(), golden_arrays[f"{name}.dense"])
    assert str(dense["layer.bias"].dtype).split(".")[-1] == expected["bias_dtype"]
    assert str(dense["norm.num_batches_tracked"].dtype).split(".")[-1] == expected["counter_dtype"]


def test_decode_in_row_chunks_matches_the_reference_hash(golden_meta):
    case = golden_meta["comfy_chunked"]
    codes, scale = comfy_codes(case["rows"], case["cols"], seed=case["seed"])
    assert hashlib.sha256(codes.numpy().tobytes()).hexdigest() == case["codes_sha"]
    dense = decode_comfy_state({"embed.weight": codes, "embed.weight_scale": scale,
                                "embed.comfy_quant": comfy_marker(case["fields"])})["embed.weight"]
    assert hashlib.sha256(dense.view(torch.int16).numpy().tobytes()).hexdigest() == case["dense_bf16_sha"]


@pytest.mark.parametrize("label", sorted(comfy_mutations()))
def test_malformed_storage_raises_the_reference_message(golden_meta, label):
    state = comfy_fixture()
    comfy_mutations()[label](state)
    with pytest.raises(ValueError) as error:
        decode_comfy_state(state)
    assert str(error.value) == golden_meta["comfy_errors"][label]


def test_regular_hadamard_semantics_and_file_load(tmp_path):
    """Codes represent W H: the decode rotates back, so x W^T == (x H) (W H)^T."""
    from safetensors.torch import save_file

    state = comfy_fixture()
    dense = decode_comfy_state(state, torch.float32)
    h4 = torch.tensor([[1.0, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]]) / 2
    rotated = state["layer.weight"].float() * state["layer.weight_scale"]
    torch.testing.assert_close(dense["layer.weight"], rotated @ h4)
    x = torch.randn(3, 4)
    torch.testing.assert_close(F.linear(x, dense["layer.weight"]), F.linear(x @ h4, rotated))
    with pytest.raises(ValueError, match="output dtype"):
        decode_comfy_state(state, torch.int8)
    q = torch.randint(-128, 128, (5, 256), dtype=torch.int8)
    scale = torch.full((5, 1), 0.01)
    saved = {"embed.weight": q, "embed.weight_scale": scale, "norm.weight": torch.ones(5),
             "embed.comfy_quant": comfy_marker({"format": "int8_tensorwise", "convrot": True})}
    path = tmp_path / "model.safetensors"
    save_file(saved, str(path))
    loaded = load_comfy_state(path)
    assert loaded["embed.weight"].dtype == torch.bfloat16 and loaded["norm.weight"].dtype == torch.bfloat16
    assert torch.equal(loaded["embed.weight"], rotate_hadamard(q.float() * scale, 256).bfloat16())


class _Tiny(nn.Module):
    def __init__(self) -> None:
        super().__init__()
        self.embed = nn.Embedding(5, 256)
        self.proj = nn.Linear(256, 6)
        self.rot = nn.Linear(64, 3, bias=False)
        self.norm = nn.LayerNorm(6)


def test_direct_load_keeps_the_stored_codes_and_decodes_only_tables():
    torch.manual_seed(3)
    codes, scale = comfy_codes(6, 256, seed=1)
    rot_codes, rot_scale = comfy_codes(3, 64, seed=2)
    table, table_scale = comfy_codes(5, 256, seed=4)
    state = {
        "proj.weight": codes, "proj.weight_scale": scale, "proj.bias": torch.randn(6),
        "proj.comfy_quant": comfy_marker({"format": "int8_tensorwise"}),
        "rot.weight": rot_codes, "rot.weight_scale": rot_scale,
        "rot.comfy_quant": comfy_marker({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 16}),
        "embed.weight": table, "embed.weight_scale": table_scale,
        "embed.comfy_quant": comfy_marker({"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 64}),
        "norm.weight": torch.randn(6), "norm.bias": torch.randn(6),
    }
    quantized, dense = split_comfy_state(state)
    assert sorted(quantized) == ["embed", "proj", "rot"] and sorted(dense) == ["norm.bias", "norm.weight",
                                                                              "proj.bias"]
    assert quantized["rot"].group == 16 and quantized["proj"].group == 1
    model = _Tiny()
    replaced = load_comfy_quantized(model, state, dtype=torch.bfloat16)
    assert replaced == ["proj", "rot"]
    assert type(model.proj) is FrozenInt8Linear and isinstance(model.rot, FrozenConvRotLinear)
    assert torch.equal(model.proj.weight_int8, codes) and torch.equal(model.proj.weight_scale, scale[:, 0])
    assert model.proj.compute_dtype == torch.bfloat16 and torch.equal(model.proj.bias, state["proj.bias"].bfloat16())
    assert model.rot.group_size == 16 and int(model.rot.rotation_group_size) == 16 and model.rot.bias is None
    assert torch.equal(model.rot.weight_int8, rot_codes)
    expected_table = decode_comfy_state({k: v for k, v in state.items() if k.startswith("embed.")},
                                        torch.bfloat16)["embed.weight"]
    assert torch.equal(model.embed.weight.detach(), expected_table.float())
    assert torch.equal(model.norm.weight.detach(), state["norm.weight"].bfloat16().float())
    keys = set(model.state_dict())
    assert {"proj.weight_int8", "proj.weight_scale", "rot.rotation_group_size"} <= keys
    with pytest.raises(ValueError, match="does not match the module"):
        load_comfy_quantized(_Tiny(), {**state, "rot.weight": torch.zeros(3, 128, dtype=torch.int8)})
    with pytest.raises(ValueError, match="does not match the model"):
        load_comfy_quantized(_Tiny(), {k: v for k, v in state.items() if not k.startswith("norm.")})
    with pytest.raises(ValueError, match="power of two that divides"):
        FrozenConvRotLinear.from_codes(rot_codes, rot_scale[:, 0], None, 128)
    with pytest.raises(ValueError, match="float32"):
        FrozenInt8Linear.from_codes(codes, scale)

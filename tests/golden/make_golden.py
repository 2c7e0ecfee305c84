"""Generate golden vectors from the reference implementation (run where it is importable).

    python tests/golden/make_golden.py --reference /path/to/MOSS-Image

Imports the reference's own ``training.quantization`` and ``training.activation_offload``
and records, on CPU:

* quantiser codes/scales for small shapes (arrays) and for every BASELINE.json weight
  shape (sha256 of the code and scale bytes), including bf16/fp16 source weights,
  all-zero rows and hand-built round-half-to-even ties;
* eager forward/input-gradient outputs of ``FrozenInt8Linear`` on ragged bf16 shapes,
  plus the bit-exact decode/bias-rounding known-answer case of the reference GPU test
  (training/tests/test_quant_kernels.py:85-129) evaluated with the reference eager path;
* ``_offload_view`` payload shapes for padded, expanded, overlapping, transposed and
  sliced layouts (training/tests/test_packed_features.py:201-235 and more);
* ConvRot (``training.convrot``): ``rotate_hadamard`` outputs in f32 and f64 for every
  group size from 1 to 512, ``effective_group_size`` answers, and the codes, scales,
  rotated weights, eager outputs and input gradients of ``FrozenConvRotLinear``;
* Comfy ``int8_tensorwise`` storage (``training.comfy_weights``): dense decodes of the seeded
  cases in ``comfy_cases.py`` (plain and ConvRot, every output dtype), the hash of a decode
  large enough to run in several row chunks, and the reference's error message for each
  malformed state.

Outputs: tests/golden/golden.npz (small arrays) and tests/golden/golden.json (hashes and
metadata). The GPU box never runs this script; the tests read the committed outputs.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch
from torch import nn

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
from comfy_cases import COMFY_CASES, comfy_codes, comfy_fixture, comfy_marker, comfy_mutations  # noqa: E402

# Weight shapes [out, in] of BASELINE.json configs 1/2/5 (q/k/v/o, MLP up/down, adaLN)
# and the real MOSS block's fused up-gate and down projections.
BASELINE_SHAPES = [(3072, 3072), (12288, 3072), (3072, 12288), (18432, 3072), (9216, 3072), (16384, 3072),
                   (3072, 8192)]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.float().numpy()
    return t.numpy()


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the MOSS-Image checkout")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    from training.activation_offload import _offload_view  # noqa: E402
    from training.quantization import FrozenInt8Linear  # noqa: E402

    arrays: dict[str, np.ndarray] = {}
    meta: dict[str, object] = {"quant_hash": {}, "offload_view": [], "cases": {}}

    # ---------------------------------------------------------------- quantiser, small arrays
    def record_quant(name: str, linear: nn.Linear) -> None:
        module = FrozenInt8Linear(linear.requires_grad_(False))
        arrays[f"{name}.w"] = to_np(linear.weight.float())
        arrays[f"{name}.q"] = module.weight_int8.numpy()
        arrays[f"{name}.s"] = module.weight_scale.numpy()

    torch.manual_seed(73)
    record_quant("q_70x37_f32", nn.Linear(70, 37))
    torch.manual_seed(7)
    lin = nn.Linear(64, 32)
    with torch.no_grad():
        lin.weight[0].zero_()
    record_quant("q_64x32_zero_row", lin)
    torch.manual_seed(11)
    record_quant("q_96x40_bf16", nn.Linear(96, 40, dtype=torch.bfloat16))
    torch.manual_seed(12)
    record_quant("q_48x24_f16", nn.Linear(48, 24, dtype=torch.float16))
    ties = nn.Linear(8, 3, bias=False)
    with torch.no_grad():
        ties.weight.copy_(torch.tensor([
            [127.0, 2.5, 3.5, -2.5, -0.5, 0.5, 1.5, 126.5],
            [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
            [1e-30, -3e-30, 2e-30, 0.0, 5e-31, -1e-30, 3e-30, -2.5e-30],
        ]))
    record_quant("q_ties", ties)

    # ---------------------------------------------------------------- quantiser, BASELINE shapes
    for out_f, in_f in BASELINE_SHAPES:
        for dtype in (torch.float32, torch.bfloat16):
            gen = torch.Generator().manual_seed(0)
            w = (torch.randn(out_f, in_f, generator=gen) * 0.02).to(dtype)
            lin = nn.Linear(in_f, out_f, bias=False, dtype=dtype)
            with torch.no_grad():
                lin.weight.copy_(w)
            module = FrozenInt8Linear(lin.requires_grad_(False))
            key = f"{out_f}x{in_f}:{str(dtype).split('.')[-1]}"
            meta["quant_hash"][key] = {
                "codes_sha256": sha(module.weight_int8.numpy()),
                "scale_sha256": sha(module.weight_scale.numpy()),
                "weight_sha256": sha(to_np(w.float())),
            }

    # ---------------------------------------------------------------- eager forward / dX
    def record_linear(name: str, in_f: int, out_f: int, lead: tuple[int, ...], dtype: torch.dtype, seed: int,
                      bias: bool = True) -> None:
        torch.manual_seed(seed)
        base = nn.Linear(in_f, out_f, bias=bias, dtype=dtype).requires_grad_(False)
        module = FrozenInt8Linear(base)
        tokens = torch.randn(*lead, in_f, dtype=dtype, requires_grad=True)
        out = module(tokens)
        grad = torch.randn_like(out)
        out.backward(grad)
        arrays[f"{name}.q"] = module.weight_int8.numpy()
        arrays[f"{name}.s"] = module.weight_scale.numpy()
        if bias:
            arrays[f"{name}.bias"] = to_np(module.bias)
        arrays[f"{name}.x"] = to_np(tokens)
        arrays[f"{name}.y"] = to_np(out)
        arrays[f"{name}.dy"] = to_np(grad)
        arrays[f"{name}.dx"] = to_np(tokens.grad)
        meta["cases"][name] = {"dtype": str(dtype).split(".")[-1], "lead": list(lead), "bias": bias}

    record_linear("lin_70x37_bf16", 70, 37, (2, 3), torch.bfloat16, 73)
    record_linear("lin_256x320_bf16", 256, 320, (5, 29), torch.bfloat16, 5)
    record_linear("lin_160x96_f16", 160, 96, (33,), torch.float16, 6, bias=False)

    # ---------------------------------------------------------------- known-answer decode/bias case
    for base_dtype in (torch.bfloat16, torch.float32):
        base = nn.Linear(70, 37, bias=True, dtype=base_dtype).requires_grad_(False)
        eager = FrozenInt8Linear(base)
        scale = 0.0002928110350837356
        with torch.no_grad():
            eager.weight_int8.zero_()
            eager.weight_int8[0, 0] = 83
            eager.weight_int8[1, 1] = -83
            eager.weight_scale.fill_(scale)
            eager.weight_int8[2:6, 2] = 1
            eager.weight_scale[2:6] = 1
            eager.bias.zero_()
            eager.bias[0] = 0.08285745223138713
        tokens = torch.zeros(1, 70, dtype=base_dtype, requires_grad=True)
        with torch.no_grad():
            tokens[0, :2] = 1
        with torch.autocast("cpu", dtype=torch.bfloat16):
            out = eager(tokens)
        grad = torch.zeros_like(out)
        grad[0, :2] = 1
        grad[0, 2:6] = torch.tensor([-0.1962890625, -2.265625, -0.52734375, 1.546875], dtype=torch.bfloat16)
        out.backward(grad)
        name = f"kat_{str(base_dtype).split('.')[-1]}"
        arrays[f"{name}.q"] = eager.weight_int8.numpy()
        arrays[f"{name}.s"] = eager.weight_scale.numpy()
        arrays[f"{name}.bias"] = to_np(eager.bias.float())
        arrays[f"{name}.x"] = to_np(tokens.float())
        arrays[f"{name}.y"] = to_np(out)
        arrays[f"{name}.dy"] = to_np(grad)
        arrays[f"{name}.dx"] = to_np(tokens.grad.float())
        meta["cases"][name] = {"base_dtype": str(base_dtype).split(".")[-1], "out_dtype": str(out.dtype).split(".")[-1],
                               "dx_dtype": str(tokens.grad.dtype).split(".")[-1]}

    # ---------------------------------------------------------------- offload payload views
    backing = torch.arange(4096, dtype=torch.float32)
    layouts = [
        ("padded", (1, 1, 5, 5), (64, 64, 8, 1)),
        ("expanded", (3, 5), (0, 1)),
        ("overlapping", (3, 3), (1, 1)),
        ("transposed", (6, 4), (1, 6)),
        ("sliced_rows", (4, 7), (16, 1)),
        ("expanded_inner", (2, 3, 4), (12, 4, 0)),
        ("scalar_broadcast", (5, 5), (0, 0)),
        ("contiguous", (2, 3, 4), (12, 4, 1)),
        ("size_one_odd_stride", (3, 1, 4), (4, 999, 1)),
        ("overlap_window", (4, 4), (2, 1)),
    ]
    for name, shape, stride in layouts:
        view = backing.as_strided(shape, stride)
        result = _offload_view(view)
        meta["offload_view"].append({
            "name": name, "shape": list(shape), "stride": list(stride),
            "payload_shape": None if result is None else list(result[1]),
        })

    # ---------------------------------------------------------------- ConvRot
    from training.convrot import FrozenConvRotLinear, effective_group_size, rotate_hadamard  # noqa: E402

    for group in (1, 2, 4, 8, 16, 32, 64, 128, 256, 512):
        gen = torch.Generator().manual_seed(500 + group)
        x = torch.randn(3, 2 * group, generator=gen)
        arrays[f"hadamard.g{group}.x"] = x.numpy()
        arrays[f"hadamard.g{group}.y32"] = rotate_hadamard(x, group).numpy()
        arrays[f"hadamard.g{group}.y64"] = rotate_hadamard(x.double(), group).numpy()
    meta["effective_group_size"] = [
        [width, req, effective_group_size(width, req)]
        for width, req in [(48, 256), (17, 256), (3072, 256), (12288, 256), (1000, 256), (1024, 512),
                           (96, 64), (5, 4), (256, 1), (24, 8)]
    ]
    for name, dtype, width, out_f, group in [("convrot_f32", torch.float32, 256, 37, 256),
                                            ("convrot_bf16", torch.bfloat16, 256, 37, 64),
                                            ("convrot_g16", torch.float32, 48, 8, 256)]:
        torch.manual_seed(91)
        base = nn.Linear(width, out_f).to(dtype).requires_grad_(False)
        module = FrozenConvRotLinear(base, group)
        arrays[f"{name}.w"] = to_np(base.weight.float())
        arrays[f"{name}.bias"] = to_np(base.bias.float())
        arrays[f"{name}.rotated"] = rotate_hadamard(base.weight.detach().float(), module.group_size).numpy()
        arrays[f"{name}.q"] = module.weight_int8.numpy()
        arrays[f"{name}.s"] = module.weight_scale.numpy()
        tokens = torch.randn(2, 5, width).to(dtype).requires_grad_(True)
        out = module(tokens)
        grad = torch.randn_like(out)
        out.backward(grad)
        arrays[f"{name}.x"] = to_np(tokens.float())
        arrays[f"{name}.y"] = to_np(out.float())
        arrays[f"{name}.dy"] = to_np(grad.float())
        arrays[f"{name}.dx"] = to_np(tokens.grad.float())
        meta["cases"][name] = {"dtype": str(dtype).split(".")[-1], "group": module.group_size,
                               "rotation_group_size": int(module.rotation_group_size.item())}

    # ---------------------------------------------------------------- Comfy int8_tensorwise
    from training.comfy_weights import decode_comfy_state  # noqa: E402

    meta["comfy"] = {}
    for name, rows, cols, fields, dtype in COMFY_CASES:
        codes, scale = comfy_codes(rows, cols, seed=len(meta["comfy"]) + 700)
        state = {"layer.weight": codes, "layer.weight_scale": scale, "layer.comfy_quant": comfy_marker(fields),
                 "layer.bias": torch.linspace(-1, 1, rows), "norm.num_batches_tracked": torch.tensor(9)}
        dense = decode_comfy_state(state, dtype)
        arrays[f"{name}.codes"] = codes.numpy()
        arrays[f"{name}.scale"] = scale.numpy()
        arrays[f"{name}.dense"] = dense["layer.weight"].to(torch.float64).numpy()
        meta["comfy"][name] = {"fields": fields, "dtype": str(dtype).split(".")[-1],
                               "keys": sorted(dense), "bias_dtype": str(dense["layer.bias"].dtype).split(".")[-1],
                               "counter_dtype": str(dense["norm.num_batches_tracked"].dtype).split(".")[-1]}
    # a table wide enough to be decoded in several row chunks: hashes only
    codes, scale = comfy_codes(600, 8192, seed=799)
    fields = {"format": "int8_tensorwise", "convrot": True, "convrot_groupsize": 256}
    dense = decode_comfy_state({"embed.weight": codes, "embed.weight_scale": scale,
                                "embed.comfy_quant": comfy_marker(fields)}, torch.bfloat16)["embed.weight"]
    meta["comfy_chunked"] = {"rows": 600, "cols": 8192, "seed": 799, "fields": fields,
                             "codes_sha": sha(codes.numpy()), "dense_bf16_sha": sha(dense.view(torch.int16).numpy())}
    meta["comfy_errors"] = {}
    for label, mutate in comfy_mutations().items():
        state = comfy_fixture()
        mutate(state)
        try:
            decode_comfy_state(state)
        except ValueError as error:
            meta["comfy_errors"][label] = str(error)
        else:
            raise AssertionError(f"reference accepted the malformed case {label}")

    np.savez_compressed(HERE / "golden.npz", **arrays)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    print(f"wrote {len(arrays)} arrays, {len(meta['quant_hash'])} hashed shapes")


if __name__ == "__main__":
    main()

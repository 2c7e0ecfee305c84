"""Pins the CPU oracle against golden vectors produced by the reference implementation.

The goldens come from tests/golden/make_golden.py, which imports the reference's own
training/quantization.py and training/activation_offload.py. Everything here runs on CPU.
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from oracle import oracle as O


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


QUANT_CASES = ["q_70x37_f32", "q_64x32_zero_row", "q_96x40_bf16", "q_48x24_f16", "q_ties"]


@pytest.mark.parametrize("name", QUANT_CASES)
def test_oracle_quantiser_matches_reference_codes_and_scales(golden_arrays, name):
    w = golden_arrays[f"{name}.w"]
    q_c, s_c, nonfinite = O.quantize(w)
    q_np, s_np = O.quantize_np(w)
    assert not nonfinite
    np.testing.assert_array_equal(q_c, golden_arrays[f"{name}.q"])
    np.testing.assert_array_equal(s_c.view(np.uint32), golden_arrays[f"{name}.s"].view(np.uint32))
    np.testing.assert_array_equal(q_np, golden_arrays[f"{name}.q"])
    np.testing.assert_array_equal(s_np.view(np.uint32), golden_arrays[f"{name}.s"].view(np.uint32))


def test_half_to_even_ties_and_zero_rows(golden_arrays):
    q = golden_arrays["q_ties.q"]
    s = golden_arrays["q_ties.s"]
    assert q[0].tolist() == [127, 2, 4, -2, 0, 0, 2, 126]
    assert s[1] == 1.0 and not q[1].any()


def test_oracle_flags_non_finite_weights():
    w = np.ones((3, 5), np.float32)
    w[1, 2] = np.inf
    assert O.quantize(w)[2]
    w[1, 2] = np.nan
    assert O.quantize(w)[2]


@pytest.mark.parametrize("shape", [(3072, 3072), (12288, 3072), (3072, 12288), (18432, 3072)])
def test_oracle_quantiser_matches_reference_hashes_at_baseline_shapes(golden_meta, shape):
    import torch

    out_f, in_f = shape
    for dtype in ("float32", "bfloat16"):
        gen = torch.Generator().manual_seed(0)
        w = (torch.randn(out_f, in_f, generator=gen) * 0.02).to(getattr(torch, dtype)).float().numpy()
        expected = golden_meta["quant_hash"][f"{out_f}x{in_f}:{dtype}"]
        assert sha(w) == expected["weight_sha256"]
        q, s, _ = O.quantize(w)
        assert sha(q) == expected["codes_sha256"]
        assert sha(s) == expected["scale_sha256"]


@pytest.mark.parametrize("name", ["lin_70x37_bf16", "lin_256x320_bf16", "lin_160x96_f16"])
def test_oracle_gemms_match_reference_eager_outputs(golden_arrays, golden_meta, name):
    case = golden_meta["cases"][name]
    kind = O.KIND_OF[case["dtype"]]
    x = golden_arrays[f"{name}.x"].reshape(-1, golden_arrays[f"{name}.x"].shape[-1])
    q, s = golden_arrays[f"{name}.q"], golden_arrays[f"{name}.s"]
    bias = golden_arrays.get(f"{name}.bias")
    y_ref = golden_arrays[f"{name}.y"].reshape(x.shape[0], -1)
    y = O.round_kind(O.gemm_fwd(x, q, s, w_kind=kind, v_kind=kind, bias=bias).astype(np.float32), kind)
    # the reference rounds once per GEMM; only the accumulation order differs
    assert O.rel_fro(y, y_ref) < 5e-3
    dy = golden_arrays[f"{name}.dy"].reshape(x.shape[0], -1)
    dx_ref = golden_arrays[f"{name}.dx"].reshape(x.shape[0], -1)
    dx = O.round_kind(O.gemm_dx(dy, q, s, w_kind=kind, v_kind=kind).astype(np.float32), kind)
    assert O.rel_fro(dx, dx_ref) < 5e-3


@pytest.mark.parametrize("base", ["bfloat16", "float32"])
def test_oracle_reproduces_the_bit_exact_decode_and_bias_kat(golden_arrays, golden_meta, base):
    name = f"kat_{base}"
    case = golden_meta["cases"][name]
    w_kind = O.KIND_OF[case["base_dtype"]]
    v_kind = O.KIND_OF[case["out_dtype"]]
    q, s = golden_arrays[f"{name}.q"], golden_arrays[f"{name}.s"]
    y = O.round_kind(
        O.gemm_fwd(golden_arrays[f"{name}.x"], q, s, w_kind=w_kind, v_kind=v_kind,
                   bias=golden_arrays[f"{name}.bias"]).astype(np.float32), v_kind)
    np.testing.assert_array_equal(y, golden_arrays[f"{name}.y"])
    dx = O.round_kind(O.gemm_dx(golden_arrays[f"{name}.dy"], q, s, w_kind=w_kind, v_kind=v_kind).astype(np.float32),
                      v_kind)
    np.testing.assert_array_equal(dx, golden_arrays[f"{name}.dx"])


def test_kat_distinguishes_decode_roundings(golden_arrays):
    """bf16(s)*bf16(q) (reference) differs from bf16(f32(s*q)) for this scale."""
    s = np.float32(0.0002928110350837356)
    ref = O.round_bf16(np.float32(83) * O.round_bf16(np.array([s]))[0])
    alt = O.round_bf16(np.array([np.float32(83) * s]))
    assert ref != alt


def test_oracle_offload_view_matches_reference(golden_meta):
    for case in golden_meta["offload_view"]:
        got = O.offload_view(tuple(case["shape"]), tuple(case["stride"]))
        expected = None if case["payload_shape"] is None else tuple(case["payload_shape"])
        assert got == expected, case["name"]
    assert O.offload_view((5,), (-1,)) is None


def test_oracle_gather_packs_padded_view_densely():
    storage = np.arange(64, dtype=np.float32)
    payload = O.gather(storage, 4, (1, 1, 5, 5), (64, 64, 8, 1))
    expected = storage.reshape(8, 8)[:5, :5].copy().tobytes()
    assert payload == expected

"""ConvRot rotation: the eager restatement and the CPU oracle against the reference's outputs.

The golden arrays come from the reference's ``training.convrot`` (tests/golden/make_golden.py):
``rotate_hadamard`` in f32 and f64 for every group size up to 512 and the answers of
``effective_group_size``. No GPU is needed here.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200.convrot import effective_group_size, rotate_hadamard
from oracle import oracle as O

GROUPS = [1, 2, 4, 8, 16, 32, 64, 128, 256, 512]


@pytest.mark.parametrize("group", GROUPS)
def test_eager_rotation_is_bit_exact_with_the_reference(golden_arrays, group):
    """The weight rotation used at quantisation time repeats the reference's expressions in
    the same order, so rotated weights (and therefore int8 codes) are identical."""
    x = torch.from_numpy(golden_arrays[f"hadamard.g{group}.x"])
    np.testing.assert_array_equal(rotate_hadamard(x, group).numpy(), golden_arrays[f"hadamard.g{group}.y32"])
    np.testing.assert_array_equal(rotate_hadamard(x.double(), group).numpy(), golden_arrays[f"hadamard.g{group}.y64"])


@pytest.mark.parametrize("group", GROUPS)
def test_oracle_rotation_matches_the_reference_to_float_precision(golden_arrays, group):
    """The oracle restates the reference's staged GPU transform (f32 per stage); it agrees
    with the reference's f64 rotation to f32 rounding."""
    x = golden_arrays[f"hadamard.g{group}.x"]
    expected = golden_arrays[f"hadamard.g{group}.y64"]
    actual = O.hadamard(x, group, O.F32)
    assert np.max(np.abs(actual - expected)) <= 4e-7 * max(1.0, np.log2(group)) * np.max(np.abs(expected))


def test_regular_h4_convention_and_self_inverse():
    regular = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float32) / 2
    np.testing.assert_array_equal(O.hadamard(np.eye(4, dtype=np.float32), 4, O.F32), regular)
    np.testing.assert_array_equal(rotate_hadamard(torch.eye(4), 4).numpy(), regular)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((5, 1024)).astype(np.float32)
    for group in (2, 8, 32, 1024):
        twice = O.hadamard(O.hadamard(x, group, O.F32), group, O.F32)
        assert np.max(np.abs(twice - x)) < 1e-5


def test_per_stage_rounding_to_bf16():
    """Every stage's output is a bf16 value, as the reference stores each stage in the tensor dtype."""
    rng = np.random.default_rng(3)
    x = O.round_kind(rng.standard_normal((4, 256)).astype(np.float32), O.BF16)
    y = O.hadamard(x, 256, O.BF16)
    np.testing.assert_array_equal(y, O.round_kind(y, O.BF16))
    assert O.rel_fro(y, O.hadamard(x, 256, O.F32)) < 1e-2


def test_effective_group_size_matches_the_reference(golden_meta):
    for width, requested, expected in golden_meta["effective_group_size"]:
        assert effective_group_size(width, requested) == expected
    with pytest.raises(ValueError, match="positive"):
        effective_group_size(16, 0)
    with pytest.raises(ValueError, match="positive"):
        effective_group_size(0, 4)
    with pytest.raises(ValueError, match="power of two"):
        rotate_hadamard(torch.zeros(2, 12), 3)
    with pytest.raises(ValueError, match="divisible"):
        rotate_hadamard(torch.zeros(2, 12), 8)


def test_rotation_entry_point_validates_arguments_without_a_gpu():
    lib = _lib.library()
    assert lib.moss_hadamard_rotate(None, 1, 4, 12, 3, None, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert "power of two" in _lib.last_error()
    assert lib.moss_hadamard_rotate(None, 1, 4, 12, 8, None, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert "divisible" in _lib.last_error()
    assert lib.moss_hadamard_rotate(None, 1, 1, 16384, 16384, None, None) == _lib.MOSS_ERR_UNSUPPORTED
    assert lib.moss_hadamard_rotate(None, 7, 1, 8, 8, None, None) == _lib.MOSS_ERR_UNSUPPORTED
    assert lib.moss_hadamard_rotate(None, 1, 0, 8, 8, None, None) == _lib.MOSS_OK

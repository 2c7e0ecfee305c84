"""The C-ABI library loads without a GPU and exports every symbol include/moss_w8.h declares."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from moss_image_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "moss_w8.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moss_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_entry_points():
    names = declared_functions()
    for required in ("moss_w8_quantize", "moss_w8a16_gemm_fwd", "moss_w8a16_gemm_dx", "moss_offload_pack",
                     "moss_offload_prefetch", "moss_offload_wait", "moss_strided_gather"):
        assert required in names


def test_library_exports_every_declared_symbol():
    lib = _lib.library()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_exported_dynamic_symbols_are_exactly_the_c_abi():
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    moss = {name for name in exported if name.startswith("moss_")}
    assert moss == set(declared_functions())


def test_version_and_argument_validation_need_no_gpu():
    lib = _lib.library()
    assert lib.moss_version() >= 100
    rc = lib.moss_w8_quantize(None, 7, 4, 4, None, None, None, None)
    assert rc == _lib.MOSS_ERR_UNSUPPORTED
    assert "dtype" in _lib.last_error()
    rc = lib.moss_w8a16_gemm_fwd(None, 2, 4, 4, None, None, 1, 4, None, 0, None, None, 0, 0, 1.0, None, 1, None, 0,
                                 None, None)
    assert rc == _lib.MOSS_ERR_UNSUPPORTED  # f32 compute dtype is refused up front
    rc = lib.moss_strided_gather(None, 3, 1, (ctypes.c_int64 * 1)(4), (ctypes.c_int64 * 1)(1), None, None)
    assert rc in (_lib.MOSS_ERR_INVALID_ARGUMENT, _lib.MOSS_ERR_UNSUPPORTED)
    rc = lib.moss_offload_ring_create(0, 0, 0, None, None, ctypes.byref(ctypes.c_void_p()))
    assert rc == _lib.MOSS_ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError):
        _lib.check(rc, "moss_offload_ring_create")


def test_empty_problems_are_no_ops_without_device_work():
    lib = _lib.library()
    assert lib.moss_w8a16_gemm_fwd(None, 1, 0, 16, None, None, 1, 8, None, 0, None, None, 0, 0, 1.0, None, 1,
                                   None, 0, None, None) == _lib.MOSS_OK
    assert lib.moss_w8a16_gemm_dx(None, 1, 0, 8, None, None, 1, 16, None, None, 0, 0, 1.0, None, 1,
                                  None, 0, None, None) == _lib.MOSS_OK
    size = ctypes.c_size_t(123)
    assert lib.moss_w8a16_gemm_workspace_bytes(0, 8, 16, ctypes.byref(size)) == _lib.MOSS_OK and size.value == 0
    assert lib.moss_w8_quantize(None, 1, 0, 16, None, None, None, None) == _lib.MOSS_OK


def _sm_count() -> int:
    """SMs the library plans for: the device's count, or 148 (B200) when no GPU is visible."""
    import torch

    if torch.cuda.is_available():
        return torch.cuda.get_device_properties(0).multi_processor_count
    return 148


def _expected_pair_tail_bytes(m: int, n_out: int, k_red: int, sms: int) -> int:
    """The CTA-pair kernel's last-round split, restated: tiles of 256 x 256, one tile per SM
    pair per round; the tiles of a partly empty last round are cut along K into as many
    units as the idle pairs allow (at most 16, each at least one load step of two 64-wide
    k-blocks), when that saves at least 8 load steps. Scratch: one f32 256 x 256 partial
    per unit."""
    tiles = -(-m // 256) * -(-n_out // 256)
    pairs = sms // 2
    steps = -(-(-(-k_red // 64)) // 2)
    tail = tiles % pairs
    if tail == 0:
        return 0
    splits = min(pairs // tail, steps, 16)
    if splits < 2 or steps - -(-steps // splits) < 8:
        return 0
    return tail * splits * 256 * 256 * 4


@pytest.mark.parametrize("m,n_out,k_red", [
    (2048, 3072, 3072),    # 96 tiles: 22 in the last round of 74 pairs, split 3 ways
    (8192, 3072, 3072),    # 384 tiles: 14 left over, split 5 ways
    (8192, 18432, 3072),   # 2304 tiles: 10 left over, split 7 ways
    (9216, 3072, 3072),    # 432 tiles: 62 left over, no room to split
    (9216, 12288, 3072),   # 1728 tiles: 26 left over, split twice saves 12 steps
    (1900, 2900, 1088),    # ragged tiles, 9 load steps: three splits save only 6
    (1000, 4800, 1088),    # 76 tiles: 2 left over, split 9 ways = one load step per unit
    (1024, 3072, 256),     # 48 tiles in one round: 2 load steps, nothing to gain
])
def test_pair_last_round_split_workspace_plan(m, n_out, k_red):
    """The workspace query reports the CTA-pair kernel's last-round split scratch, computed
    on the host without touching a GPU."""
    size = ctypes.c_size_t(123)
    lib = _lib.library()
    assert lib.moss_w8a16_gemm_workspace_bytes(m, n_out, k_red, ctypes.byref(size)) == _lib.MOSS_OK
    assert size.value == _expected_pair_tail_bytes(m, n_out, k_red, _sm_count())


def test_pair_last_round_split_plan_matches_its_restatement_on_random_shapes():
    """Random CTA-pair shapes (more than 128 rows, enough tiles to fill half the SMs): the
    library's workspace query equals the restated plan for every one."""
    import random

    rng = random.Random(7)
    lib = _lib.library()
    sms = _sm_count()
    checked = 0
    while checked < 400:
        m = rng.randint(129, 40000)
        n_out = rng.randint(1, 24000)
        k_red = 64 * rng.randint(1, 400)
        if -(-m // 256) * -(-n_out // 256) * 4 < sms:
            continue  # too few pair tiles: another kernel serves it
        size = ctypes.c_size_t(123)
        assert lib.moss_w8a16_gemm_workspace_bytes(m, n_out, k_red, ctypes.byref(size)) == _lib.MOSS_OK
        assert size.value == _expected_pair_tail_bytes(m, n_out, k_red, sms), (m, n_out, k_red)
        checked += 1

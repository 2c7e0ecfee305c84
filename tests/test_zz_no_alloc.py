"""The allocation-free forward GEMM, moss_w8a16_gemm_fwd_noalloc.

The no-alloc entry point serves callers that cannot allocate device memory on this path: a
host whose HBM belongs to another allocator, or an FFI caller with no device allocator to
pass a workspace from. Its split scratch is a fixed array inside the library, shared by
every call on a device. These tests call it through the C ABI on problems that use that
scratch: few-row problems that split the reduction, and a CTA-pair problem whose last
round of tiles is split along K. Each output is checked against the CPU oracle (the
fp64-accumulated restatement of the reference GEMM, training/quant_kernels.py:125-158) and
against moss_w8a16_gemm_fwd with a caller workspace, twice in a row, so that the second pass
runs over the first pass's leftover scratch. The file name sorts last so that pytest also
runs it after all other GPU tests in the same process; it passes alone in a fresh process
as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from moss_image_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3  # the GEMM parity bar of the other GPU tests
BF16 = 1

# (m, k, n, seed): two few-row split-K problems and one CTA-pair problem (3 x 25 tiles of
# 256 x 256 on 74 SM pairs: the 75th tile is split along K in the static array, ~2.4 MB).
PROBLEMS = [(4, 3072, 3072, 11), (32, 2048, 1280, 12), (768, 1088, 6400, 13)]


def _problem(m: int, k: int, n: int, seed: int, device: torch.device):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    w = torch.randn(n, k, generator=gen) * 0.02
    q, s, _ = O.quantize(w.numpy())
    bias = torch.randn(n, generator=gen).to(torch.bfloat16)
    return x.to(device), torch.from_numpy(q).to(device), torch.from_numpy(s).to(device), bias.to(device)


def _workspace_bytes(m: int, n: int, k: int) -> int:
    size = ctypes.c_size_t()
    _lib.check(_lib.library().moss_w8a16_gemm_workspace_bytes(m, n, k, ctypes.byref(size)), "workspace bytes")
    return size.value


def _fwd_with_workspace(x, q, scale, bias, status):
    """moss_w8a16_gemm_fwd with a caller workspace (allocated here by torch)."""
    m, k = x.shape
    n = q.shape[0]
    need = _workspace_bytes(m, n, k)
    owner = torch.empty(need + 256, dtype=torch.uint8, device=x.device)
    ws = (owner.data_ptr() + 255) // 256 * 256
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=x.device)
    rc = _lib.library().moss_w8a16_gemm_fwd(
        x.data_ptr(), BF16, m, k, q.data_ptr(), scale.data_ptr(), BF16, n, bias.data_ptr(), BF16, None, None, 0, 0,
        1.0, y.data_ptr(), BF16, ws, need, status.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "moss_w8a16_gemm_fwd")
    torch.cuda.synchronize(x.device)
    del owner
    return y


def _fwd_noalloc(x, q, scale, bias, y, status):
    m, k = x.shape
    n = q.shape[0]
    return _lib.library().moss_w8a16_gemm_fwd_noalloc(
        x.data_ptr(), BF16, m, k, q.data_ptr(), scale.data_ptr(), BF16, n, bias.data_ptr(), BF16, None, None, 0, 0,
        1.0, y.data_ptr(), BF16, status.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)


def _oracle_rows(x, q, scale, bias, rows):
    """Oracle output for a subset of rows (every tile row of the problem is represented)."""
    xs = x[rows].float().cpu().numpy()
    return O.gemm_fwd(xs, q.cpu().numpy(), scale.cpu().numpy(), w_kind=O.BF16, v_kind=O.BF16,
                      bias=bias.float().cpu().numpy())


def _rows(m: int) -> np.ndarray:
    return np.unique(np.concatenate([np.arange(0, m, max(1, m // 96)), [m - 1]]))


def test_noalloc_forward_matches_oracle_and_workspace_forward_on_two_calls_in_a_row(cuda_device):
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    for m, k, n, _ in PROBLEMS:
        need = _workspace_bytes(m, n, k)
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES, (m, k, n, need)
    inputs = [_problem(m, k, n, seed, cuda_device) for m, k, n, seed in PROBLEMS]
    expected = [_fwd_with_workspace(*args, status) for args in inputs]
    oracle = [_oracle_rows(*args, _rows(args[0].shape[0])) for args in inputs]
    for _ in range(2):  # the second pass runs over the first pass's leftover partials and counters
        outputs = []
        for x, q, scale, bias in inputs:
            y = torch.full((x.shape[0], q.shape[0]), float("nan"), dtype=torch.bfloat16, device=cuda_device)
            _lib.check(_fwd_noalloc(x, q, scale, bias, y, status), "moss_w8a16_gemm_fwd_noalloc")
            outputs.append(y)
        torch.cuda.synchronize(cuda_device)
        assert int(status.item()) == 0
        for y, ref, ora in zip(outputs, expected, oracle):
            assert torch.isfinite(y.float()).all()
            assert O.rel_fro(y.float().cpu().numpy(), ref.float().cpu().numpy()) <= REL_FRO_TOL
            sub = y[torch.from_numpy(_rows(y.shape[0])).to(cuda_device)].float().cpu().numpy()
            assert O.rel_fro(sub, ora) <= REL_FRO_TOL


def test_noalloc_pair_problem_beyond_the_array_runs_without_the_split(cuda_device):
    """A CTA-pair problem whose last-round split needs more than the static array runs the
    unsplit plan instead of being refused."""
    m, k, n = 2048, 3072, 3072
    need = _workspace_bytes(m, n, k)
    if need <= _lib.NOALLOC_SCRATCH_BYTES:
        pytest.fail(f"expected a last-round split beyond the static array for {m}x{k}x{n}, planned {need} bytes")
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    x, q, scale, bias = _problem(m, k, n, 14, cuda_device)
    y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
    _lib.check(_fwd_noalloc(x, q, scale, bias, y, status), "moss_w8a16_gemm_fwd_noalloc")
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0
    rows = _rows(m)
    sub = y[torch.from_numpy(rows).to(cuda_device)].float().cpu().numpy()
    assert O.rel_fro(sub, _oracle_rows(x, q, scale, bias, rows)) <= REL_FRO_TOL


def test_noalloc_forward_refuses_problems_beyond_the_static_scratch(cuda_device):
    candidates = [(64, 3072, 3072), (128, 12288, 3072), (64, 12288, 3072), (256, 12288, 3072), (32, 12288, 18432),
                  (128, 3072, 18432)]
    found = None
    for m, k, n in candidates:
        need = _workspace_bytes(m, n, k)
        if need > _lib.NOALLOC_SCRATCH_BYTES:
            found = (m, k, n, need)
            break
    assert found is not None, "no candidate few-row problem plans more split scratch than the static array"
    m, k, n, need = found
    rc = _lib.library().moss_w8a16_gemm_fwd_noalloc(
        None, BF16, m, k, None, None, BF16, n, None, 0, None, None, 0, 0, 1.0, None, BF16, None,
        torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == _lib.MOSS_ERR_INVALID_ARGUMENT
    message = _lib.last_error()
    assert "static array" in message and str(need) in message


def test_noalloc_forward_allocates_no_device_memory(cuda_device):
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    inputs = [_problem(m, k, n, seed, cuda_device) for m, k, n, seed in PROBLEMS]
    outputs = [torch.empty((x.shape[0], q.shape[0]), dtype=torch.bfloat16, device=cuda_device)
               for x, q, _, _ in inputs]
    for (x, q, scale, bias), y in zip(inputs, outputs):  # warm-up: module load and symbol lookup
        _lib.check(_fwd_noalloc(x, q, scale, bias, y, status), "moss_w8a16_gemm_fwd_noalloc")
    torch.cuda.synchronize(cuda_device)
    free_before, _ = torch.cuda.mem_get_info(cuda_device)
    for _ in range(3):
        for (x, q, scale, bias), y in zip(inputs, outputs):
            _lib.check(_fwd_noalloc(x, q, scale, bias, y, status), "moss_w8a16_gemm_fwd_noalloc")
    torch.cuda.synchronize(cuda_device)
    free_after, _ = torch.cuda.mem_get_info(cuda_device)
    assert free_after == free_before
    assert int(status.item()) == 0

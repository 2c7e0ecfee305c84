"""The allocation-free forward GEMM, moss_w8a16_gemm_fwd_noalloc, against moss_w8a16_gemm_fwd.

The no-alloc entry point serves callers that cannot allocate device memory on this path: a
host whose HBM belongs to another allocator, or an FFI caller with no device allocator to
pass a workspace from. Its split-K scratch is a fixed array inside the library, shared by
every call on a device. These tests call both entry points through the C ABI on few-row
problems (the ones that split the reduction and so use scratch) and compare the outputs,
twice in a row with different problems so that the second call runs over the first call's
leftover scratch. The file name sorts last so that pytest also runs it after all other GPU
tests in the same process; it passes alone in a fresh process as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from moss_image_b200 import _lib

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3  # the GEMM parity bar of the other GPU tests
BF16 = 1


def _rel_fro(a: torch.Tensor, b: torch.Tensor) -> float:
    a64, b64 = a.double().cpu().numpy(), b.double().cpu().numpy()
    return float(np.linalg.norm(a64 - b64) / max(np.linalg.norm(b64), 1e-30))


def _problem(m: int, k: int, n: int, seed: int, device: torch.device):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen).to(device, torch.bfloat16)
    q = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8).to(device)
    scale = (torch.rand(n, generator=gen) * 0.01 + 1e-3).to(device)
    bias = torch.randn(n, generator=gen).to(device, torch.bfloat16)
    return x, q, scale, bias


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


def test_noalloc_forward_matches_workspace_forward_on_two_calls_in_a_row(cuda_device):
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    # Two different split-K problems: the second runs over the first call's leftover partials
    # and counters in the shared static array.
    problems = [(4, 3072, 3072, 11), (32, 2048, 1280, 12)]
    for m, k, n, _ in problems:
        need = _workspace_bytes(m, n, k)
        assert 0 < need <= _lib.NOALLOC_SCRATCH_BYTES, (m, k, n, need)
    inputs = [_problem(m, k, n, seed, cuda_device) for m, k, n, seed in problems]
    expected = [_fwd_with_workspace(*args, status) for args in inputs]
    outputs = []
    for (x, q, scale, bias), (m, k, n, _) in zip(inputs, problems):
        y = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        _lib.check(_fwd_noalloc(x, q, scale, bias, y, status), "moss_w8a16_gemm_fwd_noalloc")
        outputs.append(y)
    torch.cuda.synchronize(cuda_device)
    assert int(status.item()) == 0
    for y, ref in zip(outputs, expected):
        assert torch.isfinite(y.float()).all()
        assert _rel_fro(y, ref) <= REL_FRO_TOL


def test_noalloc_forward_refuses_problems_beyond_the_static_scratch(cuda_device):
    m, k, n = 32, 3072, 18432
    need = _workspace_bytes(m, n, k)
    if need <= _lib.NOALLOC_SCRATCH_BYTES:
        pytest.skip(f"this GPU plans only {need} bytes of split-K scratch for {m}x{k}x{n}")
    rc = _lib.library().moss_w8a16_gemm_fwd_noalloc(
        None, BF16, m, k, None, None, BF16, n, None, 0, None, None, 0, 0, 1.0, None, BF16, None,
        torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == _lib.MOSS_ERR_INVALID_ARGUMENT
    message = _lib.last_error()
    assert "static array" in message and str(need) in message

"""The failure path of the GEMM kernels, exercised without a GPU fault.

A test hook (moss_debug_stall_next_gemm) makes the operand-swapped kernel's MMA issuer wait on
a barrier that nothing arrives on. That wait is bounded (about two seconds): the kernel then
sets MOSS_STATUS_TIMEOUT_MMA in the device status word and in its host-visible copy, every
role leaves its loop, the copies in flight are drained, TMEM is freed and the launch returns.
The tests check that the host sees the failure without synchronising the device, that the
product path (the launchers, the module, backward) raises instead of returning the garbage
result, and that the context stays usable: after a reset the same GEMM is bit-identical to a
run before the failure. Only the few-row kernel honours the hook; the CTA-pair kernel's
timeout path is not run on a GPU.
"""

from __future__ import annotations

import time

import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200 import quant_kernels as qk
from moss_image_b200.quantization import FrozenInt8Linear

pytestmark = pytest.mark.gpu

TIMEOUT_MMA = 0x4


def _problem(device):
    gen = torch.Generator(device=device).manual_seed(5)
    m, k, n = 64, 3072, 3072  # few rows: the operand-swapped kernel
    x = torch.randn(m, k, generator=gen, device=device).to(torch.bfloat16)
    q = torch.randint(-127, 128, (n, k), generator=gen, device=device, dtype=torch.int8)
    s = torch.rand(n, generator=gen, device=device) * 1e-3 + 1e-4
    return x, q, s


def _host_word(device) -> int:
    qk.status_buffer(device)
    return int(qk._status_mirrors[device.index if device.index is not None else torch.cuda.current_device()][0])


def test_timed_out_launch_is_reported_without_a_sync_and_the_context_recovers(cuda_device):
    x, q, s = _problem(cuda_device)
    qk.reset_device_status(cuda_device)
    before = qk.int8_linear_forward(x, q, s, None, torch.bfloat16, torch.bfloat16)
    torch.cuda.synchronize(cuda_device)
    assert _host_word(cuda_device) == 0

    _lib.check(_lib.library().moss_debug_stall_next_gemm(), "moss_debug_stall_next_gemm")
    start = time.monotonic()
    qk.int8_linear_forward(x, q, s, None, torch.bfloat16, torch.bfloat16)
    torch.cuda.synchronize(cuda_device)  # the launch returns: no CUDA error, no hang
    elapsed = time.monotonic() - start
    assert elapsed > 0.5, f"the stalled wait ended after {elapsed:.3f} s"
    # the host copy, read without touching the device: some timeout bit (roles that give up at
    # the same time write it without atomics, so which bit survives is not fixed)
    assert _host_word(cuda_device) & _lib.STATUS_TIMEOUT_MASK
    assert int(qk.status_buffer(cuda_device).item()) & TIMEOUT_MMA  # the device word is OR-ed atomically

    # every later GEMM call on the device raises until the failure is cleared
    with pytest.raises(RuntimeError, match="pipeline timeout"):
        qk.int8_linear_forward(x, q, s, None, torch.bfloat16, torch.bfloat16)
    module = FrozenInt8Linear.from_codes(q, s, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="pipeline timeout"):
        module(x)

    qk.reset_device_status(cuda_device)
    after = qk.int8_linear_forward(x, q, s, None, torch.bfloat16, torch.bfloat16)
    torch.cuda.synchronize(cuda_device)
    assert qk.check_device_status(cuda_device) == 0
    assert torch.equal(before, after)


def test_backward_raises_after_a_failed_launch(cuda_device):
    x, q, s = _problem(cuda_device)
    qk.reset_device_status(cuda_device)
    module = FrozenInt8Linear.from_codes(q, s, dtype=torch.bfloat16)
    tokens = x.clone().requires_grad_(True)
    _lib.check(_lib.library().moss_debug_stall_next_gemm(), "moss_debug_stall_next_gemm")
    out = module(tokens)  # this forward launch times out on the device
    torch.cuda.synchronize(cuda_device)
    with pytest.raises(RuntimeError, match="pipeline timeout"):
        out.float().sum().backward()
    qk.reset_device_status(cuda_device)
    tokens.grad = None
    module(tokens).float().sum().backward()
    torch.cuda.synchronize(cuda_device)
    assert qk.check_device_status(cuda_device) == 0
    assert torch.isfinite(tokens.grad.float()).all()


def test_the_hook_is_consumed_by_the_next_gemm_call_only(cuda_device):
    x, q, s = _problem(cuda_device)
    qk.reset_device_status(cuda_device)
    big = torch.randn(1024, 3072, device=cuda_device).to(torch.bfloat16)  # CTA-pair kernel: ignores the hook
    _lib.check(_lib.library().moss_debug_stall_next_gemm(), "moss_debug_stall_next_gemm")
    qk.int8_linear_forward(big, q, s, None, torch.bfloat16, torch.bfloat16)
    qk.int8_linear_forward(x, q, s, None, torch.bfloat16, torch.bfloat16)  # not stalled: consumed above
    torch.cuda.synchronize(cuda_device)
    assert qk.check_device_status(cuda_device) == 0


def test_status_copy_is_one_word_per_device(cuda_device):
    """moss_status_mirror returns one word per device, the same on every call."""
    import ctypes

    first = ctypes.POINTER(ctypes.c_int)()
    second = ctypes.POINTER(ctypes.c_int)()
    with torch.cuda.device(cuda_device):
        _lib.check(_lib.library().moss_status_mirror(ctypes.byref(first)), "mirror")
        _lib.check(_lib.library().moss_status_mirror(ctypes.byref(second)), "mirror")
    assert ctypes.addressof(first.contents) == ctypes.addressof(second.contents)

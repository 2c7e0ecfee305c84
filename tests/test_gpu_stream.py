"""Parity of the few-row weight-streaming kernel (M <= 16 rows, no LoRA term) with the oracle.

Covers the token counts on both sides of the kernel's one-tile/two-tile switch (8 rows),
ragged output features (forward), both 16-bit compute kinds, a weight dtype that differs from
the compute dtype (decode in f32), the bias, and the same problems with and without the
split-reduction workspace (with no workspace the kernel reduces in one CTA per tile). The
reference is the fp64-accumulated oracle (training/quant_kernels.py:125-158 forward,
:193-218 grad-input) at the north-star bar, relative Frobenius error 5e-3.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200 import quant_kernels as qk
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3
TORCH_OF = {O.F16: torch.float16, O.BF16: torch.bfloat16, O.F32: torch.float32}


def _problem(m, k, n, seed):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=gen)
    w = torch.randn(n, k, generator=gen) * 0.02
    q, s, _ = O.quantize(w.numpy())
    return x, q, s, gen


def _workspace(m, n_out, k_red, device):
    size = ctypes.c_size_t()
    _lib.check(_lib.library().moss_w8a16_gemm_workspace_bytes(m, n_out, k_red, ctypes.byref(size)), "workspace")
    if size.value == 0:
        return None, None, 0
    owner = torch.empty(size.value + 256, dtype=torch.uint8, device=device)
    return owner, (owner.data_ptr() + 255) // 256 * 256, size.value


@pytest.mark.parametrize("m", [1, 2, 3, 8, 9, 16])
@pytest.mark.parametrize("kind", [O.BF16, O.F16])
def test_forward_matches_the_oracle(cuda_device, m, kind):
    k, n = 1024, 520  # ragged feature count: the last 16-feature group is partial
    x, q, s, gen = _problem(m, k, n, seed=100 + m)
    bias = torch.randn(n, generator=gen)
    dt = TORCH_OF[kind]
    xd = x.to(dt).to(cuda_device)
    y = qk.int8_linear_forward(xd, torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device),
                               bias.to(dt).to(cuda_device), dt, dt)
    torch.cuda.synchronize()
    assert qk.check_device_status(cuda_device) & _lib.STATUS_TIMEOUT_MASK == 0
    expected = O.gemm_fwd(xd.float().cpu().numpy(), q, s, w_kind=kind, v_kind=kind, bias=bias.to(dt).float().numpy())
    assert O.rel_fro(y.float().cpu().numpy(), expected) <= REL_FRO_TOL


@pytest.mark.parametrize("m", [1, 2, 7, 8, 12, 16])
@pytest.mark.parametrize("kind", [O.BF16, O.F16])
def test_grad_input_matches_the_oracle(cuda_device, m, kind):
    k, n = 1024, 528  # 8 output strips of 128 columns, 33 reduction slabs of 16 rows
    _, q, s, gen = _problem(1, k, n, seed=200 + m)
    dy = torch.randn(m, n, generator=gen)
    dt = TORCH_OF[kind]
    dyd = dy.to(dt).to(cuda_device)
    dx = qk.int8_linear_backward(dyd, torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device),
                                 torch.Size((m, k)), dt, dt)
    torch.cuda.synchronize()
    assert qk.check_device_status(cuda_device) & _lib.STATUS_TIMEOUT_MASK == 0
    expected = O.gemm_dx(dyd.float().cpu().numpy(), q, s, w_kind=kind, v_kind=kind)
    assert O.rel_fro(dx.float().cpu().numpy(), expected) <= REL_FRO_TOL


def test_f32_module_decode_under_bf16_compute(cuda_device):
    """weight dtype f32, compute bf16 (autocast over an fp32 module): decode in f32, then round."""
    m, k, n = 4, 2048, 384
    x, q, s, gen = _problem(m, k, n, seed=7)
    xd = x.to(torch.bfloat16).to(cuda_device)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    y = qk.int8_linear_forward(xd, qd, sd, None, torch.bfloat16, torch.float32)
    dy = torch.randn(m, n, generator=gen).to(torch.bfloat16).to(cuda_device)
    dx = qk.int8_linear_backward(dy, qd, sd, torch.Size((m, k)), torch.float32, torch.float32,
                                 compute_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    ey = O.gemm_fwd(xd.float().cpu().numpy(), q, s, w_kind=O.F32, v_kind=O.BF16)
    edx = O.gemm_dx(dy.float().cpu().numpy(), q, s, w_kind=O.F32, v_kind=O.BF16)
    assert O.rel_fro(y.float().cpu().numpy(), ey) <= REL_FRO_TOL
    assert O.rel_fro(dx.float().cpu().numpy(), edx) <= REL_FRO_TOL
    assert dx.dtype == torch.float32


@pytest.mark.parametrize("direction", ["fwd", "dx"])
def test_split_and_unsplit_reductions_agree(cuda_device, direction):
    """The split plan (workspace given) and the one-CTA-per-tile plan (no workspace) give the
    same result up to f32 summation order, and each is deterministic across calls."""
    m, k, n = 2, 3072, 3072
    _, q, s, gen = _problem(1, k, n, seed=9)
    qd, sd = torch.from_numpy(q).to(cuda_device), torch.from_numpy(s).to(cuda_device)
    a = torch.randn(m, k if direction == "fwd" else n, generator=gen).to(torch.bfloat16).to(cuda_device)
    n_out, k_red = (n, k) if direction == "fwd" else (k, n)
    owner, ws, ws_bytes = _workspace(m, n_out, k_red, cuda_device)
    assert ws_bytes > 0, "expected a split plan for this shape"
    lib = _lib.library()
    status = qk.status_buffer(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    outs = []
    for use_ws in (True, True, False):
        out = torch.full((m, n_out), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        w_ptr, w_bytes = (ws, ws_bytes) if use_ws else (None, 0)
        if direction == "fwd":
            rc = lib.moss_w8a16_gemm_fwd(a.data_ptr(), 1, m, k, qd.data_ptr(), sd.data_ptr(), 1, n, None, 0, None, None,
                                         0, 0, 1.0, out.data_ptr(), 1, w_ptr, w_bytes, status.data_ptr(), stream)
        else:
            rc = lib.moss_w8a16_gemm_dx(a.data_ptr(), 1, m, n, qd.data_ptr(), sd.data_ptr(), 1, k, None, None, 0, 0,
                                        1.0, out.data_ptr(), 1, w_ptr, w_bytes, status.data_ptr(), stream)
        _lib.check(rc, direction)
        outs.append(out)
    torch.cuda.synchronize()
    del owner
    assert torch.equal(outs[0], outs[1])
    if direction == "fwd":
        expected = O.gemm_fwd(a.float().cpu().numpy(), q, s, w_kind=O.BF16, v_kind=O.BF16)
    else:
        expected = O.gemm_dx(a.float().cpu().numpy(), q, s, w_kind=O.BF16, v_kind=O.BF16)
    for out in (outs[0], outs[2]):
        assert torch.isfinite(out.float()).all()
        assert O.rel_fro(out.float().cpu().numpy(), expected) <= REL_FRO_TOL
    assert np.max(np.abs(outs[0].float().cpu().numpy() - outs[2].float().cpu().numpy())) <= 2.0 ** -6 * np.max(
        np.abs(expected))

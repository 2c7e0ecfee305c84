"""Parity on every GEMM shape the benchmark times, at full size, forward and grad-input.

The grid is the W8A16 sweep of the benchmark configuration (M in {128, 512, 2048, 8192,
32768} x (K, N) in {(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072),
(3072, 18432)}), plus the real MOSS block's fused up/gate projection 3072 -> 16384 and its
down projection 8192 -> 3072 (training/model.py:255-256), and the per-block adaLN rows of the
36-block step (2 x 3072 -> 18432). At M = 8192 and 32768 several of these shapes run the
CTA-pair kernel with its last round of tiles split along K; at M <= 512 they run the
operand-swapped kernel, split over K where its planner chooses.

The reference for each case is a float32 matmul (TF32 off) on the weight decoded with the
reference's own expression ``q.to(bf16) * scale.to(bf16)[:, None]``
(training/quantization.py:23-24); the bar is the north-star relative Frobenius error 5e-3,
computed in float64. The reference's own parity test is training/tests/test_quant_kernels.py:
61-82 (ragged shapes, 2e-2 elementwise); these cases are the same check at the sizes timed.
"""

from __future__ import annotations

import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200 import quant_kernels as qk

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3

SWEEP_M = [128, 512, 2048, 8192, 32768]
SWEEP_KN = [(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072), (3072, 18432)]
MOSS_SHAPES = [(m, 3072, 16384) for m in (2, 512, 4608, 9216)] + [(m, 8192, 3072) for m in (2, 512, 4608, 9216)]
STEP_SHAPES = [(2, 3072, 18432), (9216, 3072, 18432), (9216, 3072, 12288), (9216, 12288, 3072)]

CASES = [(m, k, n) for m in SWEEP_M for k, n in SWEEP_KN] + MOSS_SHAPES + STEP_SHAPES


def _problem(m: int, k: int, n: int, seed: int, device: torch.device):
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randint(-127, 128, (n, k), generator=gen, device=device, dtype=torch.int8)
    scale = torch.rand(n, generator=gen, device=device) * 4e-4 + 1e-4  # ~ N(0, 0.02) weights / 127
    return q, scale


def _rel_fro(actual: torch.Tensor, expected: torch.Tensor) -> float:
    num = 0.0
    den = 0.0
    # chunked so a [32768, 18432] comparison does not need a float64 copy of both operands
    for a, e in zip(actual.split(4096), expected.split(4096)):
        e64 = e.double()
        num += float((a.double() - e64).square().sum())
        den += float(e64.square().sum())
    return (num / max(den, 1e-300)) ** 0.5


@pytest.fixture(autouse=True)
def _no_tf32():
    allow = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = allow


@pytest.mark.parametrize("m,k,n", CASES, ids=[f"{m}x{k}x{n}" for m, k, n in CASES])
def test_forward_and_grad_input_against_fp32_matmul(cuda_device, m, k, n):
    q, scale = _problem(m, k, n, seed=m * 7 + k * 3 + n, device=cuda_device)
    decoded = (q.to(torch.bfloat16) * scale.to(torch.bfloat16)[:, None]).float()
    gen = torch.Generator(device=cuda_device).manual_seed(m + k + n)
    x = torch.randn(m, k, generator=gen, device=cuda_device).to(torch.bfloat16)
    y = qk.int8_linear_forward(x, q, scale, None, torch.bfloat16, torch.bfloat16)
    expected = x.float() @ decoded.t()
    err = _rel_fro(y, expected)
    del expected
    assert err <= REL_FRO_TOL, f"forward relative Frobenius error {err:.3e}"

    dy = torch.randn(m, n, generator=gen, device=cuda_device).to(torch.bfloat16)
    dx = qk.int8_linear_backward(dy, q, scale, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
    expected_dx = dy.float() @ decoded
    err_dx = _rel_fro(dx, expected_dx)
    torch.cuda.synchronize(cuda_device)
    assert qk.check_device_status(cuda_device) & _lib.STATUS_TIMEOUT_MASK == 0
    assert err_dx <= REL_FRO_TOL, f"grad-input relative Frobenius error {err_dx:.3e}"

"""ConvRot on the GPU: the one-pass rotation kernel and FrozenConvRotLinear, through the C ABI.

Rotation: bit-exact with the CPU oracle (the reference's staged transform, each stage rounded
to the tensor dtype). Module: int8 codes and scales bit-exact with the reference's module
(golden arrays); outputs and input gradients within the GEMM bar (relative Frobenius 5e-3)
of the oracle, and within the reference's own eager-vs-GPU tolerance of its eager outputs.
"""

from __future__ import annotations

import ctypes
import io

import numpy as np
import pytest
import torch
from torch import nn
from torch.nn import functional as F

from moss_image_b200 import _lib
from moss_image_b200 import quant_kernels as qk
from moss_image_b200.convrot import FrozenConvRotLinear, quantize_frozen_convrot_linears
from oracle import oracle as O

pytestmark = pytest.mark.gpu

REL_FRO_TOL = 5e-3
KIND = {torch.bfloat16: O.BF16, torch.float16: O.F16, torch.float32: O.F32}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("group", [1, 2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192])
def test_rotation_kernel_is_bit_exact_with_the_oracle(cuda_device, dtype, group):
    rows = 37
    cols = max(group, 256) * 2
    gen = torch.Generator().manual_seed(group)
    x = (torch.randn(rows, cols, generator=gen) * 3).to(dtype)
    expected = O.hadamard(_np(x), group, KIND[dtype])
    xd = x.to(cuda_device)
    y = qk.hadamard_transform(xd, group)
    np.testing.assert_array_equal(_np(y), expected)
    qk.hadamard_transform(xd, group, out=xd)  # in place
    np.testing.assert_array_equal(_np(xd), expected)


def test_rotation_kernel_handles_unaligned_and_ragged_views(cuda_device):
    base = torch.randn(5, 8 * 3 + 1, dtype=torch.bfloat16, device=cuda_device)
    view = base[:, 1:].contiguous()  # 24 columns: three groups of 8 per row, 16-byte accesses
    expected = O.hadamard(_np(view), 8, O.BF16)
    np.testing.assert_array_equal(_np(qk.hadamard_transform(view, 8)), expected)
    odd = torch.randn(3, 12, dtype=torch.float16, device=cuda_device)  # 12 columns: element accesses
    np.testing.assert_array_equal(_np(qk.hadamard_transform(odd, 4)), O.hadamard(_np(odd), 4, O.F16))
    with pytest.raises(ValueError, match="contiguous"):
        qk.hadamard_transform(base.t(), 1)


@pytest.mark.parametrize("name", ["convrot_f32", "convrot_bf16", "convrot_g16"])
def test_module_matches_the_reference_codes_and_oracle(cuda_device, golden_arrays, golden_meta, name):
    case = golden_meta["cases"][name]
    dtype = getattr(torch, case["dtype"])
    weight = torch.from_numpy(golden_arrays[f"{name}.w"]).to(dtype)
    bias = torch.from_numpy(golden_arrays[f"{name}.bias"]).to(dtype)
    base = nn.Linear(weight.shape[1], weight.shape[0]).to(dtype).requires_grad_(False)
    base.weight.copy_(weight)
    base.bias.copy_(bias)
    module = FrozenConvRotLinear(base.to(cuda_device), 256 if name != "convrot_bf16" else 64)
    assert module.group_size == case["group"] and int(module.rotation_group_size.item()) == case["rotation_group_size"]
    np.testing.assert_array_equal(module.weight_int8.cpu().numpy(), golden_arrays[f"{name}.q"])
    np.testing.assert_array_equal(module.weight_scale.cpu().numpy().view(np.uint32),
                                  golden_arrays[f"{name}.s"].view(np.uint32))
    # forward and input gradient in half precision (the GPU kernels' compute dtypes)
    v_dtype = torch.bfloat16
    v_kind = O.BF16
    module = module.to(v_dtype)
    x = torch.from_numpy(golden_arrays[f"{name}.x"]).to(v_dtype)
    xd = x.to(cuda_device).requires_grad_(True)
    y = module(xd)
    dy = torch.from_numpy(golden_arrays[f"{name}.dy"]).to(v_dtype)
    y.backward(dy.to(cuda_device))
    torch.cuda.synchronize()
    q, s = golden_arrays[f"{name}.q"], golden_arrays[f"{name}.s"]
    x2 = _np(x).reshape(-1, x.shape[-1])
    rotated = O.hadamard(x2, module.group_size, v_kind)
    expected_y = O.gemm_fwd(rotated, q, s, w_kind=v_kind, v_kind=v_kind, bias=O.round_kind(_np(bias), v_kind))
    assert O.rel_fro(_np(y).reshape(expected_y.shape), expected_y) <= REL_FRO_TOL
    dy2 = _np(dy).reshape(-1, dy.shape[-1])
    grad_rot = O.round_kind(O.gemm_dx(dy2, q, s, w_kind=v_kind, v_kind=v_kind), v_kind)
    expected_dx = O.hadamard(grad_rot, module.group_size, v_kind)
    assert O.rel_fro(_np(xd.grad).reshape(expected_dx.shape), expected_dx) <= REL_FRO_TOL
    # the reference's own eager outputs (its GPU test compares eager and Triton at 3e-2)
    np.testing.assert_allclose(_np(y), golden_arrays[f"{name}.y"], atol=3e-2, rtol=3e-2)
    np.testing.assert_allclose(_np(xd.grad), golden_arrays[f"{name}.dx"], atol=3e-2, rtol=3e-2)


def test_module_api_matches_the_reference_behaviour(cuda_device):
    torch.manual_seed(4)
    base = nn.Linear(256, 32).requires_grad_(False).to(cuda_device)
    quant = FrozenConvRotLinear(base).to(torch.bfloat16)
    x = torch.randn(2, 5, 256, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    actual = quant(x)
    expected = F.linear(x, quant.weight, quant.bias)  # the decoded weight in the unrotated basis
    assert O.rel_fro(_np(actual), _np(expected)) < 2e-2
    assert not list(quant.parameters())
    buffer = io.BytesIO()
    torch.save(quant.state_dict(), buffer)
    buffer.seek(0)
    state = torch.load(buffer, weights_only=True)
    assert state["weight_int8"].dtype == torch.int8 and state["rotation_group_size"].item() == 256
    clone = FrozenConvRotLinear(base).to(torch.bfloat16)
    clone.load_state_dict(state)
    assert torch.equal(clone(x), actual)
    with pytest.raises(RuntimeError, match="group size differs"):
        FrozenConvRotLinear(base, 16).load_state_dict(state)
    with pytest.raises(ValueError, match="Freeze"):
        FrozenConvRotLinear(nn.Linear(16, 4).to(cuda_device))
    model = nn.Sequential(nn.Linear(48, 8).requires_grad_(False), nn.Linear(8, 3)).to(cuda_device)
    assert quantize_frozen_convrot_linears(model) == ["0"]
    assert model[0].group_size == 16 and isinstance(model[1], nn.Linear)
    model.to(dtype=torch.bfloat16)
    assert model[0].compute_dtype == torch.bfloat16 and model[0].weight_scale.dtype == torch.float32


def test_large_rotation_and_gemm_shapes(cuda_device):
    """BASELINE-width activations: the rotation kernel over 512 x 3072 stays bit-exact and the
    ConvRot layer keeps the GEMM bar against rotating then multiplying with the oracle decode."""
    m, k, n = 512, 3072, 1024
    gen = torch.Generator().manual_seed(12)
    x = torch.randn(m, k, generator=gen).to(torch.bfloat16)
    np.testing.assert_array_equal(_np(qk.hadamard_transform(x.to(cuda_device), 256)), O.hadamard(_np(x), 256, O.BF16))
    base = nn.Linear(k, n, bias=False).requires_grad_(False)
    with torch.no_grad():
        base.weight.normal_(0.0, 0.02, generator=gen)
    module = FrozenConvRotLinear(base.to(cuda_device)).to(torch.bfloat16)
    y = module(x.to(cuda_device))
    torch.cuda.synchronize()
    q, s = module.weight_int8.cpu().numpy(), module.weight_scale.cpu().numpy()
    expected = O.gemm_fwd(O.hadamard(_np(x), 256, O.BF16), q, s, w_kind=O.BF16, v_kind=O.BF16)
    assert O.rel_fro(_np(y), expected) <= REL_FRO_TOL


def test_lora_over_a_convrot_base_adds_the_update_to_the_rotated_product(cuda_device):
    """A LoRA adapter wrapping a ConvRot layer (the reference injects LoRA before quantising)
    sees the unrotated input: y = (x H) dec(W H)^T + scale (x A^T) B^T."""
    from moss_image_b200.lora import LoRALinear

    torch.manual_seed(21)
    base = nn.Linear(512, 192, bias=True).requires_grad_(False).to(cuda_device)
    lora = LoRALinear(base, 8, 16.0)
    with torch.no_grad():
        lora.lora_B.normal_(0.0, 0.05)
    lora.base = FrozenConvRotLinear(base, 128)
    lora = lora.to(cuda_device, torch.bfloat16)
    x = torch.randn(3, 40, 512, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = lora(x)
    y.float().square().sum().backward()
    with torch.no_grad():
        expected = (lora.base(x).float()
                    + lora.scale * (x.float() @ lora.lora_A.float().t()) @ lora.lora_B.float().t())
    assert O.rel_fro(_np(y), expected.cpu().numpy()) <= 1e-2
    assert lora.lora_A.grad is not None and torch.isfinite(lora.lora_A.grad).all()


def _dx_then_rotate(dy, q, s, k, group, out_dtype, device):
    """moss_w8a16_gemm_dx without a workspace (no last-round split) then moss_hadamard_rotate."""
    m, n = dy.shape
    out = torch.empty(m, k, dtype=out_dtype, device=device)
    status = qk.status_buffer(device)
    stream = torch.cuda.current_stream(device).cuda_stream
    lib = _lib.library()
    codes = {torch.bfloat16: 1, torch.float16: 0, torch.float32: 2}
    v = codes[dy.dtype]
    _lib.check(lib.moss_w8a16_gemm_dx(dy.data_ptr(), v, m, n, q.data_ptr(), s.data_ptr(), v, k, None, None, 0, 0, 1.0,
                                      out.data_ptr(), codes[out_dtype], None, 0, status.data_ptr(), stream), "dx")
    _lib.check(lib.moss_hadamard_rotate(out.data_ptr(), codes[out_dtype], m, k, group, out.data_ptr(), stream), "rot")
    return out


def _dx_rotated(dy, q, s, k, group, out_dtype, device, *, workspace=True):
    m, n = dy.shape
    out = torch.full((m, k), float("nan"), dtype=out_dtype, device=device)
    codes = {torch.bfloat16: 1, torch.float16: 0, torch.float32: 2}
    v = codes[dy.dtype]
    size = ctypes.c_size_t()
    lib = _lib.library()
    _lib.check(lib.moss_w8a16_gemm_workspace_bytes(m, k, n, ctypes.byref(size)), "ws")
    owner = torch.empty(size.value + 256, dtype=torch.uint8, device=device)
    ws = (owner.data_ptr() + 255) // 256 * 256 if workspace else None
    _lib.check(lib.moss_w8a16_gemm_dx_rotated(dy.data_ptr(), v, m, n, q.data_ptr(), s.data_ptr(), v, k, group,
                                              out.data_ptr(), codes[out_dtype], ws, size.value if workspace else 0,
                                              qk.status_buffer(device).data_ptr(),
                                              torch.cuda.current_stream(device).cuda_stream), "dx_rotated")
    torch.cuda.synchronize(device)
    del owner
    return out


@pytest.mark.parametrize("m,k,n,dtype,out_dtype", [
    (2048, 3072, 3072, torch.bfloat16, torch.bfloat16),   # CTA-pair kernel: rotation in the epilogue
    (2100, 3072, 1536, torch.bfloat16, torch.bfloat16),   # ragged last row tile
    (9216, 3072, 3072, torch.bfloat16, torch.bfloat16),   # the benchmark step's q/k/v/o grad-input shape
    (4608, 12288, 3072, torch.bfloat16, torch.bfloat16),  # MLP down-projection input gradient, K = 12288
    (2048, 3072, 3072, torch.float16, torch.float16),
    (2048, 3072, 3072, torch.bfloat16, torch.float32),    # fp32 input under bf16 compute: stages unrounded
    (64, 3072, 3072, torch.bfloat16, torch.bfloat16),     # few rows: GEMM, then the rotation kernel
])
def test_rotated_grad_input_equals_gemm_then_rotation_bit_for_bit(cuda_device, m, k, n, dtype, out_dtype):
    """H (dY dec(W H)) fused into the CTA-pair epilogue (group 256) equals the grad-input GEMM
    followed by the standalone rotation kernel (itself bit-exact with the oracle's staged
    transform, training/quant_kernels.py:231-277) exactly, and is within the GEMM bar of the
    oracle."""
    gen = torch.Generator(device=cuda_device).manual_seed(m + k + n)
    q = torch.randint(-127, 128, (n, k), generator=gen, device=cuda_device, dtype=torch.int8)
    s = torch.rand(n, generator=gen, device=cuda_device) * 4e-4 + 1e-4
    dy = torch.randn(m, n, generator=gen, device=cuda_device).to(dtype)
    expected = _dx_then_rotate(dy, q, s, k, 256, out_dtype, cuda_device)
    fused = m >= 2048 and out_dtype == dtype  # the CTA-pair epilogue rotates (never a split plan)
    for workspace in (True, False):
        got = _dx_rotated(dy, q, s, k, 256, out_dtype, cuda_device, workspace=workspace)
        if fused or not workspace:
            assert torch.equal(got.view(torch.int16 if out_dtype != torch.float32 else torch.int32),
                               expected.view(torch.int16 if out_dtype != torch.float32 else torch.int32))
        else:  # a split plan groups the f32 sums differently: last-bit differences of the GEMM output
            assert O.rel_fro(_np(got), _np(expected)) <= REL_FRO_TOL / 2
    assert qk.check_device_status(cuda_device) & _lib.STATUS_TIMEOUT_MASK == 0
    rows = torch.arange(0, m, max(1, m // 48), device=cuda_device)
    dec = (q.to(torch.bfloat16) * s.to(torch.bfloat16)[:, None]).float().cpu().numpy()
    ref = (dy[rows].float().cpu().numpy().astype(np.float64) @ dec.astype(np.float64))
    ref_rot = O.hadamard(ref.astype(np.float32), 256, O.F32)
    assert O.rel_fro(_np(got[rows]), ref_rot) <= REL_FRO_TOL


def test_convrot_module_backward_uses_the_rotated_grad_input(cuda_device):
    """The module's input gradient at a CTA-pair shape equals rotate(GEMM) bit for bit."""
    m, k, n = 2048, 3072, 1024
    gen = torch.Generator().manual_seed(31)
    base = nn.Linear(k, n, bias=False).requires_grad_(False)
    with torch.no_grad():
        base.weight.normal_(0.0, 0.02, generator=gen)
    module = FrozenConvRotLinear(base.to(cuda_device)).to(torch.bfloat16)
    x = torch.randn(m, k, generator=gen).to(cuda_device, torch.bfloat16).requires_grad_(True)
    g = torch.randn(m, n, generator=gen).to(cuda_device, torch.bfloat16)
    module(x).backward(g)
    expected = _dx_then_rotate(g, module.weight_int8, module.weight_scale, k, 256, torch.bfloat16, cuda_device)
    assert torch.equal(x.grad.view(torch.int16), expected.view(torch.int16))

"""Packed batches on the GPU: the segment conditioning kernels against the reference's
expansion-then-elementwise ops, variable-length attention against per-sequence attention,
and the packed int8 block stack against per-sample traversals (resident and streamed).

The oracle for the segment kernels is the reference's own composition
(training/model.py:288-312 with :752-772) evaluated by torch on the CPU in the same dtypes:
forward outputs and the token/branch gradients must be bit-identical; the per-sequence
condition gradients (summed in f32 here, in the condition dtype by the reference's
index_add) must agree with an f64 sum of the same per-token terms to within the condition
dtype's final rounding (relative to the largest sum: 8e-3 bf16, 1e-3 f16, 1e-5 f32).
"""

from __future__ import annotations

import copy

import pytest
import torch
from torch.nn import functional as F

from moss_image_b200.dit import SyntheticDiT, inject_lora
from moss_image_b200.memory import place_model
from moss_image_b200.packed import (
    condition_for_tokens,
    cumulative_lengths,
    modulation_sample_indices,
    scaled_attention_varlen,
    segment_gate,
    segment_modulate,
)
from moss_image_b200.quantization import quantize_frozen_linears

pytestmark = pytest.mark.gpu

CASES = [  # token dtype, condition dtype, lengths, dim
    (torch.bfloat16, torch.bfloat16, [5, 1, 130, 64], 96),
    (torch.float16, torch.float16, [33, 7], 3072),
    (torch.float32, torch.float32, [3, 9, 2], 40),
    (torch.bfloat16, torch.float32, [17, 20], 64),
    (torch.float32, torch.bfloat16, [8, 8, 8], 24),
    (torch.bfloat16, torch.bfloat16, [3, 4], 13),      # element path (dim % 8 != 0)
    (torch.bfloat16, torch.bfloat16, [9216], 3072),    # one long sequence, benchmark width
]


def _reference(tokens, modulation, index, kind, branch=None):
    """training/model.py:291-293 (modulate) and :302 (gate) on the given tensors."""
    if kind == "modulate":
        return tokens * (1 + condition_for_tokens(modulation[:, 1], index)) + condition_for_tokens(modulation[:, 0], index)
    return tokens + branch * condition_for_tokens(modulation[:, 2], index)


@pytest.mark.parametrize("kind", ["modulate", "gate"])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_segment_kernels_match_the_reference_composition(cuda_device, kind, case):
    token_dtype, cond_dtype, lengths, dim = CASES[case]
    gen = torch.Generator().manual_seed(case)
    total = sum(lengths)
    tokens = (torch.randn(1, total, dim, generator=gen) * 2).to(token_dtype)
    branch = torch.randn(1, total, dim, generator=gen).to(token_dtype)
    modulation = (torch.randn(len(lengths), 6, dim, generator=gen) * 0.5).to(cond_dtype)
    upstream = torch.randn(1, total, dim, generator=gen)
    cu = cumulative_lengths(lengths, torch.device("cpu"))
    index = modulation_sample_indices(modulation, tokens, cu)

    # reference on the CPU, with gradients
    ref_inputs = [t.clone().requires_grad_(True) for t in (tokens, branch, modulation)]
    expected = _reference(ref_inputs[0], ref_inputs[2], index, kind, ref_inputs[1])
    expected.backward(upstream.to(expected.dtype))

    dev = [t.to(cuda_device).requires_grad_(True) for t in (tokens, branch, modulation)]
    offsets = cu.to(cuda_device)
    if kind == "modulate":
        actual = segment_modulate(dev[0], dev[2][:, 1], dev[2][:, 0], offsets)
    else:
        actual = segment_gate(dev[0], dev[1], dev[2][:, 2], offsets)
    assert actual.dtype == expected.dtype
    assert torch.equal(actual.cpu(), expected.detach())
    actual.backward(upstream.to(actual.dtype).to(cuda_device))
    grad_index = 0 if kind == "modulate" else 1
    assert torch.equal(dev[grad_index].grad.cpu(), ref_inputs[grad_index].grad)
    if kind == "gate":
        assert torch.equal(dev[0].grad.cpu(), ref_inputs[0].grad)
    # condition gradients: an f64 sum of the reference's per-token terms
    out_dtype = expected.dtype
    dy = upstream.to(out_dtype)
    if kind == "modulate":
        terms = {1: (dy.float() * tokens.float()).to(out_dtype).to(cond_dtype), 0: dy.to(cond_dtype)}
    else:
        terms = {2: (dy.float() * branch.float()).to(out_dtype).to(cond_dtype)}
    rows = torch.zeros(total, dtype=torch.long) if index is None else index
    for column, term in terms.items():
        reference = torch.zeros(len(lengths), dim, dtype=torch.float64).index_add_(0, rows, term[0].double())
        got = dev[2].grad[:, column].double().cpu()
        scale = reference.abs().max().clamp_min(1e-30)
        tolerance = {torch.bfloat16: 8e-3, torch.float16: 1e-3, torch.float32: 1e-5}[cond_dtype]
        assert ((got - reference).abs().max() / scale).item() <= tolerance


def test_varlen_attention_matches_per_sequence_attention(cuda_device):
    torch.manual_seed(3)
    lengths = [130, 17, 1024, 64]
    total = sum(lengths)
    q, k, v = (torch.randn(1, 8, total, 128, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
               for _ in range(3))
    cu = cumulative_lengths(lengths, cuda_device)
    out = scaled_attention_varlen(q, k, v, cu)
    bounds = cu.tolist()
    expected = torch.cat([F.scaled_dot_product_attention(q[:, :, a:b], k[:, :, a:b], v[:, :, a:b])
                          for a, b in zip(bounds[:-1], bounds[1:])], dim=2)
    torch.testing.assert_close(out, expected, atol=2e-2, rtol=2e-2)
    out.float().square().sum().backward()
    assert q.grad is not None and torch.isfinite(q.grad).all()


def _int8_model(device) -> SyntheticDiT:
    torch.manual_seed(61)
    model = SyntheticDiT(depth=3, dim=256, heads=2, mlp_dim=512).to(device)
    with torch.no_grad():
        for parameter in model.parameters():
            parameter.normal_(0.0, 0.05)
    model = model.to(torch.bfloat16).requires_grad_(False)
    inject_lora(model, rank=4, alpha=8.0, a_std=0.05)
    with torch.no_grad():
        for name, parameter in model.named_parameters():
            if name.endswith("lora_B"):
                parameter.normal_(0.0, 0.05)
    quantize_frozen_linears(model)
    return model.train()


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


def _fp32_model(device) -> SyntheticDiT:
    torch.manual_seed(71)
    model = SyntheticDiT(depth=2, dim=64, heads=2, mlp_dim=128).to(device)
    with torch.no_grad():
        for parameter in model.parameters():
            parameter.normal_(0.0, 0.1)
    model.requires_grad_(False)
    inject_lora(model, rank=2, alpha=4.0, a_std=0.1)
    with torch.no_grad():
        for name, parameter in model.named_parameters():
            if name.endswith("lora_B"):
                parameter.normal_(0.0, 0.1)
    return model.to(device).train()


def test_packed_fp32_stack_matches_per_sample_traversals_tightly(cuda_device):
    """training/tests/test_packed_cuda.py:130-154 (sdpa, fp32): outputs and gradients within
    rtol 5e-5 / atol 5e-6 of one traversal per sample, with activation offload on."""
    packed_model = _fp32_model(cuda_device)
    serial_model = copy.deepcopy(packed_model)
    packed_model.activation_offload = serial_model.activation_offload = True
    gen = torch.Generator(device=cuda_device).manual_seed(6)
    samples = [torch.randn(n, 64, device=cuda_device, generator=gen) for n in (21, 5, 40)]
    times = torch.tensor([0.1, 0.6, 0.9], device=cuda_device)
    outputs = packed_model.forward_packed(samples, times)
    sum(out.square().mean() for out in outputs).backward()
    expected = [serial_model(sample[None], times[i:i + 1])[0] for i, sample in enumerate(samples)]
    sum(out.square().mean() for out in expected).backward()
    for out, ref in zip(outputs, expected):
        torch.testing.assert_close(out, ref, rtol=5e-5, atol=5e-6)
    grads = {n: p.grad for n, p in packed_model.named_parameters() if p.requires_grad}
    for name, parameter in serial_model.named_parameters():
        if parameter.requires_grad:
            torch.testing.assert_close(grads[name], parameter.grad, rtol=5e-5, atol=5e-6, msg=name)


def test_packed_int8_stack_matches_per_sample_traversals(cuda_device):
    """bf16 int8 stack with activation offload: the reference's bf16 bar is elementwise 4e-2;
    here outputs within 2e-2 and adapter gradients within 1e-1 relative Frobenius (the
    gradients are sums over all tokens of bf16 products, computed with different GEMM tilings
    and attention kernels on the two sides)."""
    packed_model = _int8_model(cuda_device)
    serial_model = copy.deepcopy(packed_model)
    packed_model.activation_offload = serial_model.activation_offload = True
    gen = torch.Generator(device=cuda_device).manual_seed(4)
    samples = [torch.randn(n, 256, device=cuda_device, generator=gen).to(torch.bfloat16) for n in (300, 77, 1024)]
    times = torch.tensor([0.1, 0.6, 0.9], device=cuda_device)
    outputs = packed_model.forward_packed(samples, times)
    sum(out.float().square().mean() for out in outputs).backward()
    expected = [serial_model(sample[None], times[i:i + 1])[0] for i, sample in enumerate(samples)]
    sum(out.float().square().mean() for out in expected).backward()
    for out, ref in zip(outputs, expected):
        assert _rel(out, ref) <= 2e-2
    grads = {n: p.grad for n, p in packed_model.named_parameters() if p.requires_grad}
    for name, parameter in serial_model.named_parameters():
        if parameter.requires_grad:
            assert _rel(grads[name], parameter.grad) <= 1e-1, name


def test_packed_streamed_stack_matches_resident(cuda_device):
    """training/tests/test_packed_cuda.py:200-230: a packed traversal through async-streamed
    blocks equals the resident one (sampling: bit-identical)."""
    resident = _int8_model(cuda_device).eval()
    streamed = copy.deepcopy(resident).eval()
    place_model(streamed, cuda_device, 3, block_swap_mode="async")
    gen = torch.Generator(device=cuda_device).manual_seed(5)
    samples = [torch.randn(n, 256, device=cuda_device, generator=gen).to(torch.bfloat16) for n in (129, 512)]
    times = torch.tensor([0.3, 0.8], device=cuda_device)
    with torch.no_grad():
        expected = resident.forward_packed(samples, times)
        actual = streamed.forward_packed(samples, times)
    for a, e in zip(actual, expected):
        assert torch.equal(a, e)
    place_model(streamed, torch.device("cpu"), 0)

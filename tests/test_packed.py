"""Packed variable-length batches on the CPU: attention isolation, backend handling, the
sequence bookkeeping drop-ins, packed-versus-serial parity of the block stack, and the
segment kernels' argument checks.

Restates training/tests/test_packed_features.py:101-209 for this library's stack.
"""

from __future__ import annotations

import copy

import pytest
import torch
from torch.nn import functional as F

from moss_image_b200 import _lib, packed
from moss_image_b200.dit import SyntheticDiT, inject_lora
from moss_image_b200.packed import (
    condition_for_tokens,
    cumulative_lengths,
    modulation_sample_indices,
    scaled_attention_varlen,
    validate_attention_backend,
)


def test_varlen_sdpa_isolates_examples():
    torch.manual_seed(32)
    query, key, value = (torch.randn(1, 2, 7, 8) for _ in range(3))
    cumulative = torch.tensor([0, 3, 7])
    actual = scaled_attention_varlen(query, key, value, cumulative, "sdpa")
    expected = torch.cat([F.scaled_dot_product_attention(query[:, :, a:b], key[:, :, a:b], value[:, :, a:b])
                          for a, b in ((0, 3), (3, 7))], dim=2)
    torch.testing.assert_close(actual, expected, rtol=1e-6, atol=1e-6)


def test_many_sequences_use_one_jagged_call_with_the_same_result():
    torch.manual_seed(6)
    lengths = tuple(int(n) for n in torch.randint(1, 9, (packed.VARLEN_LOOP_MAX_SEQUENCES + 8,)))
    total = sum(lengths)
    q, k, v = (torch.randn(total, 2, 8, requires_grad=True) for _ in range(3))
    offsets = cumulative_lengths(list(lengths), torch.device("cpu"))
    jagged = packed.varlen_attention(q, k, v, offsets, lengths)
    looped = torch.cat([F.scaled_dot_product_attention(a.transpose(0, 1)[None], b.transpose(0, 1)[None],
                                                       c.transpose(0, 1)[None])[0].transpose(0, 1)
                        for a, b, c in zip(q.split(lengths), k.split(lengths), v.split(lengths))])
    torch.testing.assert_close(jagged, looped, rtol=1e-6, atol=1e-6)
    jagged.square().sum().backward()
    assert torch.isfinite(q.grad).all()


def test_varlen_gradients_stay_inside_each_sequence():
    torch.manual_seed(5)
    query, key, value = (torch.randn(1, 2, 9, 8, requires_grad=True) for _ in range(3))
    out = scaled_attention_varlen(query, key, value, torch.tensor([0, 4, 9]))
    out[:, :, :4].sum().backward()
    assert torch.count_nonzero(query.grad[:, :, 4:]) == 0 and torch.count_nonzero(value.grad[:, :, 4:]) == 0
    assert torch.count_nonzero(value.grad[:, :, :4]) > 0


def test_varlen_flash_uses_packed_thd_layout(monkeypatch):
    calls = []

    def fake_flash(query, key, value, cu_q, cu_k, max_q, max_k, *, dropout_p, causal):
        calls.append((query.shape, cu_q.tolist(), max_q, dropout_p, causal))
        return value

    monkeypatch.setattr(packed, "validate_attention_backend", lambda *args, **kwargs: "flash_attn_2")
    monkeypatch.setattr(packed, "_flash_attn_function", lambda name: fake_flash)
    query, key, value = (torch.randn(1, 2, 7, 8) for _ in range(3))
    actual = scaled_attention_varlen(query, key, value, torch.tensor([0, 3, 7]), "flash_attn_2")
    assert calls == [((7, 2, 8), [0, 3, 7], 4, 0.0, False)]
    torch.testing.assert_close(actual, value)


def test_varlen_cudnn_and_malformed_boundaries_fail(monkeypatch):
    query = torch.randn(1, 2, 7, 8)
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        scaled_attention_varlen(query, query, query, torch.tensor([0, 3, 7]), "sdpa_cudnn")
    with monkeypatch.context() as patch:
        patch.setattr(packed, "validate_attention_backend", lambda *args, **kwargs: "sdpa_cudnn")
        with pytest.raises(ValueError, match="does not support packed"):
            scaled_attention_varlen(query, query, query, torch.tensor([0, 3, 7]), "sdpa_cudnn")
    with pytest.raises(ValueError, match="singleton packed batch"):
        scaled_attention_varlen(torch.randn(2, 2, 7, 8), *(torch.randn(2, 2, 7, 8) for _ in range(2)),
                                torch.tensor([0, 7]))
    for bad in (torch.tensor([1, 7]), torch.tensor([0, 6]), torch.tensor([0, 3, 3, 7]), torch.tensor([7])):
        with pytest.raises(ValueError):
            scaled_attention_varlen(query, query, query, bad)
    with pytest.raises(ValueError, match="attention backend must be one of"):
        validate_attention_backend("xformers")
    assert validate_attention_backend(" SDPA ") == "sdpa"
    with pytest.raises(ValueError, match="requires CUDA tensors"):
        validate_attention_backend("sdpa_cudnn", device="cpu")


def test_modulation_indices_and_conditions_match_the_reference_rules():
    modulation = torch.randn(3, 6, 4)
    tokens = torch.randn(1, 10, 4)
    cu = cumulative_lengths([2, 5, 3], torch.device("cpu"))
    assert cu.tolist() == [0, 2, 7, 10] and cu.dtype == torch.int64
    index = modulation_sample_indices(modulation, tokens, cu)
    assert index.tolist() == [0, 0, 1, 1, 1, 1, 1, 2, 2, 2]
    assert torch.equal(condition_for_tokens(modulation[:, 1], index)[0, 3], modulation[1, 1])
    assert modulation_sample_indices(torch.randn(1, 6, 4), tokens, None) is None
    assert condition_for_tokens(modulation[:1, 0], None).shape == (1, 1, 4)
    with pytest.raises(ValueError, match="one row per sequence"):
        modulation_sample_indices(modulation, tokens, cumulative_lengths([5, 5], torch.device("cpu")))


def _tiny() -> SyntheticDiT:
    torch.manual_seed(41)
    model = SyntheticDiT(depth=2, dim=32, heads=2, mlp_dim=64)
    with torch.no_grad():
        for parameter in model.parameters():
            parameter.normal_(0.0, 0.1)
    model.requires_grad_(False)
    inject_lora(model, rank=2, alpha=4.0, a_std=0.1)
    with torch.no_grad():
        for name, parameter in model.named_parameters():
            if name.endswith("lora_B"):
                parameter.normal_(0.0, 0.1)
    return model.train()


def test_packed_traversal_matches_per_sample_traversals():
    """One packed pass over samples of 7, 3 and 12 tokens gives each sample's own result
    and the same adapter gradients as three separate passes."""
    packed_model = _tiny()
    serial_model = copy.deepcopy(packed_model)
    torch.manual_seed(8)
    samples = [torch.randn(n, 32) for n in (7, 3, 12)]
    times = torch.tensor([0.2, 0.5, 0.9])
    outputs = packed_model.forward_packed(samples, times)
    sum(out.square().mean() for out in outputs).backward()
    expected = [serial_model(sample[None], times[i:i + 1])[0] for i, sample in enumerate(samples)]
    sum(out.square().mean() for out in expected).backward()
    for out, ref in zip(outputs, expected):
        torch.testing.assert_close(out, ref, rtol=3e-5, atol=3e-6)
    for (name, a), b in zip(packed_model.named_parameters(), serial_model.parameters()):
        if a.requires_grad:
            torch.testing.assert_close(a.grad, b.grad, rtol=5e-5, atol=5e-6, msg=name)
    with pytest.raises(ValueError, match="at least one sample"):
        packed_model.forward_packed([], times)


def test_packed_streamed_block_keeps_checkpoint_and_varlen_inputs():
    model = _tiny()
    model.gradient_checkpointing = False
    calls = []

    class Manager:
        def block(self, index, *inputs, forward_prefetch, backward_prefetch, checkpoint_block):
            calls.append((index, len(inputs), checkpoint_block, inputs[-1].tolist()))
            return model.layers[index](*inputs)

    model.blocks_to_swap = 1
    model.block_swap_manager = Manager()
    outputs = model.forward_packed([torch.randn(6, 32), torch.randn(5, 32)], torch.tensor([0.2, 0.7]))
    sum(out.square().mean() for out in outputs).backward()
    assert calls == [(1, 3, True, [0, 6, 11])]


def test_segment_entry_points_validate_arguments_without_a_gpu():
    lib = _lib.library()
    ok, invalid, unsupported = _lib.MOSS_OK, _lib.MOSS_ERR_INVALID_ARGUMENT, _lib.MOSS_ERR_UNSUPPORTED
    assert lib.moss_segment_modulate(None, 1, 0, 8, None, None, 1, 8, None, 1, None, None) == ok
    assert lib.moss_segment_modulate(None, 1, 4, 8, None, None, 1, 8, None, 1, None, None) == invalid
    assert lib.moss_segment_modulate(None, 1, 4, 8, None, None, 1, 4, None, 1, None, None) == invalid
    assert "cond_stride" in _lib.last_error()
    assert lib.moss_segment_modulate(None, 9, 4, 8, None, None, 1, 8, None, 1, None, None) == unsupported
    assert lib.moss_segment_gate(None, None, 1, 4, 8, None, 1, 8, None, 0, None, None) == invalid
    assert lib.moss_segment_modulate_bwd(None, None, 1, 4, 8, None, 1, 8, None, 1, None, None, None,
                                         None) == invalid
    assert lib.moss_segment_gate_bwd(None, None, 1, 4, 8, None, 1, 8, None, 1, None, None, None) == invalid
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        packed.segment_modulate(torch.zeros(2, 8), torch.zeros(1, 8), torch.zeros(1, 8),
                                torch.tensor([0, 2]))

"""CPU tests of the host-side API: validation strings, converters, offload selection logic.

Ports the CPU parts of training/tests/test_quant_kernels.py:16-58,
training/tests/test_quantization.py:67-71 and training/tests/test_packed_features.py:188-235.
No CUDA is initialised here.
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

from moss_image_b200 import activation_offload as ao
from moss_image_b200 import quant_kernels as qk
from moss_image_b200.quantization import FrozenInt8Linear, configure_quantized_backend, quantize_frozen_linears
from oracle import oracle as O


def test_backend_validation_messages():
    for backend in ("auto", "eager", "triton"):
        assert qk.validate_quantized_backend(backend) == backend
    with pytest.raises(ValueError, match="quantized backend must be auto, eager or triton."):
        qk.validate_quantized_backend("cuda")


def test_trainable_or_meta_bases_are_rejected_before_any_device_work():
    with pytest.raises(ValueError, match="Freeze"):
        FrozenInt8Linear(nn.Linear(4, 4))
    with pytest.raises(ValueError, match="Load the base weights"):
        FrozenInt8Linear(nn.Linear(4, 4, device="meta").requires_grad_(False))
    with pytest.raises(ValueError, match="auto, eager or triton"):
        FrozenInt8Linear(nn.Linear(4, 4).requires_grad_(False), backend="cuda")
    model = nn.Sequential(nn.Linear(4, 4))
    assert quantize_frozen_linears(model) == []
    assert configure_quantized_backend(model, "auto") == []


def test_quantisation_without_cuda_fails_loudly(monkeypatch):
    monkeypatch.setattr(torch.cuda, "is_available", lambda: False)
    with pytest.raises(RuntimeError, match="needs a CUDA device"):
        FrozenInt8Linear(nn.Linear(8, 5).requires_grad_(False))


def test_resolve_rejects_cpu_inputs_with_reference_style_message():
    tokens = torch.randn(2, 8)
    weight = torch.zeros(5, 8, dtype=torch.int8)
    scale = torch.ones(5)
    for backend in ("auto", "eager", "triton"):
        with pytest.raises(RuntimeError, match="quantized backend is unavailable.*not on CUDA"):
            qk.resolve_quantized_backend(backend, tokens, weight, scale)


def test_autocast_dtype_rule_is_cuda_only():
    t = torch.randn(2, 3)
    with torch.autocast("cpu", dtype=torch.bfloat16):
        assert qk.autocast_compute_dtype(t, torch.float32) == torch.float32


def test_offload_is_a_cpu_noop():
    """test_packed_features.py:188-198: no hooks on CPU, disabled, or without grad."""
    model = nn.Linear(4, 4)
    assert type(ao.activation_cpu_offload(model, True, torch.device("cpu"))).__name__ == "nullcontext"
    assert type(ao.activation_cpu_offload(model, False, torch.device("cuda"))).__name__ == "nullcontext"
    with torch.no_grad():
        assert type(ao.activation_cpu_offload(model, True, torch.device("cuda"))).__name__ == "nullcontext"
    assert not torch.cuda.is_initialized()


def test_offload_view_and_restore_match_reference_goldens(golden_meta):
    backing = torch.arange(4096, dtype=torch.float32)
    for case in golden_meta["offload_view"]:
        view = backing.as_strided(case["shape"], case["stride"])
        got = ao._offload_view(view)
        expected = None if case["payload_shape"] is None else tuple(case["payload_shape"])
        assert (None if got is None else got[1]) == expected, case["name"]
        if got is not None:
            source, payload_shape = got
            restored = ao._restore_layout(source.contiguous(), torch.device("cpu"), tuple(view.shape),
                                          tuple(view.stride()), payload_shape, non_blocking=False)
            assert restored.stride() == view.stride()
            torch.testing.assert_close(restored, view)
            assert O.gather(backing.numpy(), 4, payload_shape, tuple(view.stride()),
                            view.storage_offset()) == source.contiguous().numpy().tobytes()


def test_contiguity_helper():
    assert ao._c_contiguous((2, 3), (3, 1))
    assert ao._c_contiguous((3, 1, 4), (4, 999, 1))
    assert ao._c_contiguous((1, 5), (0, 1))
    assert not ao._c_contiguous((3, 4), (1, 3))
    assert not ao._c_contiguous((1, 1, 5, 5), (64, 64, 8, 1))

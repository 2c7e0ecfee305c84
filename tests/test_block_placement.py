"""Block placement without a GPU: validation before mutation, the synchronous CPU path, and
the native block stager's argument checks.

Reference behaviour: training/memory.py:22-36 (synchronous blocks), :367-421 (validation) and
the CPU-side cases of training/tests/test_async_memory.py:423-447.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from moss_image_b200 import _lib
from moss_image_b200.dit import SyntheticDiT, inject_lora
from moss_image_b200.memory import place_model


def _tiny(depth: int = 4) -> SyntheticDiT:
    torch.manual_seed(5)
    model = SyntheticDiT(depth=depth, dim=64, heads=2, mlp_dim=128)
    with torch.no_grad():
        for parameter in model.parameters():
            parameter.normal_(0.0, 0.05)
    return model


def _lora(depth: int = 4) -> SyntheticDiT:
    model = _tiny(depth).requires_grad_(False)
    inject_lora(model, rank=2, alpha=4.0, a_std=None)
    with torch.no_grad():
        for name, parameter in model.named_parameters():
            if name.endswith("lora_B"):
                parameter.normal_(0.0, 0.03)
    return model


def _trainables(model):
    return {name: p for name, p in model.named_parameters() if p.requires_grad}


def test_async_rejects_full_training_before_mutating_the_model():
    model = _tiny()
    ids = {name: id(p) for name, p in model.named_parameters()}
    with pytest.raises(ValueError, match="H2D-only.*frozen base weights"):
        place_model(model, torch.device("cuda"), 2, block_swap_mode="async")
    assert {name: id(p) for name, p in model.named_parameters()} == ids
    assert all(p.device.type == "cpu" for p in model.parameters())
    assert not hasattr(model, "block_swap_manager")


def test_async_rejects_cpu_unknown_mode_and_bad_counts_before_mutating_the_model():
    model = _lora()
    ids = {name: id(p) for name, p in _trainables(model).items()}
    with pytest.raises(ValueError, match="requires a CUDA device"):
        place_model(model, torch.device("cpu"), 2, block_swap_mode="async")
    with pytest.raises(ValueError, match="block_swap_mode must be 'sync' or 'async'"):
        place_model(model, torch.device("cpu"), 2, block_swap_mode="overlap")
    with pytest.raises(ValueError, match="between zero and the number of joint blocks"):
        place_model(model, torch.device("cpu"), 5)
    with pytest.raises(ValueError, match="between zero and the number of joint blocks"):
        place_model(model, torch.device("cpu"), -1)
    with pytest.raises(NotImplementedError, match="async_full"):
        place_model(model, torch.device("cuda"), 2, block_swap_mode="async_full")
    assert {name: id(p) for name, p in _trainables(model).items()} == ids
    assert not hasattr(model, "block_swap_manager")


def test_sync_swapped_blocks_match_resident_training_on_the_cpu():
    """Synchronous swapping runs each block from copies of its CPU masters under a checkpoint;
    gradients reach the masters and an optimizer step updates them in place."""
    resident = _lora().train()
    swapped = _lora().train()
    swapped.load_state_dict(resident.state_dict())
    place_model(resident, torch.device("cpu"), 0)
    place_model(swapped, torch.device("cpu"), 3)
    assert swapped.blocks_to_swap == 3 and swapped.block_swap_mode == "sync" and swapped.block_swap_manager is None
    optimizers = [torch.optim.AdamW(_trainables(m).values(), lr=1e-3) for m in (resident, swapped)]
    torch.manual_seed(9)
    tokens = torch.randn(2, 12, 64)
    t = torch.rand(2)
    for model, optimizer in zip((resident, swapped), optimizers):
        for _ in range(2):
            loss = model(tokens, t).square().mean()
            loss.backward()
        optimizer.step()
    for (name, first), second in zip(_trainables(resident).items(), _trainables(swapped).values()):
        torch.testing.assert_close(second.grad, first.grad, atol=1e-6, rtol=1e-5, msg=name)
        torch.testing.assert_close(second, first, atol=1e-6, rtol=1e-5, msg=name)
    resident.eval()
    swapped.eval()
    with torch.no_grad():
        torch.testing.assert_close(swapped(tokens, t, skip_layers=(1, 3)), resident(tokens, t, skip_layers=(1, 3)))


def test_block_stager_validates_arguments_without_a_gpu():
    lib = _lib.library()
    handle = ctypes.c_void_p()
    assert lib.moss_block_stager_create(0, 2, None, ctypes.byref(handle)) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert "copy stream" in _lib.last_error()
    assert lib.moss_block_stager_create(0, 0, 1, ctypes.byref(handle)) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_block_stager_create(0, 2, 1, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_block_stager_destroy(None, 0) == _lib.MOSS_OK
    slot = ctypes.c_int()
    assert lib.moss_block_stager_select(None, 0, None, 0, ctypes.byref(slot)) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_block_stager_stage(None, 0, 0, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_block_stager_lease(None, 0, None, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    assert lib.moss_block_stager_release(None, 0, -1, 0, None) == _lib.MOSS_ERR_INVALID_ARGUMENT
    block = ctypes.c_int64()
    assert lib.moss_block_stager_add_block(None, None, 0, ctypes.byref(block)) == _lib.MOSS_ERR_INVALID_ARGUMENT

"""Asynchronous frozen-block streaming on the GPU: streamed training and sampling match a fully
resident model, and the native stager's copies are byte-exact.

Mirrors training/tests/test_async_memory.py:135-447 on this library's block stack (the
reference's fixtures are tiny DiTs with 4 blocks and rank-2 adapters; here width 128, 2 heads,
MLP 256, 4 blocks). Tolerances are the reference's (fp32 2e-5/2e-3, bf16 4e-3/3e-2) for
training; sampling outputs must be bit-identical, because a streamed block runs the same
kernels on byte-identical copies of its frozen tensors.
"""

from __future__ import annotations

import copy
import ctypes
import gc

import numpy as np
import pytest
import torch
from torch import nn

from moss_image_b200 import _lib
from moss_image_b200.activation_offload import offload_ring
from moss_image_b200.convrot import quantize_frozen_convrot_linears
from moss_image_b200.dit import SyntheticDiT, inject_lora
from moss_image_b200.lora import LoRALinear
from moss_image_b200.memory import place_model
from moss_image_b200.quantization import quantize_frozen_linears

pytestmark = pytest.mark.gpu

DIM, HEADS, MLP, DEPTH = 128, 2, 256, 4


def _prepare(quantization: str, dtype: torch.dtype, device: torch.device) -> SyntheticDiT:
    """Build, cast, freeze, inject LoRA, quantise - the trainer's order (training/train.py:577-589)."""
    model = SyntheticDiT(depth=DEPTH, dim=DIM, heads=HEADS, mlp_dim=MLP).to(device)
    with torch.no_grad():
        for module in model.modules():
            if isinstance(module, nn.Linear):
                module.weight.normal_(0.0, 0.05)
                if module.bias is not None:
                    module.bias.normal_(0.0, 0.02)
    model = model.to(dtype).requires_grad_(False)
    inject_lora(model, rank=2, alpha=4.0, a_std=None)
    with torch.no_grad():
        for module in model.modules():
            if isinstance(module, LoRALinear):
                module.lora_B.normal_(std=0.03)
    if quantization == "int8":
        assert quantize_frozen_linears(model)
    elif quantization == "int8_convrot":
        assert quantize_frozen_convrot_linears(model, 64)
    return model


def _frozen_layer_tensors(model: nn.Module) -> dict[str, torch.Tensor]:
    tensors = {f"parameters.{n}": p for n, p in model.layers.named_parameters() if not p.requires_grad}
    tensors.update({f"buffers.{n}": b for n, b in model.layers.named_buffers()})
    return tensors


def _trainables(model: nn.Module) -> dict[str, nn.Parameter]:
    return {name: p for name, p in model.named_parameters() if p.requires_grad}


def _batches(device: torch.device, dtype: torch.dtype) -> list[tuple[torch.Tensor, torch.Tensor]]:
    return [(torch.randn(1, 20, DIM, device=device, dtype=dtype), torch.tensor([0.25], device=device)),
            (torch.randn(2, 13, DIM, device=device, dtype=dtype), torch.tensor([0.75, 0.5], device=device))]


def _step(model, optimizer, batches, *, autocast: bool):
    optimizer.zero_grad(set_to_none=True)
    outputs = []
    for tokens, t in batches:
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            output = model(tokens, t)
            loss = output.float().square().mean() / 2
        outputs.append(output.detach().cpu())
        loss.backward()
    params = _trainables(model)
    assert params and all(p.grad is not None and torch.isfinite(p.grad).all() for p in params.values())
    assert all(torch.count_nonzero(p.grad).item() > 0 for n, p in params.items() if n.endswith("lora_A"))
    gradients = {n: p.grad.detach().cpu().clone() for n, p in params.items()}
    optimizer.step()
    return outputs, gradients, {n: p.detach().cpu().clone() for n, p in params.items()}


def _assert_named_close(actual, expected, *, atol, rtol):
    assert actual.keys() == expected.keys()
    for name in actual:
        torch.testing.assert_close(actual[name], expected[name], atol=atol, rtol=rtol, msg=lambda m: f"{name}: {m}")


CASES = [("dense", "fp32"), ("dense", "bf16"), ("int8", "bf16"), ("int8_convrot", "bf16")]


@pytest.mark.parametrize("quantization,precision", CASES)
def test_async_frozen_lora_matches_resident_training_and_sampling(cuda_device, quantization, precision):
    torch.manual_seed(83)
    dtype = torch.bfloat16 if precision == "bf16" else torch.float32
    resident = _prepare(quantization, dtype, cuda_device).train()
    streamed = copy.deepcopy(resident).train()
    frozen_before = {n: t.detach().cpu().clone() for n, t in _frozen_layer_tensors(streamed).items()}
    adapter_ids = {n: id(p) for n, p in _trainables(streamed).items()}
    initial = {n: p.detach().cpu().clone() for n, p in _trainables(resident).items()}

    place_model(resident, cuda_device, 0)
    place_model(streamed, cuda_device, len(streamed.layers), block_swap_mode="async")
    manager = streamed.block_swap_manager
    assert manager is not None and manager.h2d_copy_count == 0 and manager.owned_cuda_buffers() == ()
    adapters = _trainables(streamed)
    assert {n: id(p) for n, p in adapters.items()} == adapter_ids
    assert all(p.device.type == "cuda" for p in adapters.values())
    placed = _frozen_layer_tensors(streamed)
    assert placed.keys() == frozen_before.keys()
    assert all(t.device.type == "cpu" and (t.numel() == 0 or t.is_pinned()) for t in placed.values())
    int8_names = [n for n in placed if n.endswith("weight_int8")]
    assert bool(int8_names) == (quantization != "dense")

    opt_resident = torch.optim.AdamW(_trainables(resident).values(), lr=2e-3)
    opt_streamed = torch.optim.AdamW(adapters.values(), lr=2e-3)
    atol, rtol = (4e-3, 3e-2) if precision == "bf16" else (2e-5, 2e-3)
    for step in range(2):
        torch.manual_seed(200 + step)
        batches = _batches(cuda_device, dtype)
        expected = _step(resident, opt_resident, batches, autocast=precision == "bf16")
        actual = _step(streamed, opt_streamed, batches, autocast=precision == "bf16")
        for a, e in zip(actual[0], expected[0]):
            torch.testing.assert_close(a, e, atol=atol, rtol=rtol)
        _assert_named_close(actual[1], expected[1], atol=atol, rtol=rtol)
        _assert_named_close(actual[2], expected[2], atol=atol, rtol=rtol)
        if step == 0:
            resident.eval()
            streamed.eval()
            tokens, t = batches[1]
            with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=precision == "bf16"):
                outs = [m(tokens, t) for m in (resident, streamed)]
                skipped = [m(-tokens, t, skip_layers=(1, 3)) for m in (resident, streamed)]
            assert torch.equal(outs[1], outs[0])
            assert torch.equal(skipped[1], skipped[0])
            resident.train()
            streamed.train()

    final = {n: p.detach().cpu() for n, p in _trainables(resident).items()}
    assert any(not torch.equal(final[n], initial[n]) for n in final)
    assert {n: id(p) for n, p in _trainables(streamed).items()} == adapter_ids
    assert 1 <= manager.peak_resident_blocks <= 2
    after = _frozen_layer_tensors(streamed)
    for name, original in frozen_before.items():
        assert after[name].device.type == "cpu" and (after[name].numel() == 0 or after[name].is_pinned())
        assert torch.equal(after[name], original), name
    assert all(after[n].dtype == torch.int8 for n in int8_names)


def test_partial_swap_supports_two_live_graphs_and_one_backward(cuda_device):
    torch.manual_seed(97)
    resident = _prepare("dense", torch.float32, cuda_device).train()
    streamed = copy.deepcopy(resident).train()
    place_model(resident, cuda_device, 0)
    place_model(streamed, cuda_device, 2, block_swap_mode="async")
    for layer in streamed.layers[:2]:
        assert all(p.device.type == "cuda" for p in layer.parameters())
    for layer in streamed.layers[2:]:
        assert all(p.device.type == ("cuda" if p.requires_grad else "cpu") for p in layer.parameters())
    batches = _batches(cuda_device, torch.float32)
    results = []
    for model in (resident, streamed):
        optimizer = torch.optim.AdamW(_trainables(model).values(), lr=2e-3)
        optimizer.zero_grad(set_to_none=True)
        outputs = [model(tokens, t) for tokens, t in batches]
        assert all(o.grad_fn is not None for o in outputs)
        sum(o.float().square().mean() / len(outputs) for o in outputs).backward()
        grads = {n: p.grad.detach().cpu().clone() for n, p in _trainables(model).items()}
        optimizer.step()
        results.append(([o.detach().cpu() for o in outputs], grads,
                        {n: p.detach().cpu().clone() for n, p in _trainables(model).items()}))
    for a, e in zip(results[1][0], results[0][0]):
        torch.testing.assert_close(a, e, atol=2e-5, rtol=2e-3)
    _assert_named_close(results[1][1], results[0][1], atol=2e-5, rtol=2e-3)
    _assert_named_close(results[1][2], results[0][2], atol=2e-5, rtol=2e-3)
    assert 1 <= streamed.block_swap_manager.peak_resident_blocks <= 2


def test_grad_enabled_eval_forward_backpropagates_through_streamed_blocks(cuda_device):
    torch.manual_seed(101)
    resident = _prepare("dense", torch.float32, cuda_device).eval()
    streamed = copy.deepcopy(resident).eval()
    place_model(resident, cuda_device, 0)
    place_model(streamed, cuda_device, DEPTH, block_swap_mode="async")
    tokens, t = _batches(cuda_device, torch.float32)[0]
    out_r, out_s = resident(tokens, t), streamed(tokens, t)
    assert torch.is_grad_enabled() and out_r.grad_fn is not None and out_s.grad_fn is not None
    out_r.float().square().mean().backward()
    out_s.float().square().mean().backward()
    torch.testing.assert_close(out_s, out_r, atol=2e-5, rtol=2e-3)
    _assert_named_close({n: p.grad.cpu() for n, p in _trainables(streamed).items()},
                        {n: p.grad.cpu() for n, p in _trainables(resident).items()}, atol=2e-5, rtol=2e-3)


def test_autograd_grad_releases_streamed_blocks_for_next_iteration_and_teardown(cuda_device):
    torch.manual_seed(103)
    model = _prepare("dense", torch.float32, cuda_device).train()
    place_model(model, cuda_device, DEPTH, block_swap_mode="async")
    manager = model.block_swap_manager
    params = _trainables(model)
    optimizer = torch.optim.AdamW(params.values(), lr=2e-3)
    batches = _batches(cuda_device, torch.float32)
    first = model(*batches[0]).float().square().mean()
    grads = torch.autograd.grad(first, tuple(params.values()))
    assert len(grads) == len(params) and all(g.is_cuda and torch.isfinite(g).all() for g in grads)
    assert all(p.grad is None for p in params.values())
    optimizer.zero_grad(set_to_none=True)
    model(*batches[1]).float().square().mean().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in params.values())
    optimizer.step()
    place_model(model, torch.device("cpu"), 0)
    assert manager.closed and manager.resident_block_indices == () and model.block_swap_manager is None
    assert all(p.device.type == "cpu" for p in model.parameters())


def test_retained_graph_supports_two_backward_traversals(cuda_device):
    torch.manual_seed(107)
    model = _prepare("dense", torch.float32, cuda_device).train()
    place_model(model, cuda_device, DEPTH, block_swap_mode="async")
    params = _trainables(model)
    loss = model(*_batches(cuda_device, torch.float32)[0]).float().square().mean()
    loss.backward(retain_graph=True)
    first = {n: p.grad.detach().clone() for n, p in params.items()}
    loss.backward()
    for n, p in params.items():
        torch.testing.assert_close(p.grad, first[n] * 2, atol=2e-5, rtol=2e-3)


def test_recompute_exception_allows_cleanup_and_fresh_placement(cuda_device):
    torch.manual_seed(109)
    model = _prepare("dense", torch.float32, cuda_device).train()
    place_model(model, cuda_device, DEPTH, block_swap_mode="async")
    failed = model.block_swap_manager
    layer = model.layers[-1]
    original = layer.forward
    calls = 0

    def fail_during_recompute(*args, **kwargs):
        nonlocal calls
        calls += 1
        if calls == 2:
            raise RuntimeError("recompute failure")
        return original(*args, **kwargs)

    layer.forward = fail_during_recompute
    loss = model(*_batches(cuda_device, torch.float32)[0]).float().square().mean()
    try:
        with pytest.raises(RuntimeError, match="recompute failure"):
            loss.backward()
    finally:
        layer.forward = original
    assert calls == 2
    del loss
    gc.collect()
    place_model(model, torch.device("cpu"), 0)
    assert failed.closed and failed.resident_block_indices == () and model.block_swap_manager is None
    place_model(model, cuda_device, DEPTH, block_swap_mode="async")
    recovered = model.block_swap_manager
    assert recovered is not failed
    model.zero_grad(set_to_none=True)
    model(*_batches(cuda_device, torch.float32)[1]).float().square().mean().backward()
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in _trainables(model).values())
    place_model(model, torch.device("cpu"), 0)
    assert recovered.closed


def test_cpu_placement_closes_manager_after_eval_prefetch(cuda_device):
    torch.manual_seed(113)
    model = _prepare("dense", torch.float32, cuda_device).eval()
    place_model(model, cuda_device, DEPTH, block_swap_mode="async")
    manager = model.block_swap_manager
    assert manager.h2d_copy_count == 0
    with torch.no_grad():
        output = model(*_batches(cuda_device, torch.float32)[0])
    assert output.is_cuda and manager.resident_block_indices
    assert manager.h2d_copy_count == DEPTH
    stats = manager.copy_statistics()
    assert stats["timed_bytes"] == stats["bytes"] == manager.h2d_bytes > 0 and stats["copy_ms"] > 0
    place_model(model, torch.device("cpu"), 0)
    assert manager.closed and manager.resident_block_indices == () and model.block_swap_manager is None
    assert all(p.device.type == "cpu" for p in model.parameters())
    assert all(b.device.type == "cpu" for b in model.buffers())


def test_streamed_weights_are_never_offloaded_as_activations(cuda_device):
    """With activation offload on, the streamer's staging slots count as weights (it reports them
    through ``owned_cuda_buffers``): the offloaded bytes equal the resident model's and the
    adapter gradients agree."""
    torch.manual_seed(127)
    resident = _prepare("int8", torch.bfloat16, cuda_device).train()
    streamed = copy.deepcopy(resident).train()
    place_model(resident, cuda_device, 0)
    place_model(streamed, cuda_device, DEPTH, block_swap_mode="async")
    tokens, t = _batches(cuda_device, torch.bfloat16)[1]
    ring = offload_ring(cuda_device)
    moved = []
    outputs = []
    for model in (resident, streamed):
        model.activation_offload = True
        torch.cuda.synchronize()
        before = ring.stats()["d2h_bytes"]
        loss = model(tokens, t).float().square().mean()
        torch.cuda.synchronize()
        moved.append(ring.stats()["d2h_bytes"] - before)
        loss.backward()
        outputs.append({n: p.grad.detach().cpu() for n, p in _trainables(model).items()})
    assert moved[0] > 0 and moved[1] == moved[0]
    _assert_named_close(outputs[1], outputs[0], atol=4e-3, rtol=3e-2)


def test_block_stager_copies_and_slot_rules(cuda_device):
    """The native state machine: byte-exact staging, slot choice, leases, checked releases."""
    lib = _lib.library()
    gen = np.random.default_rng(5)
    sizes = [3 << 20, 1 << 20, 0, (2 << 20) + 256]
    masters = []
    for n in sizes:
        host = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        host.copy_(torch.from_numpy(gen.integers(0, 256, n, dtype=np.uint8)))
        masters.append(host)
    copy_stream = torch.cuda.Stream(cuda_device)
    compute = torch.cuda.current_stream(cuda_device)
    handle = ctypes.c_void_p()
    _lib.check(lib.moss_block_stager_create(cuda_device.index, 2, copy_stream.cuda_stream, ctypes.byref(handle)),
               "create")
    s = handle.value
    try:
        ids = []
        for host in masters:
            block = ctypes.c_int64()
            _lib.check(lib.moss_block_stager_add_block(s, host.data_ptr() if host.numel() else None, host.numel(),
                                                       ctypes.byref(block)), "add")
            ids.append(block.value)
        assert ids == [0, 1, 2, 3]
        pageable = torch.empty(64, dtype=torch.uint8)
        assert lib.moss_block_stager_add_block(s, pageable.data_ptr(), 64, ctypes.byref(ctypes.c_int64())) \
            == _lib.MOSS_ERR_INVALID_ARGUMENT
        slots = [torch.empty(max(sizes), dtype=torch.uint8, device=cuda_device) for _ in range(2)]
        slot = ctypes.c_int()
        generation = ctypes.c_uint64()

        def select(block, protected=()):
            arr = (ctypes.c_int64 * max(1, len(protected)))(*protected)
            rc = lib.moss_block_stager_select(s, block, arr, len(protected), ctypes.byref(slot))
            return rc, slot.value

        assert select(0) == (_lib.MOSS_OK, 0)
        assert lib.moss_block_stager_stage(s, 0, 0, ctypes.byref(generation)) == _lib.MOSS_ERR_INVALID_ARGUMENT
        for i, buf in enumerate(slots):
            _lib.check(lib.moss_block_stager_set_slot(s, i, buf.data_ptr(), buf.numel()), "set_slot")
        _lib.check(lib.moss_block_stager_stage(s, 0, 0, ctypes.byref(generation)), "stage")
        assert generation.value == 1
        assert select(0) == (_lib.MOSS_OK, 0)          # resident
        assert select(1) == (_lib.MOSS_OK, 1)          # empty
        _lib.check(lib.moss_block_stager_stage(s, 1, 1, None), "stage")
        _lib.check(lib.moss_block_stager_lease(s, 0, compute.cuda_stream, ctypes.byref(generation)), "lease")
        assert lib.moss_block_stager_lease(s, 0, compute.cuda_stream, None) == _lib.MOSS_ERR_BUSY
        assert torch.equal(slots[0][: sizes[0]].cpu(), masters[0])
        assert select(3, (1,))[0] == _lib.MOSS_ERR_BUSY    # slot 0 leased, slot 1 protected
        assert select(3) == (_lib.MOSS_OK, 1)
        assert lib.moss_block_stager_stage(s, 3, 0, None) == _lib.MOSS_ERR_BUSY  # leased slot
        _lib.check(lib.moss_block_stager_hold(s, 0), "hold")
        assert lib.moss_block_stager_destroy(s, 0) == _lib.MOSS_ERR_BUSY
        # a checked release must name the slot's block and generation
        assert lib.moss_block_stager_release(s, 0, 1, 1, compute.cuda_stream) == _lib.MOSS_ERR_NOT_FOUND
        _lib.check(lib.moss_block_stager_release(s, 0, 0, 1, compute.cuda_stream), "release")
        _lib.check(lib.moss_block_stager_stage(s, 3, 0, ctypes.byref(generation)), "restage")
        assert generation.value == 2
        _lib.check(lib.moss_block_stager_stage(s, 2, 1, None), "stage empty block")
        _lib.check(lib.moss_block_stager_lease(s, 0, compute.cuda_stream, None), "lease")
        assert torch.equal(slots[0][: sizes[3]].cpu(), masters[3])
        _lib.check(lib.moss_block_stager_release(s, 0, -1, 0, compute.cuda_stream), "release")
        block, leased = ctypes.c_int64(), ctypes.c_int()
        _lib.check(lib.moss_block_stager_slot_info(s, 1, ctypes.byref(block), None, ctypes.byref(leased)), "info")
        assert block.value == 2 and leased.value == 0
        copies, nbytes, timed = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        peak, ms = ctypes.c_int(), ctypes.c_double()
        _lib.check(lib.moss_block_stager_stats(s, ctypes.byref(copies), ctypes.byref(nbytes), ctypes.byref(peak),
                                               ctypes.byref(ms), ctypes.byref(timed)), "stats")
        assert copies.value == 4 and nbytes.value == sizes[0] + sizes[1] + sizes[3] + 0
        assert peak.value == 2 and timed.value == nbytes.value and ms.value > 0
    finally:
        assert lib.moss_block_stager_destroy(s, 0) == _lib.MOSS_OK

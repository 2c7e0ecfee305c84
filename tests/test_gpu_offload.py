"""GPU tests of the saved-activation offload: byte-identical round trips through the ring.

Covers the layouts of training/tests/test_packed_features.py:201-235 (padded, expanded,
overlapping) and more, prefetching, ring reuse across steps, a NaN-poisoned pinned ring
(a restore that read before its copy finished would surface the poison), the ring-full
path, and offload-vs-resident gradient equality on a model (the differential check of
training/tests/test_packed_cuda.py:173-201).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch
from torch import nn

from moss_image_b200 import _lib
from moss_image_b200 import activation_offload as ao
from moss_image_b200.quantization import FrozenInt8Linear
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _bytes_of(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes() if t.numel() else b""


LAYOUTS = [
    ("contiguous", (4, 33, 17), None),
    ("padded", (1, 1, 5, 5), (64, 64, 8, 1)),
    ("expanded", (3, 5), (0, 1)),
    ("transposed", (96, 40), (1, 96)),
    ("sliced_rows", (40, 70), (128, 1)),
    ("expanded_inner", (2, 3, 4), (12, 4, 0)),
    ("scalar_broadcast", (5, 5), (0, 0)),
    ("size_one_odd_stride", (3, 1, 4), (4, 999, 1)),
]


def _make(device, dtype, shape, stride):
    if stride is None:
        return torch.randn(shape, device=device).to(dtype) if dtype.is_floating_point else \
            torch.randint(-100, 100, shape, device=device).to(dtype)
    extent = 1 + sum((s - 1) * st for s, st in zip(shape, stride))
    backing = torch.randn(extent + 7, device=device).to(dtype) if dtype.is_floating_point else \
        torch.randint(-100, 100, (extent + 7,), device=device).to(dtype)
    return backing.as_strided(shape, stride)


class _Capture(torch.autograd.Function):
    """Saves its input for backward so the pack/unpack hooks see exactly that tensor."""

    @staticmethod
    def forward(ctx, x, probe):
        ctx.save_for_backward(x)
        return probe.clone()

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        _Capture.restored.append(x)
        return None, g


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.int64, torch.uint8])
@pytest.mark.parametrize("name,shape,stride", LAYOUTS)
def test_round_trip_is_byte_identical_with_original_strides(cuda_device, dtype, name, shape, stride):
    x = _make(cuda_device, dtype, shape, stride)
    before = _bytes_of(x)
    probe = torch.zeros(1, device=cuda_device, requires_grad=True)
    _Capture.restored = []
    holder = nn.Module()
    with ao.activation_cpu_offload(holder, True, cuda_device):
        out = _Capture.apply(x, probe)
    out.sum().backward()
    (restored,) = _Capture.restored
    assert restored.shape == x.shape and restored.stride() == x.stride()
    assert _bytes_of(restored) == before
    expected_payload = O.offload_view(tuple(x.shape), tuple(x.stride()))
    view = ao._offload_view(x)
    assert (None if view is None else view[1]) == expected_payload


def test_overlapping_layout_stays_resident(cuda_device):
    backing = torch.randn(16, device=cuda_device)
    overlapping = backing.as_strided((3, 3), (1, 1))
    assert ao._offload_view(overlapping) is None
    probe = torch.zeros(1, device=cuda_device, requires_grad=True)
    _Capture.restored = []
    with ao.activation_cpu_offload(nn.Module(), True, cuda_device):
        out = _Capture.apply(overlapping, probe)
    out.sum().backward()
    assert _Capture.restored[0] is overlapping or _Capture.restored[0].data_ptr() == overlapping.data_ptr()


def test_parameters_and_buffers_stay_resident(cuda_device):
    lin = FrozenInt8Linear(nn.Linear(32, 16).to(cuda_device, torch.bfloat16).requires_grad_(False))
    holder = nn.Module()
    holder.lin = lin
    ring = ao.offload_ring(cuda_device)
    before = ring.stats()["d2h_bytes"]
    x = torch.randn(4, 32, device=cuda_device, dtype=torch.bfloat16, requires_grad=True)
    with ao.activation_cpu_offload(holder, True, cuda_device):
        y = lin(x)  # saves only the int8 weight and the scale: both are module buffers
    y.float().sum().backward()
    torch.cuda.synchronize()
    assert ring.stats()["d2h_bytes"] == before


def test_many_tensors_with_prefetch_and_ring_reuse(cuda_device):
    """A deep chain of saved activations, restored in reverse with a small prefetch window,
    over three steps: the ring rewinds between steps and every byte round-trips."""
    torch.manual_seed(0)
    layers = nn.ModuleList(nn.Linear(256, 256).to(cuda_device) for _ in range(24))
    holder = nn.Module()
    holder.layers = layers
    x0 = torch.randn(512, 256, device=cuda_device)
    grads = []
    for offload in (False, True, True, True):
        x = x0.clone().requires_grad_()
        with ao.activation_cpu_offload(holder, offload, cuda_device, prefetch_bytes=2 << 20):
            h = x
            for layer in layers:
                h = torch.tanh(layer(h)) * 1.5
        h.square().sum().backward()
        grads.append((x.grad.clone(), [p.grad.clone() for p in layers.parameters()]))
        for p in layers.parameters():
            p.grad = None
    for g in grads[1:]:
        assert torch.equal(g[0], grads[0][0])
        assert all(torch.equal(a, b) for a, b in zip(g[1], grads[0][1]))
    torch.cuda.synchronize()
    stats = ao.offload_ring(cuda_device).stats()
    assert stats["live"] == 0


def test_poisoned_ring_never_leaks_into_restores(cuda_device):
    ring = ao.OffloadRing(cuda_device, segment_bytes=8 << 20, max_bytes=8 << 20)
    compute = torch.cuda.current_stream(cuda_device)
    filler = torch.empty(8 << 20, dtype=torch.uint8, device=cuda_device)
    ticket = ring.pack(filler.data_ptr(), filler.numel(), compute)
    ring.d2h_stream.synchronize()
    host = ctypes.c_void_p()
    _lib.check(_lib.library().moss_offload_host_ptr(ring.handle, ticket, ctypes.byref(host)), "host_ptr")
    nan = np.full((8 << 20) // 4, np.nan, np.float32)
    ctypes.memmove(host.value, nan.ctypes.data, nan.nbytes)
    ring.release(ticket)
    # the whole arena is now NaN; pack/restore many tensors through it
    payloads = [torch.randn(n, device=cuda_device) for n in (1, 1000, 65536, 300001, 4096)]
    tickets = [ring.pack(p.data_ptr(), p.numel() * 4, compute) for p in payloads]
    outs = []
    for p, t in zip(reversed(payloads), reversed(tickets)):
        dst = torch.empty_like(p)
        ring.prefetch(t, dst.data_ptr())
        ring.wait(t, compute)
        outs.append(dst)
    for p, o in zip(reversed(payloads), outs):
        assert torch.equal(p, o)
    for t in tickets:
        ring.release(t)
    assert ring.stats()["live"] == 0


def test_ring_full_keeps_tensor_resident(cuda_device):
    ring = ao.OffloadRing(cuda_device, segment_bytes=1 << 20, max_bytes=1 << 20)
    compute = torch.cuda.current_stream(cuda_device)
    big = torch.empty(2 << 20, dtype=torch.uint8, device=cuda_device)
    assert ring.pack(big.data_ptr(), big.numel(), compute) is None
    small = torch.arange(1000, device=cuda_device, dtype=torch.float32)
    t = ring.pack(small.data_ptr(), small.numel() * 4, compute)
    assert t is not None
    assert ring.host_bytes(t, small.numel() * 4) == small.cpu().numpy().tobytes()
    ring.release(t)


def test_offload_matches_resident_on_int8_lora_model(cuda_device):
    from moss_image_b200.dit import build_lora_model, flow_matching_loss

    torch.manual_seed(0)
    model = build_lora_model(2, device=cuda_device, dim=256, heads=2, mlp_dim=512, rank=8, seed=3)
    with torch.no_grad():
        for p in model.parameters():
            if p.requires_grad:
                p.add_(torch.randn_like(p) * 0.02)
    gen = torch.Generator(device=cuda_device).manual_seed(1)
    latents = torch.randn(2, 96, 256, device=cuda_device, generator=gen).to(torch.bfloat16)
    text = torch.randn(2, 32, 256, device=cuda_device, generator=gen).to(torch.bfloat16)
    noise = torch.randn(2, 96, 256, device=cuda_device, generator=gen).to(torch.bfloat16)
    t = torch.rand(2, device=cuda_device, generator=gen)
    results = []
    from torch.nn.attention import SDPBackend, sdpa_kernel

    for offload in (False, True):
        model.activation_offload = offload
        # deterministic attention (also during the checkpoint recompute inside backward) so
        # that any difference can only come from the offload
        with sdpa_kernel(SDPBackend.MATH):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = flow_matching_loss(model, latents, text, t, noise)
            loss.backward()
        results.append((loss.detach().clone(), [p.grad.clone() for p in model.parameters() if p.requires_grad]))
        model.zero_grad(set_to_none=True)
    assert torch.equal(results[0][0], results[1][0])
    for a, b in zip(results[0][1], results[1][1]):
        assert torch.equal(a, b)


def test_deferred_copies_keep_the_newest_tensors_and_gradients_identical(cuda_device):
    """With a deferral budget the newest saved tensors stay on the GPU (never copied out and
    back) and only the older ones go through the ring; the gradients are bit-identical to the
    run without offload for every budget, and the bytes copied shrink as the budget grows."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from moss_image_b200.dit import build_lora_model, flow_matching_loss

    torch.manual_seed(0)
    model = build_lora_model(3, device=cuda_device, dim=256, heads=2, mlp_dim=512, rank=8, seed=4)
    with torch.no_grad():
        for p in model.parameters():
            if p.requires_grad:
                p.add_(torch.randn_like(p) * 0.02)
    gen = torch.Generator(device=cuda_device).manual_seed(2)
    latents = torch.randn(2, 96, 256, device=cuda_device, generator=gen).to(torch.bfloat16)
    text = torch.randn(2, 32, 256, device=cuda_device, generator=gen).to(torch.bfloat16)
    noise = torch.randn(2, 96, 256, device=cuda_device, generator=gen).to(torch.bfloat16)
    t = torch.rand(2, device=cuda_device, generator=gen)
    ring = ao.offload_ring(cuda_device)
    block_input = 2 * 128 * 256 * 2  # one checkpointed block's saved input

    def run(offload: bool, defer_bytes: int):
        model.activation_offload = offload
        model.activation_offload_defer_bytes = defer_bytes
        before = ring.stats()["d2h_bytes"]
        with sdpa_kernel(SDPBackend.MATH):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = flow_matching_loss(model, latents, text, t, noise)
            loss.backward()
        torch.cuda.synchronize()
        grads = [p.grad.clone() for p in model.parameters() if p.requires_grad]
        model.zero_grad(set_to_none=True)
        return loss.detach().clone(), grads, ring.stats()["d2h_bytes"] - before

    reference = run(False, 0)
    moved = []
    for budget in (0, 3 * block_input, 1 << 40):
        loss, grads, nbytes = run(True, budget)
        assert torch.equal(loss, reference[0])
        for a, b in zip(grads, reference[1]):
            assert torch.equal(a, b)
        moved.append(nbytes)
    model.activation_offload_defer_bytes = 0
    assert moved[0] >= 3 * block_input  # every block input goes out
    assert 0 < moved[1] <= moved[0] - 2 * block_input  # the newest ~3 block inputs' worth stays
    assert moved[2] == 0  # everything stays
    assert ring.stats()["live"] == 0

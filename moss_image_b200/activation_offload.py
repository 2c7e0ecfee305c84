"""Scoped saved-activation offload through a pinned-host ring, with restore prefetch.

Drop-in for ``training/activation_offload.py``: ``activation_cpu_offload(model, enabled,
device)`` returns the same kind of context (``nullcontext`` on CPU, when disabled or with
grad disabled) and applies the same selection rules: parameter/buffer-backed tensors and
block-swap staging buffers stay resident, expanded dimensions are narrowed to one element,
and negative-stride or overlapping layouts stay on the device.

What changes is the transport (``libmoss_w8.so``):

* each saved payload is copied device-to-host on a dedicated copy stream into a
  bump-allocated pinned ring (no per-tensor pinned allocation, no copy on the compute
  stream); non-contiguous payload views are gathered on the GPU first so every tensor is
  one copy-engine transfer;
* restores run host-to-device on a second copy stream and are issued ahead of use: when
  backward unpacks a tensor, the tensors packed just before it (the previous block's, in
  backward order) are restored too, up to ``prefetch_bytes`` in flight; the compute stream
  waits only for the tensor it needs;
* restored tensors get the original strides back (``_restore_layout`` semantics), so
  round trips are byte-identical.
"""

from __future__ import annotations

import ctypes
import os
import threading
import weakref
from contextlib import nullcontext
from typing import ContextManager

import torch
from torch import nn

from . import _lib

DEFAULT_PREFETCH_BYTES = 256 << 20
DEFAULT_SEGMENT_BYTES = 256 << 20


def _storage_key(tensor: torch.Tensor) -> tuple[str, int | None, int]:
    """Reference: training/activation_offload.py:27-29."""
    device = tensor.device
    return device.type, device.index, tensor.untyped_storage().data_ptr()


def _offload_view(tensor: torch.Tensor) -> tuple[torch.Tensor, tuple[int, ...]] | None:
    """Return a non-overlapping view suitable for a dense payload, or ``None``.

    Same rule as training/activation_offload.py:32-61: negative strides stay resident;
    a stride-0 dimension of size > 1 is narrowed to one element; the remaining dimensions
    (sorted by stride, size-1 dimensions ignored) must occupy unique storage offsets.
    """
    shape = list(tensor.shape)
    strides = tensor.stride()
    source = tensor
    for dim, (size, stride) in enumerate(zip(tensor.shape, strides)):
        if stride < 0:
            return None
        if stride == 0 and size > 1:
            source = source.narrow(dim, 0, 1)
            shape[dim] = 1
    extent = 1
    for stride, size in sorted((st, sz) for sz, st in zip(shape, strides) if sz > 1):
        if stride < extent:
            return None
        extent += (size - 1) * stride
    return source, tuple(shape)


def _restore_layout(
    payload: torch.Tensor,
    device: torch.device,
    shape: tuple[int, ...],
    stride: tuple[int, ...],
    payload_shape: tuple[int, ...],
    *,
    non_blocking: bool,
) -> torch.Tensor:
    """Copy a dense payload into the original padded or expanded layout.

    Reference helper semantics (training/activation_offload.py:64-77); kept for API
    compatibility. The offload hooks below restore through the ring and the scatter kernel.
    """
    restored = torch.empty_strided(payload_shape, stride, dtype=payload.dtype, device=device)
    restored.copy_(payload, non_blocking=non_blocking)
    return restored.as_strided(shape, stride)


def _c_contiguous(shape: tuple[int, ...], stride: tuple[int, ...]) -> bool:
    expected = 1
    for size, st in zip(reversed(shape), reversed(stride)):
        if size == 1:
            continue
        if st != expected:
            return False
        expected *= size
    return True


def bind_to_device_numa_node(device: torch.device) -> list[int] | None:
    """Restrict this process to the CPU cores NVML reports as local to ``device``.

    Call it once per rank, before the first offload: the offload ring's pinned host memory is
    then allocated (and first touched) on the NUMA node next to the GPU's PCIe root, so the
    copy engines of the GPUs of a multi-socket host write to local memory instead of crossing
    the socket interconnect. Reads the affinity only (no GPU setting changes); returns the
    cores, or ``None`` when NVML or the affinity query is unavailable (nothing is changed).
    """
    try:
        import pynvml
    except ImportError:
        return None
    props = torch.cuda.get_device_properties(device)
    bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    ncpu = os.cpu_count() or 1
    try:
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, (ncpu + 63) // 64)
    except Exception:  # NVML missing on the host, or the query is not supported
        return None
    cpus = [64 * i + b for i, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1 and 64 * i + b < ncpu]
    if not cpus:
        return None
    try:
        os.sched_setaffinity(0, cpus)
    except OSError:
        return None
    return cpus


def _host_memory_bytes() -> int:
    try:
        return os.sysconf("SC_PAGE_SIZE") * os.sysconf("SC_PHYS_PAGES")
    except (ValueError, OSError, AttributeError):
        return 64 << 30


class OffloadRing:
    """Python handle of one device's C++ pinned ring and its two copy streams."""

    def __init__(self, device: torch.device, *, segment_bytes: int = DEFAULT_SEGMENT_BYTES,
                 max_bytes: int | None = None) -> None:
        self.device = device
        self.d2h_stream = torch.cuda.Stream(device)
        self.h2d_stream = torch.cuda.Stream(device)
        if max_bytes is None:
            max_bytes = max(segment_bytes, min(_host_memory_bytes() // 2, 256 << 30))
        handle = ctypes.c_void_p()
        lib = _lib.library()
        rc = lib.moss_offload_ring_create(
            device.index, segment_bytes, max_bytes, self.d2h_stream.cuda_stream, self.h2d_stream.cuda_stream,
            ctypes.byref(handle),
        )
        _lib.check(rc, "moss_offload_ring_create")
        self.handle = handle.value
        self._finalizer = weakref.finalize(self, _destroy_ring, self.handle)

    def pack(self, src_ptr: int, nbytes: int, compute: torch.cuda.Stream) -> int | None:
        ticket = ctypes.c_int64()
        rc = _lib.library().moss_offload_pack(self.handle, src_ptr, nbytes, compute.cuda_stream, ctypes.byref(ticket))
        if rc == _lib.MOSS_ERR_RING_FULL:
            return None
        _lib.check(rc, "moss_offload_pack")
        return ticket.value

    def prefetch(self, ticket: int, dst_ptr: int) -> None:
        _lib.check(_lib.library().moss_offload_prefetch(self.handle, ticket, dst_ptr), "moss_offload_prefetch")

    def wait(self, ticket: int, compute: torch.cuda.Stream) -> None:
        _lib.check(_lib.library().moss_offload_wait(self.handle, ticket, compute.cuda_stream), "moss_offload_wait")

    def release(self, ticket: int) -> None:
        lib = _lib.library()
        rc = lib.moss_offload_release(self.handle, ticket)
        if rc != _lib.MOSS_OK and rc != _lib.MOSS_ERR_NOT_FOUND:
            _lib.check(rc, "moss_offload_release")

    def host_bytes(self, ticket: int, nbytes: int) -> bytes:
        """Copy of a ticket's pinned payload (synchronises the D2H stream first)."""
        self.d2h_stream.synchronize()
        out = ctypes.c_void_p()
        _lib.check(_lib.library().moss_offload_host_ptr(self.handle, ticket, ctypes.byref(out)), "moss_offload_host_ptr")
        return ctypes.string_at(out.value, nbytes)

    def stats(self) -> dict[str, int]:
        d2h, h2d, pinned = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        live = ctypes.c_int64()
        _lib.check(
            _lib.library().moss_offload_stats(self.handle, ctypes.byref(d2h), ctypes.byref(h2d), ctypes.byref(live),
                                              ctypes.byref(pinned)),
            "moss_offload_stats",
        )
        return {"d2h_bytes": d2h.value, "h2d_bytes": h2d.value, "live": live.value, "pinned_bytes": pinned.value}

    def set_timing(self, enable: bool) -> None:
        """Time every later copy with a CUDA event pair on its stream (measurement only)."""
        _lib.check(_lib.library().moss_offload_set_timing(self.handle, 1 if enable else 0), "moss_offload_set_timing")

    def copy_time(self) -> dict[str, float]:
        """Summed copy-engine time and bytes of the timed copies, per direction (waits for them)."""
        d2h_ms, h2d_ms = ctypes.c_double(), ctypes.c_double()
        d2h_b, h2d_b = ctypes.c_uint64(), ctypes.c_uint64()
        _lib.check(_lib.library().moss_offload_copy_time(self.handle, ctypes.byref(d2h_ms), ctypes.byref(h2d_ms),
                                                         ctypes.byref(d2h_b), ctypes.byref(h2d_b)),
                   "moss_offload_copy_time")
        return {"d2h_ms": d2h_ms.value, "h2d_ms": h2d_ms.value, "d2h_bytes": d2h_b.value, "h2d_bytes": h2d_b.value}





def _destroy_ring(handle: int) -> None:
    try:
        _lib.library().moss_offload_ring_destroy(handle)
    except Exception:  # interpreter shutdown
        pass


_rings: dict[int, OffloadRing] = {}
_rings_lock = threading.Lock()


def offload_ring(device: torch.device) -> OffloadRing:
    """The process-wide ring of a CUDA device (created on first use)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    with _rings_lock:
        ring = _rings.get(index)
        if ring is None:
            ring = OffloadRing(torch.device("cuda", index))
            _rings[index] = ring
        return ring


class _OffloadedTensor:
    """A saved activation living in the pinned ring (reference fields plus a ticket).

    While its copy is deferred (the most recently saved tensors, see ``defer_bytes``) it has no
    ticket and ``resident`` holds the saved tensor itself.
    """

    __slots__ = ("ring", "ticket", "device", "dtype", "shape", "stride", "payload_shape", "nbytes", "index",
                 "restored", "resident", "deferred", "__weakref__")

    def __init__(self, ring, ticket, device, dtype, shape, stride, payload_shape, nbytes, index):
        self.ring = ring
        self.ticket = ticket
        self.device = device
        self.dtype = dtype
        self.shape = shape
        self.stride = stride
        self.payload_shape = payload_shape
        self.nbytes = nbytes
        self.index = index
        self.restored: torch.Tensor | None = None
        self.resident: torch.Tensor | None = None
        self.deferred = False  # counted in its scope's deferred bytes

    def __del__(self):
        ring, ticket = self.ring, self.ticket
        if ring is not None and ticket is not None:
            self.ticket = None
            try:
                ring.release(ticket)
            except Exception:
                pass


class _OffloadScope:
    """Book-keeping of one forward: saved tensors in pack order, deferred copies and restore
    prefetch."""

    def __init__(self, ring: OffloadRing, prefetch_bytes: int, defer_bytes: int = 0) -> None:
        self.ring = ring
        self.prefetch_bytes = prefetch_bytes
        self.defer_bytes = defer_bytes
        self.entries: list[weakref.ref] = []
        self.next_scan = -1  # next pack index to consider for prefetch (walks downwards)
        self.in_flight = 0
        self.lock = threading.Lock()
        self.packed_bytes = 0
        self.deferred: list[weakref.ref] = []  # saved, not copied yet, oldest first
        self.deferred_bytes = 0

    def add(self, entry: _OffloadedTensor) -> None:
        self.entries.append(weakref.ref(entry))
        self.packed_bytes += entry.nbytes

    def defer(self, entry: _OffloadedTensor, offload) -> None:
        """Keep `entry` resident for now; copy out the oldest deferred tensors beyond the budget.

        Backward needs the saved tensors in reverse order, so the newest ones are needed first:
        copying them out would only bring them straight back, and on a shared host link their
        copies would queue behind every earlier one.
        """
        with self.lock:
            entry.deferred = True
            self.deferred.append(weakref.ref(entry))
            self.deferred_bytes += entry.nbytes
            while self.deferred_bytes > self.defer_bytes and self.deferred:
                oldest = self.deferred.pop(0)()
                if oldest is None or not oldest.deferred:
                    continue
                oldest.deferred = False
                self.deferred_bytes -= oldest.nbytes
                offload(oldest)

    def _issue(self, entry: _OffloadedTensor) -> None:
        ring = self.ring
        with torch.cuda.stream(ring.h2d_stream):
            if _c_contiguous(entry.payload_shape, entry.stride):
                dst = torch.empty_strided(entry.payload_shape, entry.stride, dtype=entry.dtype, device=entry.device)
            else:
                dst = torch.empty(entry.payload_shape, dtype=entry.dtype, device=entry.device)
        ring.prefetch(entry.ticket, dst.data_ptr())
        entry.restored = dst
        self.in_flight += entry.nbytes

    def restore(self, entry: _OffloadedTensor) -> torch.Tensor:
        with self.lock:
            if entry.resident is not None:  # never copied out: hand back the saved tensor itself
                resident = entry.resident
                entry.resident = None
                if entry.deferred:
                    entry.deferred = False
                    self.deferred_bytes -= entry.nbytes
                return resident
            if entry.restored is None:
                self._issue(entry)
            # Prefetch the tensors packed before this one (backward walks blocks in reverse).
            if entry.index >= 0:
                if self.next_scan < 0 or entry.index - 1 < self.next_scan:
                    self.next_scan = entry.index - 1
                while self.next_scan >= 0 and self.in_flight < self.prefetch_bytes:
                    other = self.entries[self.next_scan]()
                    if other is not None and other.restored is None and other.ticket is not None:
                        self._issue(other)
                    self.next_scan -= 1
            restored = entry.restored
            entry.restored = None
            self.in_flight = max(0, self.in_flight - entry.nbytes)
        compute = torch.cuda.current_stream(entry.device)
        self.ring.wait(entry.ticket, compute)
        restored.record_stream(compute)
        if not _c_contiguous(entry.payload_shape, entry.stride):
            target = torch.empty_strided(entry.payload_shape, entry.stride, dtype=entry.dtype, device=entry.device)
            sizes = (_int64_array(entry.payload_shape), _int64_array(entry.stride))
            rc = _lib.library().moss_strided_scatter(
                restored.data_ptr(), restored.element_size(), len(entry.payload_shape), sizes[0], sizes[1],
                target.data_ptr(), compute.cuda_stream,
            )
            _lib.check(rc, "moss_strided_scatter")
            _lib.count_launch("strided_copy")
            restored = target
        return restored.as_strided(entry.shape, entry.stride)


def _int64_array(values) -> ctypes.Array:
    return (ctypes.c_int64 * max(1, len(values)))(*values)


# Attribute that keeps a saved tensor resident. Packed batches set it on their sequence
# boundaries: the boundaries are tiny, and a jagged attention recomputed under a checkpoint
# must see the same boundaries tensor the forward saw.
KEEP_RESIDENT = "moss_keep_resident"


def activation_cpu_offload(
    model: nn.Module,
    enabled: bool,
    device: torch.device,
    *,
    prefetch_bytes: int | None = None,
    defer_bytes: int | None = None,
) -> ContextManager[object]:
    """Offload tensors saved by autograd to the pinned host ring.

    Reference: training/activation_offload.py:80-149 (same arguments, same resident-set
    rules, CPU no-op). ``prefetch_bytes`` (default: ``model.activation_offload_prefetch_bytes``
    or 256 MiB) bounds the restores kept in flight ahead of backward. ``defer_bytes`` (default:
    ``model.activation_offload_defer_bytes`` or 0, the reference's behaviour) keeps up to that
    many bytes of the most recently saved tensors on the GPU, copying a tensor out only once
    newer ones push it past the budget: the tensors backward needs first are then never sent
    out and back. Every tensor's bytes are the same either way.
    """
    if not enabled or device.type != "cuda" or not torch.is_grad_enabled():
        return nullcontext()

    resident_storages = {
        _storage_key(tensor)
        for tensor in (*model.parameters(), *model.buffers())
        if tensor.device.type == "cuda" and tensor.untyped_storage().nbytes()
    }

    def is_weight_backed(tensor: torch.Tensor) -> bool:
        key = _storage_key(tensor)
        if key in resident_storages:
            return True
        manager = getattr(model, "block_swap_manager", None)
        owned = getattr(manager, "owned_cuda_buffers", None)
        if not callable(owned):
            return False
        return any(buffer.device.type == "cuda" and _storage_key(buffer) == key for buffer in owned())

    if prefetch_bytes is None:
        prefetch_bytes = int(getattr(model, "activation_offload_prefetch_bytes", DEFAULT_PREFETCH_BYTES))
    scope_device = device if device.index is not None else torch.device("cuda", torch.cuda.current_device())
    if defer_bytes is None:
        defer_bytes = int(getattr(model, "activation_offload_defer_bytes", 0))
    scope = _OffloadScope(offload_ring(scope_device), prefetch_bytes, defer_bytes)

    def copy_out(entry: _OffloadedTensor, tensor: torch.Tensor, source: torch.Tensor) -> bool:
        """Issue the D2H copy of a saved tensor's payload; False when the ring is full."""
        ring = entry.ring
        compute = torch.cuda.current_stream(tensor.device)
        nbytes = entry.nbytes
        payload_shape = entry.payload_shape
        if source.is_contiguous():
            staged = source
        else:
            staged = torch.empty(payload_shape, dtype=tensor.dtype, device=tensor.device)
            rc = _lib.library().moss_strided_gather(
                source.data_ptr(), source.element_size(), source.dim(), _int64_array(payload_shape),
                _int64_array(source.stride()), staged.data_ptr(), compute.cuda_stream,
            )
            _lib.check(rc, "moss_strided_gather")
            _lib.count_launch("strided_copy")
        ticket = ring.pack(staged.data_ptr(), nbytes, compute)
        if ticket is None:  # ring at its limit: keep this tensor resident, like other exclusions
            return False
        staged.record_stream(ring.d2h_stream)
        entry.ticket = ticket
        return True

    def deferred_copy_out(entry: _OffloadedTensor) -> None:
        tensor = entry.resident
        view = _offload_view(tensor)
        if view is not None and copy_out(entry, tensor, view[0]):
            entry.resident = None
        # else: stays resident (ring full); restore() hands the tensor back

    def pack(tensor: torch.Tensor):
        if tensor.device.type != "cuda" or is_weight_backed(tensor) or getattr(tensor, KEEP_RESIDENT, False):
            return tensor
        view = _offload_view(tensor)
        if view is None:
            return tensor
        source, payload_shape = view
        ring = scope.ring if tensor.device == scope.ring.device else offload_ring(tensor.device)
        nbytes = source.numel() * source.element_size()
        own = ring is scope.ring
        entry = _OffloadedTensor(ring, None, tensor.device, tensor.dtype, tuple(tensor.shape),
                                 tuple(tensor.stride()), payload_shape, nbytes, len(scope.entries) if own else -1)
        if own and scope.defer_bytes > 0:
            entry.resident = tensor
            scope.add(entry)
            scope.defer(entry, deferred_copy_out)
            return (entry, scope)
        if not copy_out(entry, tensor, source):
            return tensor
        if own:
            scope.add(entry)
        return (entry, scope if own else None)

    def unpack(saved):
        if isinstance(saved, torch.Tensor):
            return saved
        entry, owner = saved
        if owner is None:
            owner = _OffloadScope(entry.ring, 0)
        return owner.restore(entry)

    return torch.autograd.graph.saved_tensors_hooks(pack, unpack)

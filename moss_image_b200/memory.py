"""Block placement: resident, synchronous CPU masters, or asynchronous frozen-block streaming.

Drop-in for ``training/memory.py`` (same names, arguments, attributes and error messages):

* ``place_model(model, device, blocks_to_swap, block_swap_mode="sync" | "async")`` keeps the
  first ``len(model.layers) - blocks_to_swap`` blocks on the device and swaps the rest;
* ``sync`` keeps whole swapped blocks on the CPU and runs each invocation from device copies
  of its parameters under non-reentrant checkpointing (:func:`offloaded_block`);
* ``async`` packs the frozen tensors of every swapped block (int8 weights, scales, biases,
  norms) into one pinned host master, keeps the trainable LoRA adapters on the device, and
  streams masters through two device staging slots with :class:`AsyncBlockStreamer`.

The staging-slot state machine (slot choice, copy fencing, leases, release events) is the
native block stager of ``libmoss_w8.so`` (``moss_block_stager_*``): one copy-engine H2D
transfer per staged block on a dedicated copy stream, prefetched one block ahead in the
direction of traversal. This module adds only what needs autograd: ``functional_call`` over
the staged views, checkpoint recomputation and the gradient hook that ends a backward lease.

``async_full`` (streaming of trainable full-precision blocks) is validated like the reference
but not provided: it is outside this library's int8 frozen-weight path.
"""

from __future__ import annotations

import ctypes
from contextlib import nullcontext
from contextvars import ContextVar
from dataclasses import dataclass

import torch
from torch import nn
from torch.func import functional_call
from torch.utils.checkpoint import checkpoint

from . import _lib
from .packed import CHECKPOINT_CHECK

NUM_STAGING_SLOTS = 2
_ALIGNMENT = 256


def offloaded_block(layer: nn.Module, *args: torch.Tensor) -> torch.Tensor:
    """Run a block whose parameters live on the CPU from per-invocation device copies.

    Reference: training/memory.py:22-36. Parameters enter the checkpointed function as
    inputs, so gradients flow back to the CPU masters through the copies.
    """
    device = args[0].device
    names, parameters = zip(*layer.named_parameters())
    buffers = dict(layer.named_buffers())

    def run(*inputs: torch.Tensor) -> torch.Tensor:
        values = {name: value.to(device) for name, value in zip(names, inputs[: len(names)])}
        values.update({name: value.to(device) for name, value in buffers.items()})
        return functional_call(layer, values, inputs[len(names):], strict=True)

    if torch.is_grad_enabled():
        return checkpoint(run, *parameters, *args, use_reentrant=False, determinism_check=CHECKPOINT_CHECK)
    return run(*parameters, *args)


@dataclass(frozen=True)
class _TensorView:
    offset: int
    nbytes: int
    shape: torch.Size
    dtype: torch.dtype


@dataclass
class _BlockTensors:
    cpu_buffer: torch.Tensor
    views: dict[str, _TensorView]
    trainable: dict[str, nn.Parameter]


def _typed_view(buffer: torch.Tensor, view: _TensorView) -> torch.Tensor:
    return buffer[view.offset: view.offset + view.nbytes].view(view.dtype).view(view.shape)


class _RecomputeContext:
    """Marks checkpoint recomputation (re-entrant and nestable) in a context variable."""

    def __init__(self, phase: ContextVar[bool]) -> None:
        self._phase = phase
        self._tokens: ContextVar[tuple] = ContextVar("moss_block_recompute_tokens", default=())

    def __enter__(self) -> None:
        self._tokens.set(self._tokens.get() + (self._phase.set(True),))

    def __exit__(self, exc_type, exc_value, traceback) -> bool:
        tokens = self._tokens.get()
        if not tokens:
            raise RuntimeError("Async block recompute context exited without being entered.")
        self._tokens.set(tokens[:-1])
        self._phase.reset(tokens[-1])
        return False


def _is_checkpoint_early_stop(error: BaseException) -> bool:
    """Non-reentrant checkpointing stops a recomputation with a private exception type."""
    kind = type(error)
    return kind.__name__ == "_StopRecomputationError" and kind.__module__ == "torch.utils.checkpoint"


class _Stager:
    """Owner of one native block stager (``moss_block_stager_*``)."""

    def __init__(self, device: torch.device, num_slots: int, copy_stream: torch.cuda.Stream) -> None:
        self.lib = _lib.library()
        handle = ctypes.c_void_p()
        _lib.check(self.lib.moss_block_stager_create(device.index, num_slots, copy_stream.cuda_stream,
                                                     ctypes.byref(handle)), "moss_block_stager_create")
        self.handle = handle.value

    def add_block(self, buffer: torch.Tensor) -> int:
        block = ctypes.c_int64()
        nbytes = buffer.numel()
        _lib.check(self.lib.moss_block_stager_add_block(self.handle, buffer.data_ptr() if nbytes else None, nbytes,
                                                        ctypes.byref(block)), "moss_block_stager_add_block")
        return block.value

    def select(self, block: int, protected: tuple[int, ...]) -> int | None:
        slot = ctypes.c_int()
        array = (ctypes.c_int64 * max(1, len(protected)))(*protected)
        rc = self.lib.moss_block_stager_select(self.handle, block, array, len(protected), ctypes.byref(slot))
        if rc == _lib.MOSS_ERR_BUSY:
            return None
        _lib.check(rc, "moss_block_stager_select")
        return slot.value

    def set_slot(self, slot: int, buffer: torch.Tensor) -> None:
        _lib.check(self.lib.moss_block_stager_set_slot(self.handle, slot, buffer.data_ptr(), buffer.numel()),
                   "moss_block_stager_set_slot")

    def stage(self, block: int, slot: int) -> int:
        generation = ctypes.c_uint64()
        _lib.check(self.lib.moss_block_stager_stage(self.handle, block, slot, ctypes.byref(generation)),
                   "moss_block_stager_stage")
        return generation.value

    def lease(self, slot: int, stream: torch.cuda.Stream) -> int | None:
        generation = ctypes.c_uint64()
        rc = self.lib.moss_block_stager_lease(self.handle, slot, stream.cuda_stream, ctypes.byref(generation))
        if rc == _lib.MOSS_ERR_BUSY:
            return None
        _lib.check(rc, "moss_block_stager_lease")
        return generation.value

    def hold(self, slot: int) -> None:
        _lib.check(self.lib.moss_block_stager_hold(self.handle, slot), "moss_block_stager_hold")

    def release(self, slot: int, stream: torch.cuda.Stream, block: int = -1, generation: int = 0) -> bool:
        """Record the slot's release on ``stream``; False if a checked slot changed meanwhile."""
        rc = self.lib.moss_block_stager_release(self.handle, slot, block, generation, stream.cuda_stream)
        if rc == _lib.MOSS_ERR_NOT_FOUND:
            return False
        _lib.check(rc, "moss_block_stager_release")
        return True

    def slot_block(self, slot: int) -> int:
        block = ctypes.c_int64()
        _lib.check(self.lib.moss_block_stager_slot_info(self.handle, slot, ctypes.byref(block), None, None),
                   "moss_block_stager_slot_info")
        return block.value

    def stats(self, *, timing: bool = False) -> dict[str, float]:
        copies, nbytes, timed = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        peak, copy_ms = ctypes.c_int(), ctypes.c_double()
        _lib.check(self.lib.moss_block_stager_stats(
            self.handle, ctypes.byref(copies), ctypes.byref(nbytes), ctypes.byref(peak),
            ctypes.byref(copy_ms) if timing else None, ctypes.byref(timed) if timing else None),
            "moss_block_stager_stats")
        out = {"copies": copies.value, "bytes": nbytes.value, "peak_resident": peak.value}
        if timing:
            out.update(copy_ms=copy_ms.value, timed_bytes=timed.value)
        return out

    def destroy(self, *, force: bool) -> bool:
        """Free the stager after its copies and releases finish; False while a slot is leased."""
        if self.handle is None:
            return True
        rc = self.lib.moss_block_stager_destroy(self.handle, 1 if force else 0)
        if rc == _lib.MOSS_ERR_BUSY:
            return False
        self.handle = None
        _lib.check(rc, "moss_block_stager_destroy")
        return True


class AsyncBlockStreamer:
    """H2D-only streamer of frozen blocks through two reusable device staging slots.

    Reference: training/memory.py:92-360 (same constructor, ``block``/``close`` signatures,
    attributes and errors). Trainable LoRA parameters are read from the module at every
    invocation, so an optimizer step never leaves a stale adapter behind. Frozen tensors are
    views of the staging slot that holds the block; a block's slot is leased while it runs
    and, during a checkpoint recomputation, until the block's backward has finished.
    """

    def __init__(
        self,
        layers: nn.ModuleList,
        device: torch.device,
        first_streamed_block: int,
        blocks: dict[int, _BlockTensors],
    ) -> None:
        device = torch.device(device)
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.layers = layers
        self.device = device
        self.first_streamed_block = first_streamed_block
        self.copy_stream = torch.cuda.Stream(device=device)
        self._blocks = blocks
        self._slot_capacity = max(block.cpu_buffer.numel() for block in blocks.values())
        self._stager = _Stager(device, NUM_STAGING_SLOTS, self.copy_stream)
        self._ids = {index: self._stager.add_block(block.cpu_buffer) for index, block in blocks.items()}
        self._indices = {block: index for index, block in self._ids.items()}
        self._buffers: list[torch.Tensor | None] = [None] * NUM_STAGING_SLOTS
        self._views: list[tuple[int, int, dict[str, torch.Tensor]] | None] = [None] * NUM_STAGING_SLOTS
        self._in_recompute: ContextVar[bool] = ContextVar("moss_block_recompute", default=False)
        self._recompute_context = _RecomputeContext(self._in_recompute)
        self._final_stats: dict[str, float] | None = None
        self._closed = False

    # ------------------------------------------------------------------ inspection
    @property
    def peak_resident_blocks(self) -> int:
        return int(self._counters()["peak_resident"])

    @property
    def h2d_copy_count(self) -> int:
        return int(self._counters()["copies"])

    @property
    def h2d_bytes(self) -> int:
        """Bytes copied host to device by this streamer."""
        return int(self._counters()["bytes"])

    def copy_statistics(self) -> dict[str, float]:
        """Copies, bytes and copy-engine milliseconds so far (waits for copies in flight)."""
        if self._closed:
            return dict(self._final_stats or {})
        return self._stager.stats(timing=True)

    def _counters(self) -> dict[str, float]:
        if self._closed:
            return self._final_stats or {"copies": 0, "bytes": 0, "peak_resident": 0}
        return self._stager.stats()

    @property
    def resident_block_indices(self) -> tuple[int, ...]:
        """Block indices currently held in the CUDA staging slots."""
        if self._closed:
            return ()
        held = (self._stager.slot_block(slot) for slot in range(NUM_STAGING_SLOTS))
        return tuple(sorted(self._indices[block] for block in held if block >= 0))

    @property
    def closed(self) -> bool:
        """Whether teardown has released this manager's staging resources."""
        return self._closed

    def owned_cuda_buffers(self) -> tuple[torch.Tensor, ...]:
        """Currently allocated CUDA staging buffers (allocates nothing)."""
        return tuple(buffer for buffer in self._buffers if buffer is not None)

    # ------------------------------------------------------------------ staging
    def _stage(self, index: int, protected: frozenset[int]) -> int:
        block = self._ids[index]
        slot = self._stager.select(block, tuple(self._ids[item] for item in protected))
        if slot is None:
            raise RuntimeError("Async block streamer exhausted its two protected staging slots.")
        if self._buffers[slot] is None:
            buffer = torch.empty(self._slot_capacity, dtype=torch.uint8, device=self.device)
            buffer.record_stream(self.copy_stream)
            self._stager.set_slot(slot, buffer)
            self._buffers[slot] = buffer
        self._stager.stage(block, slot)
        return slot

    def _staged_tensors(self, slot: int, index: int, generation: int) -> dict[str, torch.Tensor]:
        cached = self._views[slot]
        if cached is not None and cached[0] == index and cached[1] == generation:
            return cached[2]
        buffer = self._buffers[slot]
        tensors = {name: _typed_view(buffer, view) for name, view in self._blocks[index].views.items()}
        self._views[slot] = (index, generation, tensors)
        return tensors

    def _record_backward_use(self, slot: int, index: int, generation: int,
                             tensors: tuple[torch.Tensor, ...]) -> torch.utils.hooks.RemovableHandle:
        """Keep the slot leased until gradients for every block input exist."""
        differentiable = tuple(tensor for tensor in tensors if tensor.requires_grad)
        if not differentiable:
            raise RuntimeError("Async block checkpoint recomputation requires differentiable tensors.")
        self._stager.hold(slot)
        block = self._ids[index]
        handle_box: list[torch.utils.hooks.RemovableHandle] = []

        def finished(gradients) -> None:
            try:
                if self._closed:
                    return
                stream = torch.cuda.current_stream(self.device)
                if not self._stager.release(slot, stream, block, generation):
                    raise RuntimeError("Async block staging slot changed before backward completed.")
            finally:
                handle_box[0].remove()

        handle = torch.autograd.graph.register_multi_grad_hook(differentiable, finished, mode="all")
        handle_box.append(handle)
        return handle

    def _run(
        self,
        index: int,
        inputs: tuple[torch.Tensor, ...],
        trainable: dict[str, torch.Tensor],
        completion_tensors: tuple[torch.Tensor, ...],
        forward_prefetch: int | None,
        backward_prefetch: int | None,
    ) -> torch.Tensor:
        if self._closed:
            raise RuntimeError("Async block streamer is closed.")
        recomputing = self._in_recompute.get()
        prefetch = backward_prefetch if recomputing else forward_prefetch
        protected = frozenset(item for item in (index, prefetch) if item is not None)
        slot = self._stage(index, protected)
        compute_stream = torch.cuda.current_stream(self.device)
        generation = self._stager.lease(slot, compute_stream)
        if generation is None:
            raise RuntimeError(f"Async block {index} is already executing in another graph.")
        backward_handle = None
        try:
            if prefetch is not None:
                self._stage(prefetch, protected)
            self._buffers[slot].record_stream(compute_stream)
            values = dict(self._staged_tensors(slot, index, generation))
            values.update(trainable)
            if recomputing:
                # registered before the call: the checkpoint may stop the recomputation as soon
                # as the tensors it needs exist
                backward_handle = self._record_backward_use(slot, index, generation, completion_tensors)
            output = functional_call(self.layers[index], values, inputs, strict=True)
        except BaseException as error:
            # an early-stopped recomputation keeps its lease: the gradient hook ends it
            if not recomputing or not _is_checkpoint_early_stop(error):
                if backward_handle is not None:
                    backward_handle.remove()
                self._stager.release(slot, compute_stream)
            raise
        if not recomputing:
            self._stager.release(slot, compute_stream)
        return output

    def _checkpoint_contexts(self):
        return nullcontext(), self._recompute_context

    def block(
        self,
        index: int,
        *inputs: torch.Tensor,
        forward_prefetch: int | None,
        backward_prefetch: int | None,
        checkpoint_block: bool,
    ) -> torch.Tensor:
        """Run one streamed block and prefetch the next one in the direction of traversal."""
        if index not in self._blocks:
            raise ValueError(f"Block {index} is not configured for async streaming.")
        if not checkpoint_block:
            return self._run(index, inputs, self._blocks[index].trainable, (), forward_prefetch, backward_prefetch)

        count = len(inputs)
        names = tuple(self._blocks[index].trainable)
        # aliases give the gradient hook tensors that belong to this invocation alone
        input_aliases = tuple(tensor.view_as(tensor) if tensor.requires_grad else tensor for tensor in inputs)
        adapter_aliases = tuple(parameter.view_as(parameter) for parameter in self._blocks[index].trainable.values())

        def run(*arguments: torch.Tensor) -> torch.Tensor:
            adapters = dict(zip(names, arguments[count:]))
            completion = tuple(tensor for tensor in arguments if tensor.requires_grad)
            return self._run(index, arguments[:count], adapters, completion, forward_prefetch, backward_prefetch)

        return checkpoint(run, *input_aliases, *adapter_aliases, use_reentrant=False,
                          determinism_check=CHECKPOINT_CHECK,
                          context_fn=self._checkpoint_contexts)

    def close(self) -> None:
        """Finish owned transfers and release the staging slots."""
        if self._closed:
            return
        stats = self._stager.stats(timing=True)
        if not self._stager.destroy(force=False):
            raise RuntimeError("Cannot replace async block placement while a block backward is active.")
        self._final_stats = stats
        self._buffers = [None] * NUM_STAGING_SLOTS
        self._views = [None] * NUM_STAGING_SLOTS
        self._blocks.clear()
        self._closed = True

    def __del__(self) -> None:
        stager = getattr(self, "_stager", None)
        if stager is not None and not getattr(self, "_closed", True):
            try:
                stager.destroy(force=True)
            except Exception:  # interpreter teardown: the library may already be gone
                pass


def _is_lora_parameter(name: str) -> bool:
    return name.endswith("lora_A") or name.endswith("lora_B")


def _validate_placement(model: nn.Module, device: torch.device, blocks_to_swap: int, block_swap_mode: str) -> None:
    """Reject a placement before anything moves. Reference: training/memory.py:367-421."""
    if block_swap_mode not in {"sync", "async", "async_full"}:
        raise ValueError(
            "block_swap_mode must be 'sync' or 'async'. Full training additionally accepts 'async_full'.")
    if not 0 <= blocks_to_swap <= len(model.layers):
        raise ValueError("blocks_to_swap must be between zero and the number of joint blocks.")
    if block_swap_mode == "sync":
        return
    if device.type != "cuda":
        raise ValueError(f"{block_swap_mode} block swapping requires a CUDA device.")
    boundary = len(model.layers) - blocks_to_swap
    if block_swap_mode == "async_full":
        raise NotImplementedError(
            "async_full (streaming trainable full-precision blocks) is not provided by moss_image_b200; "
            "use block_swap_mode='async' with frozen base weights and LoRA adapters.")
    for index, layer in enumerate(model.layers):
        if index < boundary:
            continue
        for name, parameter in layer.named_parameters():
            if parameter.requires_grad and not _is_lora_parameter(name):
                raise ValueError(
                    "async block swapping is H2D-only and requires frozen base weights; "
                    f"only LoRA adapters may be trainable (found layers.{index}.{name}).")


def _swap_parameter_storage(parameter: nn.Parameter, moved: torch.Tensor) -> None:
    """Move a parameter without changing its identity (optimizers keep their references)."""
    replacement = nn.Parameter(moved, requires_grad=parameter.requires_grad)
    if parameter.grad is not None:
        replacement.grad = parameter.grad.detach().to(moved.device)
    torch.utils.swap_tensors(parameter, replacement)


def _align_bytes(offset: int, alignment: int = _ALIGNMENT) -> int:
    return -(-offset // alignment) * alignment


def _place_async_layer(layer: nn.Module, device: torch.device) -> _BlockTensors:
    """Adapters to the device; frozen parameters and buffers into one pinned master.

    Reference: training/memory.py:442-471. Every tensor starts on a 256-byte boundary of the
    master, so its view in a staging slot is aligned for the GEMM's vector and TMA loads.
    """
    parameters = dict(layer.named_parameters())
    buffers = dict(layer.named_buffers())
    trainable = {name: parameter for name, parameter in parameters.items() if parameter.requires_grad}
    for parameter in trainable.values():
        _swap_parameter_storage(parameter, parameter.detach().to(device))
    frozen = {name: parameter for name, parameter in parameters.items() if not parameter.requires_grad}
    frozen.update(buffers)
    views: dict[str, _TensorView] = {}
    offset = 0
    for name, tensor in frozen.items():
        offset = _align_bytes(offset)
        nbytes = tensor.numel() * tensor.element_size()
        views[name] = _TensorView(offset, nbytes, tensor.shape, tensor.dtype)
        offset += nbytes
    cpu_buffer = torch.empty(_align_bytes(offset), dtype=torch.uint8, pin_memory=True)
    modules = dict(layer.named_modules())
    for name, source in frozen.items():
        packed = _typed_view(cpu_buffer, views[name])
        packed.copy_(source.detach().to("cpu"))
        if name in parameters:
            _swap_parameter_storage(parameters[name], packed)
        else:
            owner, _, leaf = name.rpartition(".")
            modules[owner]._buffers[leaf] = packed
    return _BlockTensors(cpu_buffer=cpu_buffer, views=views, trainable=trainable)


def place_model(model: nn.Module, device: torch.device, blocks_to_swap: int, *, block_swap_mode: str = "sync") -> None:
    """Place a model resident, with synchronous CPU blocks, or with async frozen-block streaming.

    Reference: training/memory.py:474-532. A previous streamer is closed first; the model
    gets ``blocks_to_swap``, ``block_swap_mode`` and ``block_swap_manager`` attributes.
    """
    device = torch.device(device)
    _validate_placement(model, device, blocks_to_swap, block_swap_mode)
    existing = getattr(model, "block_swap_manager", None)
    if existing is not None:
        existing.close()
    model.blocks_to_swap = blocks_to_swap
    model.block_swap_mode = block_swap_mode
    model.block_swap_manager = None
    for name, child in model.named_children():
        if name != "layers":
            child.to(device)
    boundary = len(model.layers) - blocks_to_swap
    if block_swap_mode == "sync":
        for index, layer in enumerate(model.layers):
            layer.to("cpu" if index >= boundary else device)
        return
    packed: dict[int, _BlockTensors] = {}
    for index, layer in enumerate(model.layers):
        if index < boundary:
            layer.to(device)
        else:
            packed[index] = _place_async_layer(layer, device)
    if blocks_to_swap:
        model.block_swap_manager = AsyncBlockStreamer(model.layers, device, boundary, packed)

"""Data-parallel gradient exchange for the trainable (LoRA / full) parameters.

The reference trainer is single-process (training/train.py:554-557 rejects WORLD_SIZE != 1).
Each rank here runs an identical replica on its own samples; the only exchange is a
bucketed all-reduce (SUM, then / world) of the trainable gradients over NCCL, launched from
post-accumulate-grad hooks as soon as a bucket is complete so that it overlaps the rest of
backward. The same class runs on ``gloo`` for CPU tests.

Gradient accumulation (the reference's ``accum`` micro-batches, training/config.py:44 and
training/train.py:662): run every micro-batch but the last inside ``reducer.no_sync()``, so
their gradients only accumulate in ``param.grad``, then run the last one normally. Its hooks
send the buckets, and ``finish()`` averages what ``param.grad`` holds at that point.
"""

from __future__ import annotations

import contextlib
from typing import Iterable, Iterator

import torch
import torch.distributed as dist


class GradAllReducer:
    """Bucketed, hook-driven all-reduce of parameter gradients.

    Buckets are filled in reverse parameter order (the order backward produces them) and
    sent strictly in bucket order: a bucket goes out once it and every bucket before it are
    complete, and ``finish()`` sends whatever is left. Every rank therefore issues the same
    collectives in the same order, even when a parameter gets no gradient on some rank (its
    gradient is sent as zeros). Every rank must own the same parameters in the same order and
    call ``finish()`` once per optimizer step.

    A synchronised backward that changes a gradient whose bucket was already sent in the same
    step (a second backward without ``no_sync()``) raises ``RuntimeError``: the sum already on
    the wire would miss that contribution.

    With ``timing=True`` (CUDA parameters), ``finish()`` brackets its waits with CUDA events
    on the current stream; ``last_wait_ms()`` returns how long the compute stream stood still
    waiting for the exchange in the last step (the part of the all-reduce not hidden under
    backward).
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], *, bucket_bytes: int = 32 << 20,
                 group: dist.ProcessGroup | None = None, timing: bool = False) -> None:
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.buckets: list[list[torch.nn.Parameter]] = []
        current: list[torch.nn.Parameter] = []
        size = 0
        for p in reversed(self.params):
            current.append(p)
            size += p.numel() * p.element_size()
            if size >= bucket_bytes:
                self.buckets.append(current)
                current, size = [], 0
        if current:
            self.buckets.append(current)
        self.bucket_bytes = [sum(p.numel() * p.element_size() for p in b) for b in self.buckets]
        self._bucket_of = {id(p): i for i, b in enumerate(self.buckets) for p in b}
        self._seen: list[set[int]] = [set() for _ in self.buckets]
        self._next = 0  # first bucket not sent yet
        self._pending: list[tuple[dist.Work | None, torch.Tensor]] = []
        self._sync = True
        self._handles = []
        self.enabled = self.world > 1
        self.timing = timing
        self._events: tuple[torch.cuda.Event, torch.cuda.Event] | None = None
        self.sent_from_hooks = 0  # buckets sent during backward in the current step (overlapped)
        self.last_sent_from_hooks = 0  # the same count for the last finished step
        if self.enabled:
            for p in self.params:
                self._handles.append(p.register_post_accumulate_grad_hook(self._on_grad))

    @contextlib.contextmanager
    def no_sync(self) -> Iterator[None]:
        """Backward passes inside only accumulate into ``param.grad``; nothing is sent."""
        previous = self._sync
        self._sync = False
        try:
            yield
        finally:
            self._sync = previous

    def _on_grad(self, param: torch.nn.Parameter) -> None:
        if not self._sync:
            return
        index = self._bucket_of[id(param)]
        if index < self._next:
            raise RuntimeError(
                "GradAllReducer: a gradient changed after its bucket was sent in this step; run all "
                "micro-batches but the last inside reducer.no_sync().")
        self._seen[index].add(id(param))
        while self._next < len(self.buckets) and len(self._seen[self._next]) == len(self.buckets[self._next]):
            self._launch(self._next)
            self._next += 1
            self.sent_from_hooks += 1

    def _launch(self, index: int) -> None:
        bucket = self.buckets[index]
        for p in bucket:
            if p.grad is None:
                p.grad = torch.zeros_like(p)
        flat = torch.cat([p.grad.reshape(-1) for p in bucket])
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self._pending.append((work, flat))

    def finish(self) -> None:
        """Send the buckets not sent yet (in order), wait for all of them and average."""
        if not self.enabled:
            return
        start = end = None
        if self.timing and self.params and self.params[0].is_cuda:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
        while self._next < len(self.buckets):
            self._launch(self._next)
            self._next += 1
        for index, (work, flat) in enumerate(self._pending):
            if work is not None:
                work.wait()
            flat.div_(self.world)
            offset = 0
            for p in self.buckets[index]:
                n = p.numel()
                p.grad.copy_(flat[offset:offset + n].view_as(p.grad))
                offset += n
        if start is not None:
            end.record()
            self._events = (start, end)
        self.last_sent_from_hooks = self.sent_from_hooks
        self.sent_from_hooks = 0
        self._pending.clear()
        self._next = 0
        self._seen = [set() for _ in self.buckets]

    def last_wait_ms(self) -> float | None:
        """Device time the current stream spent in the last ``finish()`` (needs ``timing``)."""
        if self._events is None:
            return None
        start, end = self._events
        end.synchronize()
        return start.elapsed_time(end)

    def remove(self) -> None:
        for handle in self._handles:
            handle.remove()
        self._handles.clear()

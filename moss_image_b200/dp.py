"""Data-parallel gradient exchange for the trainable (LoRA / full) parameters.

The reference trainer is single-process (training/train.py:554-557 rejects WORLD_SIZE != 1).
Each rank here runs an identical replica on its own samples; the only exchange is a
bucketed all-reduce (SUM, then / world) of the trainable gradients over NCCL, launched from
post-accumulate-grad hooks as soon as a bucket is complete so that it overlaps the rest of
backward. The same class runs on ``gloo`` for CPU tests.
"""

from __future__ import annotations

from typing import Iterable

import torch
import torch.distributed as dist


class GradAllReducer:
    """Bucketed, hook-driven all-reduce of parameter gradients.

    Buckets are filled in reverse parameter order (the order backward produces them).
    ``finish()`` waits for every bucket and writes the averaged gradient back into
    ``param.grad``. Every rank must own the same parameters in the same order.
    """

    def __init__(self, params: Iterable[torch.nn.Parameter], *, bucket_bytes: int = 32 << 20,
                 group: dist.ProcessGroup | None = None) -> None:
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
        self._bucket_of = {id(p): i for i, b in enumerate(self.buckets) for p in b}
        self._ready = [0] * len(self.buckets)
        self._pending: list[tuple[int, dist.Work | None, torch.Tensor]] = []
        self._handles = []
        self.enabled = self.world > 1
        if self.enabled:
            for p in self.params:
                self._handles.append(p.register_post_accumulate_grad_hook(self._on_grad))

    def _on_grad(self, param: torch.nn.Parameter) -> None:
        index = self._bucket_of[id(param)]
        self._ready[index] += 1
        if self._ready[index] == len(self.buckets[index]):
            self._launch(index)

    def _launch(self, index: int) -> None:
        bucket = self.buckets[index]
        flat = torch.cat([p.grad.reshape(-1) for p in bucket])
        work = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)
        self._pending.append((index, work, flat))

    def finish(self) -> None:
        """Wait for all buckets (launching any whose hooks did not fire) and average."""
        if not self.enabled:
            return
        launched = {i for i, _, _ in self._pending}
        for index, bucket in enumerate(self.buckets):
            if index not in launched:
                for p in bucket:
                    if p.grad is None:
                        p.grad = torch.zeros_like(p)
                self._launch(index)
        for index, work, flat in sorted(self._pending, key=lambda item: item[0]):
            if work is not None:
                work.wait()
            flat.div_(self.world)
            offset = 0
            for p in self.buckets[index]:
                n = p.numel()
                p.grad.copy_(flat[offset:offset + n].view_as(p.grad))
                offset += n
        self._pending.clear()
        self._ready = [0] * len(self.buckets)

    def remove(self) -> None:
        for handle in self._handles:
            handle.remove()
        self._handles.clear()

"""Data-parallel gradient exchange on CPU ``gloo`` ranks (world size 2).

Checks that the hook-driven bucketed all-reduce gives every rank the average of the
per-rank gradients (what one process would compute on the union of the samples), with
buckets small enough that several are in flight, and that a rank whose parameter got no
gradient still takes part (zeros) so the ranks never diverge in collective order.

Gradient accumulation (the reference trainer's ``accum`` micro-batches,
training/train.py:662): two micro-batches per step, the first inside ``no_sync()``, with a
parameter that gets no gradient on one micro-batch of one rank only; the averaged gradient
must equal the single-process gradient over the union of all ranks' samples, and a second
synchronised backward in one step must raise instead of silently dropping a micro-batch.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model() -> nn.Module:
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(16, 32), nn.Tanh(), nn.Linear(32, 8), nn.Linear(8, 8))


def _inputs(rank: int) -> torch.Tensor:
    return torch.randn(4, 16, generator=torch.Generator().manual_seed(100 + rank))


def _worker(rank: int, world: int, port: int, skip_last: bool, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from moss_image_b200.dp import GradAllReducer

        model = _model()
        reducer = GradAllReducer(model.parameters(), bucket_bytes=512)
        assert len(reducer.buckets) >= 2
        out = model[:3](_inputs(rank)) if skip_last else model(_inputs(rank))
        out.square().sum().backward()
        reducer.finish()
        got = [p.grad.clone() for p in model.parameters()]
        # expected: average of the per-rank gradients, computed locally
        expected = None
        for r in range(world):
            ref = _model()
            o = ref[:3](_inputs(r)) if skip_last else ref(_inputs(r))
            o.square().sum().backward()
            grads = [p.grad.clone() if p.grad is not None else torch.zeros_like(p) for p in ref.parameters()]
            expected = grads if expected is None else [a + b for a, b in zip(expected, grads)]
        expected = [e / world for e in expected]
        ok = all(torch.allclose(a, b, atol=1e-6, rtol=1e-5) for a, b in zip(got, expected))
        queue.put((rank, ok))
    finally:
        dist.destroy_process_group()


def _micro_inputs(rank: int, micro: int) -> torch.Tensor:
    return torch.randn(3, 16, generator=torch.Generator().manual_seed(1000 + 10 * rank + micro))


def _micro_loss(model: nn.Module, rank: int, micro: int) -> torch.Tensor:
    # rank 1's second micro-batch skips the last layer: those parameters get no gradient there
    skip = rank == 1 and micro == 1
    out = model[:3](_micro_inputs(rank, micro)) if skip else model(_micro_inputs(rank, micro))
    return out.square().sum() / 2  # the trainer scales each micro-batch by 1 / accum


def _accum_worker(rank: int, world: int, port: int, queue) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from moss_image_b200.dp import GradAllReducer

        model = _model()
        reducer = GradAllReducer(model.parameters(), bucket_bytes=512)
        results = {}
        for step in range(2):  # the second step checks that the state resets between steps
            for p in model.parameters():
                p.grad = None
            with reducer.no_sync():
                _micro_loss(model, rank, 0).backward()
            _micro_loss(model, rank, 1).backward()
            reducer.finish()
            got = [p.grad.clone() for p in model.parameters()]
            expected = None
            ref = _model()
            for r in range(world):
                for micro in range(2):
                    _micro_loss(ref, r, micro).backward()
            expected = [p.grad / world for p in ref.parameters()]
            results[step] = all(torch.allclose(a, b, atol=1e-6, rtol=1e-5) for a, b in zip(got, expected))
        # misuse: a second synchronised backward in one step raises instead of dropping it
        _micro_loss(model, 0, 0).backward()
        try:
            _micro_loss(model, 0, 0).backward()
            raised = False
        except RuntimeError as error:
            raised = "no_sync" in str(error)
        reducer.finish()  # both ranks drain the same collectives
        queue.put((rank, (results[0], results[1], raised)))
    finally:
        dist.destroy_process_group()


def _spawn(target, extra_args) -> dict:
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, *extra_args, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(queue.get(timeout=5) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    return results


def test_accumulated_micro_batches_average_over_the_union_of_samples():
    results = _spawn(_accum_worker, ())
    assert results == {0: (True, True, True), 1: (True, True, True)}


@pytest.mark.parametrize("skip_last", [False, True])
def test_bucketed_allreduce_averages_gradients_across_ranks(skip_last):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, skip_last, queue)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    results = dict(queue.get(timeout=5) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}

"""CPU restatement of one checkpointed LoRA block step - TEST/BASELINE INFRASTRUCTURE ONLY.

Used by ``bench.py`` for the ``cpu_baseline`` leg and for ``--impl reference``: it times
the reference's own CPU algorithm for the hot path on the host cores:

* frozen int8 linear, eager branch of ``_FrozenInt8Linear`` (training/quantization.py:43 and
  :61-64): decode ``bf16(q) * bf16(s)`` (training/quantization.py:23-24) then a bf16 GEMM,
  input-gradient ``g @ dec(W)``;
* LoRA composition of ``LoRALinear.forward`` under bf16 autocast (training/lora.py:70-86);
* a block with the benchmark's structure (RMSNorm + modulation, q/k/v/o, joint attention,
  GELU MLP, gated residuals) run as gradient checkpointing does (training/model.py:687-709):
  a no-grad forward, then the recompute forward and the backward.

Weights are quantised with the oracle quantiser (numpy). Nothing here touches CUDA.
"""

from __future__ import annotations

import os
import time

import numpy as np
import torch
from torch.nn import functional as F

from . import oracle as O


def _dequantize(q: torch.Tensor, s: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """training/quantization.py:23-24."""
    return q.to(dtype) * s.to(dtype)[:, None]


class _EagerInt8Linear(torch.autograd.Function):
    """Eager branch of training/quantization.py:27-65."""

    @staticmethod
    def forward(ctx, tokens, q, s, bias, dtype):
        ctx.save_for_backward(q, s)
        ctx.dtype = dtype
        ctx.input_dtype = tokens.dtype
        return F.linear(tokens.to(dtype), _dequantize(q, s, dtype), bias)

    @staticmethod
    def backward(ctx, g):
        q, s = ctx.saved_tensors
        dx = g.to(ctx.dtype).matmul(_dequantize(q, s, ctx.dtype)).to(ctx.input_dtype)
        return dx, None, None, None, None


class _Linear:
    def __init__(self, out_f: int, in_f: int, gen: np.random.Generator, bias: bool, dtype: torch.dtype):
        w = (gen.standard_normal((out_f, in_f), dtype=np.float32) * np.float32(0.02))
        w = O.round_kind(w, O.BF16)  # the module is cast to bf16 before quantisation
        q, s, _ = O.quantize(w)
        self.q = torch.from_numpy(q)
        self.s = torch.from_numpy(s)
        self.bias = torch.zeros(out_f, dtype=dtype) if bias else None
        self.dtype = dtype

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return _EagerInt8Linear.apply(x, self.q, self.s, self.bias, self.dtype)


class _LoRA:
    """training/lora.py:70-86 with bf16 adapter math (autocast)."""

    def __init__(self, base: _Linear, rank: int, gen: np.random.Generator):
        self.base = base
        in_f = base.q.shape[1]
        out_f = base.q.shape[0]
        self.A = torch.from_numpy(gen.standard_normal((rank, in_f), dtype=np.float32) * np.float32(0.01)).requires_grad_()
        self.B = torch.zeros(out_f, rank, requires_grad=True)
        self.scale = 1.0

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        result = self.base(x)
        xb = x.to(torch.bfloat16)
        update = F.linear(F.linear(xb, self.A.to(torch.bfloat16)), self.B.to(torch.bfloat16))
        return result + update.to(result.dtype) * self.scale


def _rms(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    h = x.float()
    return (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


class CpuBlock:
    def __init__(self, dim: int, heads: int, mlp_dim: int, rank: int, seed: int = 0):
        gen = np.random.default_rng(seed)
        bf = torch.bfloat16
        self.dim, self.heads = dim, heads
        self.proj = {n: _LoRA(_Linear(dim, dim, gen, False, bf), rank, gen) for n in ("q", "k", "v", "o")}
        self.up = _Linear(mlp_dim, dim, gen, True, bf)
        self.down = _Linear(dim, mlp_dim, gen, True, bf)
        self.adaln = _Linear(6 * dim, dim, gen, True, bf)

    def parameters(self):
        for lora in self.proj.values():
            yield lora.A
            yield lora.B

    def __call__(self, tokens: torch.Tensor, cond: torch.Tensor) -> torch.Tensor:
        b, t, d = tokens.shape
        mod = self.adaln(F.silu(cond)).view(b, 6, d)
        sa, ca, ga, sf, cf, gf = (m.unsqueeze(1) for m in mod.unbind(1))
        h = _rms(tokens) * (1 + ca) + sa
        q = _rms(self.proj["q"](h).unflatten(-1, (self.heads, -1)))
        k = _rms(self.proj["k"](h).unflatten(-1, (self.heads, -1)))
        v = self.proj["v"](h).unflatten(-1, (self.heads, -1))
        att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        tokens = tokens + self.proj["o"](att.transpose(1, 2).flatten(2)) * ga
        h = _rms(tokens) * (1 + cf) + sf
        return tokens + self.down(F.gelu(self.up(h), approximate="tanh")) * gf


def time_block_sample(*, dim: int = 3072, heads: int = 24, mlp_dim: int = 12288, rank: int = 32,
                      seq: int = 4608, reps: int = 1, warmup: int = 0, threads: int | None = None) -> dict:
    """Time `reps` checkpointed fwd+bwd steps of one block on one sample (seconds each)."""
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    block = CpuBlock(dim, heads, mlp_dim, rank)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(1, seq, dim, generator=gen).to(torch.bfloat16)
    cond = torch.randn(1, dim, generator=gen).to(torch.bfloat16)
    g = torch.randn(1, seq, dim, generator=gen).to(torch.bfloat16)

    def step() -> None:
        with torch.autocast("cpu", dtype=torch.bfloat16):
            with torch.no_grad():
                block(x, cond)  # checkpointed forward (no saved activations)
            xi = x.detach().requires_grad_()
            out = block(xi, cond)  # recompute during backward
        out.backward(g)
        for p in block.parameters():
            p.grad = None

    for _ in range(warmup):
        step()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    return {"seconds": times, "threads": torch.get_num_threads(), "seq": seq}


def time_config1_ops(*, m: int = 4096, k: int = 3072, n: int = 3072, reps: int = 5, warmup: int = 2,
                     threads: int | None = None) -> dict:
    """The reference's CPU path for the benchmark's single-linear configuration, op by op.

    X bf16 [m, k] ~ N(0, 1), W [n, k] ~ N(0, 0.02) quantised per output channel (the oracle
    quantiser, training/quantization.py:87-91), bias bf16 zeros, dY bf16 [m, n] ~ N(0, 1):
    * forward: the eager ``F.linear(x, dec(W), bias)`` (training/quantization.py:43);
    * grad-input: ``dY @ dec(W)`` (training/quantization.py:61-64);
    * offload round trip of X: on CPU the reference's hooks are a no-op
      (training/activation_offload.py:92-93), so the pack/unpack pair is restated as the two
      host copies it would make: the dense payload into a new buffer (pack,
      training/activation_offload.py:123-126) and back into an ``empty_strided`` tensor
      (unpack, :139-147).
    Median seconds of ``reps`` after ``warmup`` untimed repetitions, on ``threads`` threads.
    """
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    gen = np.random.default_rng(0)
    w = gen.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    q, s, _ = O.quantize(w)
    qt, st = torch.from_numpy(q), torch.from_numpy(s)
    tg = torch.Generator().manual_seed(0)
    x = torch.randn(m, k, generator=tg).to(torch.bfloat16)
    dy = torch.randn(m, n, generator=tg).to(torch.bfloat16)
    bias = torch.zeros(n, dtype=torch.bfloat16)

    def fwd() -> None:
        F.linear(x, _dequantize(qt, st, torch.bfloat16), bias)

    def dx() -> None:
        dy.matmul(_dequantize(qt, st, torch.bfloat16))

    def round_trip() -> None:
        packed = torch.empty(x.shape, dtype=x.dtype)
        packed.copy_(x)
        restored = torch.empty_strided(x.shape, x.stride(), dtype=x.dtype)
        restored.copy_(packed)

    out = {"threads": torch.get_num_threads(), "shape": [m, k, n], "reps": reps, "warmup": warmup}
    for name, fn in (("fwd", fwd), ("dx", dx), ("offload_round_trip", round_trip)):
        for _ in range(warmup):
            fn()
        times = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        out[f"{name}_s"] = float(np.median(times))
    flops = 2.0 * m * n * k
    out["fwd_tflops"] = flops / out["fwd_s"] / 1e12
    out["dx_tflops"] = flops / out["dx_s"] / 1e12
    out["offload_round_trip_gbs"] = 2.0 * x.numel() * x.element_size() / out["offload_round_trip_s"] / 1e9
    return out


def cpu_model_name() -> str:
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"

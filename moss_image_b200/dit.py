"""Synthetic DiT block and block stack that host the int8 hot path (benchmark harness).

The shapes follow the benchmark configuration of this path: width 3072, 24 heads x 128,
joint attention over image + text tokens, MLP 3072 -> 12288 -> 3072 with GELU, and a
per-block adaLN modulation linear 3072 -> 6 x 3072. The block mirrors the structure of the
reference ``Block._forward_impl`` (training/model.py:269-314): RMSNorm + scale/shift
modulation, q/k/v projections with per-head RMSNorm on q and k, joint attention, gated
residual, modulated MLP with a gated residual. Every linear is a
:class:`~moss_image_b200.quantization.FrozenInt8Linear`; q/k/v/o carry LoRA adapters.

The stack wraps its forward in :func:`activation_cpu_offload` and checkpoints each block
(non-reentrant), as the reference trainer does with ``grad_checkpointing: true``
(training/model.py:687-709), so the offloaded tensors are the block inputs. Blocks may be
swapped or streamed with :func:`~moss_image_b200.memory.place_model`, and
:meth:`SyntheticDiT.forward_packed` runs a heterogeneous batch as one packed stream.
Per-sample modulation and gates are applied by the native segment kernels on CUDA
(:mod:`moss_image_b200.packed`). Attention uses torch's scaled-dot-product attention (library
code; the jagged, variable-length form for packed streams).
"""

from __future__ import annotations

import math

import torch
from torch import nn
from torch.nn import functional as F
from torch.utils.checkpoint import checkpoint

from .activation_offload import KEEP_RESIDENT, activation_cpu_offload
from .lora import LoRALinear
from .memory import offloaded_block
from .norms import rms_norm
from .packed import (
    CHECKPOINT_CHECK,
    batch_offsets,
    condition_for_tokens,
    cumulative_lengths,
    modulation_sample_indices,
    segment_gate,
    segment_modulate,
    sequence_lengths,
    varlen_attention,
)
from .quantization import quantize_frozen_linears


class RMSNorm(nn.Module):
    """Root-mean-square norm with a learned gain (training/model.py:154-172 arithmetic:
    f32 statistics, cast to the input dtype, then times the gain). CUDA inputs run the
    native norm kernels."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.is_cuda:
            return rms_norm(x, self.weight, self.eps)
        normalized = x.float() * torch.rsqrt(x.float().square().mean(-1, keepdim=True) + self.eps)
        return normalized.to(x.dtype) * self.weight


class SyntheticBlock(nn.Module):
    """One joint attention + MLP block with its own adaLN modulation linear."""

    def __init__(self, dim: int = 3072, heads: int = 24, mlp_dim: int = 12288) -> None:
        super().__init__()
        self.dim = dim
        self.heads = heads
        self.norm1 = RMSNorm(dim)
        self.norm2 = RMSNorm(dim)
        self.q_norm = RMSNorm(dim // heads)
        self.k_norm = RMSNorm(dim // heads)
        self.proj = nn.ModuleDict({name: nn.Linear(dim, dim, bias=False) for name in ("q", "k", "v", "o")})
        self.mlp_up = nn.Linear(dim, mlp_dim, bias=True)
        self.mlp_down = nn.Linear(mlp_dim, dim, bias=True)
        self.adaln = nn.Linear(dim, 6 * dim, bias=True)

    def forward(self, tokens: torch.Tensor, cond: torch.Tensor, cu_seqlens: torch.Tensor | None = None) -> torch.Tensor:
        """tokens: [B, T, dim] with cond [B, dim] (timestep embedding per sample), or a packed
        [1, total, dim] stream with cu_seqlens (int64 [S + 1]) and cond [S, dim].

        The conditioning follows training/model.py:288-312: ``norm(x) * (1 + scale) + shift``
        and ``x + branch * gate`` per sample, each op rounded in the activation dtype. On CUDA
        the per-sample conditions are applied by the native segment kernels; attention is
        block-diagonal over the packed sequences.
        """
        batch, seq, dim = tokens.shape
        sequences = cond.shape[0]
        modulation = self.adaln(F.silu(cond)).view(sequences, 6, dim)
        shift_a, scale_a, gate_a, shift_f, scale_f, gate_f = modulation.unbind(1)
        offsets = batch_offsets(batch, seq, tokens.device) if cu_seqlens is None else cu_seqlens
        if tokens.is_cuda:
            def modulate(x, scale, shift):
                return segment_modulate(x, scale, shift, offsets)

            def gated(x, branch, gate):
                return segment_gate(x, branch, gate, offsets)
        else:  # the reference's expansion (training/model.py:752-772)
            index = modulation_sample_indices(modulation, tokens, cu_seqlens)

            def modulate(x, scale, shift):
                return x * (1 + condition_for_tokens(scale, index)) + condition_for_tokens(shift, index)

            def gated(x, branch, gate):
                return x + branch * condition_for_tokens(gate, index)

        h = modulate(self.norm1(tokens), scale_a, shift_a)
        q = self.q_norm(self.proj["q"](h).unflatten(-1, (self.heads, -1)))
        k = self.k_norm(self.proj["k"](h).unflatten(-1, (self.heads, -1)))
        v = self.proj["v"](h).unflatten(-1, (self.heads, -1))
        if cu_seqlens is None:
            attended = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
            attended = attended.transpose(1, 2).flatten(2)
        else:
            attended = varlen_attention(q[0], k[0], v[0], offsets, sequence_lengths(cu_seqlens)).flatten(1)[None]
        tokens = gated(tokens, self.proj["o"](attended), gate_a)
        h = modulate(self.norm2(tokens), scale_f, shift_f)
        return gated(tokens, self.mlp_down(F.gelu(self.mlp_up(h), approximate="tanh")), gate_f)


class TimestepEmbedding(nn.Module):
    """Sinusoidal flow-matching time embedding followed by a small MLP (kept in fp32)."""

    def __init__(self, dim: int, freq_dim: int = 256) -> None:
        super().__init__()
        self.freq_dim = freq_dim
        self.mlp = nn.Sequential(nn.Linear(freq_dim, dim), nn.SiLU(), nn.Linear(dim, dim))

    def forward(self, t: torch.Tensor) -> torch.Tensor:
        half = self.freq_dim // 2
        freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=t.device, dtype=torch.float32) / half)
        phase = (1000.0 * t.float())[:, None] * freqs[None]
        emb = torch.cat((phase.cos(), phase.sin()), -1)
        return self.mlp(emb.to(self.mlp[0].weight.dtype))


class SyntheticDiT(nn.Module):
    """Stack of synthetic blocks with checkpointing and saved-activation offload."""

    def __init__(self, depth: int = 36, dim: int = 3072, heads: int = 24, mlp_dim: int = 12288,
                 gradient_checkpointing: bool = True) -> None:
        super().__init__()
        self.time_embedding = TimestepEmbedding(dim)
        self.layers = nn.ModuleList(SyntheticBlock(dim, heads, mlp_dim) for _ in range(depth))
        self.final_norm = RMSNorm(dim)
        self.gradient_checkpointing = gradient_checkpointing
        self.activation_offload = False

    def forward(self, tokens: torch.Tensor, timestep: torch.Tensor, skip_layers: tuple[int, ...] = ()) -> torch.Tensor:
        with activation_cpu_offload(self, self.activation_offload, tokens.device):
            cond = self.time_embedding(timestep).to(tokens.dtype)
            tokens = self._run_layers(tokens, cond, frozenset(skip_layers))
            return self.final_norm(tokens)

    def forward_packed(self, samples: list[torch.Tensor], timestep: torch.Tensor) -> list[torch.Tensor]:
        """One traversal over a heterogeneous batch: ``samples[i]`` is ``[tokens_i, dim]``.

        Mirrors ``forward_packed`` (training/model.py:502-626): the samples are concatenated
        into one ``[1, total, dim]`` stream with cumulative boundaries, every linear runs once
        over all tokens, attention is isolated per sample, and each sample keeps its own
        timestep conditioning. Returns the per-sample outputs.
        """
        if not samples:
            raise ValueError("forward_packed requires at least one sample.")
        device = samples[0].device
        if any(sample.ndim != 2 or sample.shape[0] == 0 or sample.device != device for sample in samples):
            raise ValueError("Each packed sample must be a non-empty [tokens, dim] tensor on one device.")
        lengths = [sample.shape[0] for sample in samples]
        times = torch.as_tensor(timestep, device=device).reshape(-1).expand(len(samples))
        cu_seqlens = cumulative_lengths(lengths, device)
        cu_seqlens.moss_lengths = tuple(lengths)  # known on the host: no device read per block
        setattr(cu_seqlens, KEEP_RESIDENT, True)  # the same boundaries tensor in every recomputation
        tokens = torch.cat(samples, 0).unsqueeze(0)
        with activation_cpu_offload(self, self.activation_offload, device):
            cond = self.time_embedding(times).to(tokens.dtype)
            tokens = self._run_layers(tokens, cond, frozenset(), cu_seqlens)
            return list(self.final_norm(tokens)[0].split(lengths, 0))

    def _run_layers(self, tokens: torch.Tensor, cond: torch.Tensor, skipped: frozenset[int],
                    cu_seqlens: torch.Tensor | None = None) -> torch.Tensor:
        """Resident, synchronously swapped or streamed blocks, as ``place_model`` left them.

        Mirrors training/model.py:672-709: blocks at or past ``len(layers) - blocks_to_swap``
        run through the streamer (prefetching the next streamed block in the direction of
        traversal, checkpointed whenever gradients are enabled) or, without a streamer,
        from their CPU masters; the others are checkpointed when training.
        """
        boundary = len(self.layers) - getattr(self, "blocks_to_swap", 0)
        manager = getattr(self, "block_swap_manager", None)
        streamed = [index for index in range(boundary, len(self.layers)) if index not in skipped]
        position = {index: slot for slot, index in enumerate(streamed)}
        for index, layer in enumerate(self.layers):
            if index in skipped:
                continue
            inputs = (tokens, cond) if cu_seqlens is None else (tokens, cond, cu_seqlens)
            if manager is not None and index >= boundary:
                at = position[index]
                tokens = manager.block(
                    index, *inputs,
                    forward_prefetch=streamed[at + 1] if at + 1 < len(streamed) else None,
                    backward_prefetch=streamed[at - 1] if at else None,
                    checkpoint_block=torch.is_grad_enabled(),
                )
            elif index >= boundary:
                tokens = offloaded_block(layer, *inputs)
            elif self.gradient_checkpointing and self.training and torch.is_grad_enabled():
                tokens = checkpoint(layer, *inputs, use_reentrant=False, determinism_check=CHECKPOINT_CHECK)
            else:
                tokens = layer(*inputs)
        return tokens


def inject_lora(model: nn.Module, rank: int, alpha: float, targets: tuple[str, ...] = ("q", "k", "v", "o"),
                a_std: float | None = 0.01) -> list[str]:
    """Wrap the named projections of every block in :class:`LoRALinear`.

    A ~ N(0, a_std) (the benchmark's adapter init; ``None`` keeps the reference's Kaiming
    init), B = 0. Returns the wrapped module paths.
    """
    names = []
    for index, layer in enumerate(model.layers):
        _inject_block(layer, rank, alpha, targets, a_std)
        names.extend(f"layers.{index}.proj.{name}" for name in targets)
    return names


def _inject_block(layer: SyntheticBlock, rank: int, alpha: float, targets: tuple[str, ...],
                  a_std: float | None) -> None:
    for name in targets:
        base = layer.proj[name]
        wrapped = LoRALinear(base, rank, alpha).to(device=base.weight.device)
        if a_std is not None:
            with torch.no_grad():
                wrapped.lora_A.normal_(0.0, a_std)
        layer.proj[name] = wrapped


def build_lora_model(depth: int, *, device: torch.device, dim: int = 3072, heads: int = 24, mlp_dim: int = 12288,
                     rank: int = 32, alpha: float | None = None, seed: int = 0,
                     dtype: torch.dtype = torch.bfloat16, full_qkvo: bool = False) -> SyntheticDiT:
    """Random-init stack (weights ~ N(0, 0.02)), int8 base, LoRA on q/k/v/o.

    Mirrors the trainer's order (training/train.py:577-589): build, cast, inject LoRA,
    quantise the frozen linears - done block by block on the device so that the
    full-precision weights of only one block exist at a time.

    With ``full_qkvo`` the q/k/v/o projections are trained in full instead (trainable
    ``dtype`` masters, no adapters) and every other linear is frozen int8: the hybrid that
    ``quantize_frozen_linears`` allows at module level (training/quantization.py:156-157;
    the reference trainer itself only pairs int8 bases with LoRA, training/train.py:543-545).
    """
    torch.manual_seed(seed)
    alpha = float(rank if alpha is None else alpha)
    model = SyntheticDiT(depth=0, dim=dim, heads=heads, mlp_dim=mlp_dim)
    model.time_embedding.to(device=device, dtype=dtype)
    model.final_norm.to(device=device, dtype=dtype)
    model.requires_grad_(False)
    quantize_frozen_linears(model.time_embedding)
    layers = []
    for _ in range(depth):
        block = SyntheticBlock(dim, heads, mlp_dim).to(device=device)
        with torch.no_grad():
            for module in block.modules():
                if isinstance(module, nn.Linear):
                    module.weight.normal_(0.0, 0.02)
                    if module.bias is not None:
                        module.bias.zero_()
        block.to(dtype=dtype)
        block.requires_grad_(False)
        if full_qkvo:
            for name in ("q", "k", "v", "o"):
                block.proj[name].requires_grad_(True)
        else:
            _inject_block(block, rank, alpha, ("q", "k", "v", "o"), 0.01)
        quantize_frozen_linears(block)
        layers.append(block)
    model.layers = nn.ModuleList(layers)
    return model


def packed_flow_matching_loss(model: SyntheticDiT, latents: list[torch.Tensor], text: list[torch.Tensor],
                              t: torch.Tensor, noise: list[torch.Tensor]) -> torch.Tensor:
    """The flow-matching loss of a heterogeneous batch in one packed traversal.

    ``latents[i]``/``noise[i]``: ``[image_tokens_i, dim]``; ``text[i]``: ``[text_tokens_i, dim]``.
    Each sample's loss is its mean over its image tokens; the batch loss is their mean.
    """
    samples = []
    for latent, context, noise_i, sigma in zip(latents, text, noise, t):
        sigma = sigma.to(latent.dtype)
        samples.append(torch.cat(((1 - sigma) * latent + sigma * noise_i, context), 0))
    outputs = model.forward_packed(samples, t)
    losses = [F.mse_loss(out[: latent.shape[0]].float(), (noise_i - latent).float())
              for out, latent, noise_i in zip(outputs, latents, noise)]
    return torch.stack(losses).mean()


def flow_matching_loss(model: SyntheticDiT, latents: torch.Tensor, text: torch.Tensor, t: torch.Tensor,
                       noise: torch.Tensor) -> torch.Tensor:
    """Rectified-flow velocity loss on the image tokens (text tokens are conditioning)."""
    sigma = t.view(-1, 1, 1).to(latents.dtype)
    noisy = (1 - sigma) * latents + sigma * noise
    tokens = torch.cat((noisy, text), dim=1)
    pred = model(tokens, t)[:, : latents.shape[1]]
    target = noise - latents
    return F.mse_loss(pred.float(), target.float())

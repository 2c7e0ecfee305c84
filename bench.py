"""Benchmark of the int8 weight-only DiT LoRA training step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the per-GPU shape of the benchmark's 1/2/4/8-GPU configuration): a 36-block
synthetic DiT (width 3072, 24 heads x 128, MLP 3072 -> 12288 -> 3072 GELU, per-block adaLN
3072 -> 18432), every linear int8 weight-only, LoRA rank 32 on q/k/v/o, batch 2 x (4096
image + 512 text) tokens per GPU, bf16 autocast, gradient checkpointing per block, saved
activations offloaded to the pinned-host ring, AdamW on the adapters, and (N > 1) a
bucketed NCCL all-reduce of the adapter gradients. One "step" is one such training step.

Rank 0 prints one JSON line: whole-job tokens/s with inputs resident in HBM (``value``),
the same through host buffers (``e2e``), the roofline of the dominant kernel (the int8
GEMM, every launch timed with CUDA events inside the timed region), the CPU baseline
(the reference's CPU algorithm restated in ``oracle/``, timed on this host), SM clocks
sampled during the timed region, and the number of this library's kernel launches.

``--impl reference`` times the reference's CPU implementation of the same step (rank 0
only) and prints the same kind of line with ``"impl": "reference"``.
``--kernel gemm_fwd|gemm_dx --m M --k K --n N`` runs only the int8 GEMM (profiling aid).
``--sweep`` runs the GEMM sweep (M x (K, N) grid) and prints one JSON line per case.
``--blocks-to-swap N`` streams the frozen int8 weights of the last N blocks from pinned host
memory through the block stager (``place_model(..., block_swap_mode="async")``) and adds a
``block_swap`` object (copy-engine GB/s against the host link); ``--img-tokens``/``--txt-tokens``
change the per-sample token counts (e.g. 16384 + 4096 for 2048^2 images).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
METRIC = "INT8-W DiT train tokens/s at 1/2/4/8 B200; W8 GEMM TFLOP/s; offload GB/s"
IMG_TOKENS, TXT_TOKENS, DIM, HEADS, MLP, DEPTH, BATCH, RANK = 4096, 512, 3072, 24, 12288, 36, 2, 32


def parse_args() -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--depth", type=int, default=DEPTH)
    p.add_argument("--batch", type=int, default=BATCH)
    p.add_argument("--no-offload", action="store_true")
    p.add_argument("--blocks-to-swap", type=int, default=0,
                   help="stream the frozen int8 weights of the last N blocks from pinned host memory (async)")
    p.add_argument("--packed", default=None,
                   help="heterogeneous batch 'img:txt,img:txt,...': time one packed traversal against per-sample ones")
    p.add_argument("--no-numa-bind", action="store_true",
                   help="do not restrict each rank to the CPU cores local to its GPU")
    p.add_argument("--full-qkvo", action="store_true",
                   help="train the q/k/v/o projections in full (bf16 masters) instead of LoRA; other linears int8")
    p.add_argument("--img-tokens", type=int, default=IMG_TOKENS)
    p.add_argument("--txt-tokens", type=int, default=TXT_TOKENS)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--offload-pairs", type=int, default=2,
                   help="alternated (offload off, offload on) arm pairs timed after the main region (0: none)")
    p.add_argument("--offload-arm-steps", type=int, default=3)
    p.add_argument("--offload-defer-mb", type=int, default=1536,
                   help="keep up to this many MiB of the newest saved activations on the GPU (copied out only when "
                        "newer ones push them past the budget)")
    p.add_argument("--kernel", choices=["gemm_fwd", "gemm_dx", "hadamard", "convrot_fwd", "convrot_dx",
                                        "convrot_dx_separate", "comfy_load",
                                        "segment_modulate", "segment_gate", "rmsnorm", "rmsnorm_bwd"], default=None)
    p.add_argument("--group", type=int, default=256, help="ConvRot / Hadamard group size")
    p.add_argument("--m", type=int, default=9216)
    p.add_argument("--k", type=int, default=3072)
    p.add_argument("--n", type=int, default=3072)
    p.add_argument("--sweep", action="store_true")
    p.add_argument("--no-ref-gpu-arm", action="store_true",
                   help="skip timing the step with the reference's own modules after a 1-GPU run")
    p.add_argument("--ref-gpu-modules", action="store_true",
                   help="the training step with the reference's own int8 linears (Triton backend), LoRA and "
                        "activation offload from baseline/_ref swapped into the same model (1 GPU)")
    p.add_argument("--sweep-m", default=None, help="comma-separated M values of the sweep (default: the config grid)")
    return p.parse_args()


def measured_peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: str) -> None:
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        loaded = [s for s, p in zip(sm, power) if p > 0.3 * max(power)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power)}


# ----------------------------------------------------------------------------- GEMM timing
class GemmTimer:
    """Launch observer: CUDA events around every int8 GEMM launch on its stream."""

    def __init__(self) -> None:
        import torch

        self.torch = torch
        self.records: list[tuple[str, int, int, int, object, object]] = []
        self.active = False

    def __call__(self, kind, m, n, k, device):
        if not self.active:
            return None
        torch = self.torch
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        stream = torch.cuda.current_stream(device)
        start.record(stream)

        def done():
            end.record(stream)
            self.records.append((kind, m, n, k, start, end))

        return done

    def summary(self) -> dict:
        out = {}
        for kind in ("fwd", "dx"):
            recs = [r for r in self.records if r[0] == kind]
            if not recs:
                continue
            total_ms = sum(r[4].elapsed_time(r[5]) for r in recs)
            flops = sum(2.0 * r[1] * r[2] * r[3] for r in recs)
            bytes_ = sum(r[2] * r[3] + 4 * r[2] + 2 * r[1] * r[3] + 2 * r[1] * r[2] for r in recs)
            out[kind] = {"launches": len(recs), "total_ms": total_ms, "flops": flops, "bytes": bytes_,
                         "avg_us": 1e3 * total_ms / len(recs)}
        return out


def load_traffic(kind: str) -> float | None:
    path = REPO / "profiles" / f"w8a16_gemm_{kind}_traffic.json"
    if path.exists():
        try:
            return float(json.loads(path.read_text())["traffic_bytes_per_launch_at_bench_shape"])
        except (KeyError, ValueError):
            return None
    return None


def host_link_gbs(dev, nbytes: int = 256 << 20, reps: int = 5) -> float:
    """Best pinned-host -> device copy rate of one plain copy-engine transfer (GB/s)."""
    import torch

    host = torch.empty(nbytes, dtype=torch.uint8, pin_memory=True)
    device = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    best = float("inf")
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        device.copy_(host, non_blocking=True)
        b.record()
        b.synchronize()
        best = min(best, a.elapsed_time(b))
    return nbytes / (best * 1e-3) / 1e9


def block_swap_summary(before: dict, after: dict, steps: int, elapsed_ms: float, dev) -> dict:
    """Streamed-weight traffic of the timed region against the host link's copy rate."""
    copies = after["copies"] - before["copies"]
    nbytes = after["bytes"] - before["bytes"]
    copy_ms = after["copy_ms"] - before["copy_ms"]
    timed = after["timed_bytes"] - before["timed_bytes"]
    link = host_link_gbs(dev)
    engine = timed / (copy_ms * 1e-3) / 1e9 if copy_ms > 0 else None
    return {"copies_per_step": copies / steps, "bytes_per_step": nbytes / steps,
            "copy_engine_gbs": engine, "host_link_gbs": link,
            "frac_of_host_link": engine / link if engine else None,
            "link_busy_frac_of_step": copy_ms / elapsed_ms,
            "note": "copy_engine_gbs: block bytes / summed copy time of the stager's H2D transfers (CUDA events on "
                    "its copy stream); host_link_gbs: best plain 256 MiB pinned->device copy on an idle GPU"}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_baseline_sample(reps: int = 5, warmup: int = 2) -> dict:
    """The reference's CPU algorithm on this host: one checkpointed block step on one sample
    (median of `reps` after `warmup`), plus the single-linear configuration op by op."""
    sys.path.insert(0, str(REPO))
    from oracle import cpu_step

    seq = IMG_TOKENS + TXT_TOKENS
    result = cpu_step.time_block_sample(dim=DIM, heads=HEADS, mlp_dim=MLP, rank=RANK, seq=seq, reps=reps,
                                        warmup=warmup)
    per_block = statistics.median(result["seconds"])
    value = seq / (per_block * DEPTH)  # tokens/s of the full 36-block step, per sample
    ops = cpu_step.time_config1_ops(reps=reps, warmup=warmup)
    return {"value": value, "unit": "tokens/s", "cores": result["threads"], "kind": "port",
            "sample": (f"1 of {DEPTH} blocks x 1 sample ({seq} tokens), checkpointed fwd + recompute + bwd, "
                       f"median of {reps} after {warmup} warm-ups; value = {seq} tokens / ({DEPTH} x the block "
                       f"time); cpu={cpu_step.cpu_model_name()}, os.cpu_count()={os.cpu_count()}"),
            "seconds_per_block_sample": per_block, "extrapolated_x": DEPTH,
            "config1_ops": ops}


def run_reference(args: argparse.Namespace) -> None:
    """The reference's CPU implementation of the step, on this host's cores.

    Each timed step is a bounded sample of the workload: one of the 36 blocks on one of the
    2 samples, run as gradient checkpointing runs it (no-grad forward, recompute forward,
    backward). ``ms_per_step`` is that sample's measured time; ``value`` converts it to the
    metric's tokens/s of a full step, which is ``extrapolated_x`` = 36 blocks x 2 samples
    such samples long.
    """
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, str(REPO))
    from oracle import cpu_step

    seq = IMG_TOKENS + TXT_TOKENS
    steps = max(1, args.steps)
    t0 = time.perf_counter()
    result = cpu_step.time_block_sample(dim=DIM, heads=HEADS, mlp_dim=MLP, rank=RANK, seq=seq,
                                        reps=steps, warmup=args.warmup)
    wall = time.perf_counter() - t0
    per_sample = statistics.median(result["seconds"])
    value = seq / (per_sample * DEPTH)
    extrapolated = DEPTH * args.batch
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": steps, "warmup": args.warmup, "ms_per_step": per_sample * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": (f"reference CPU path (oracle port of the eager int8 LoRA block) on the "
                                f"{DEPTH}-block step, batch {args.batch} x {seq} tokens; each timed step is a "
                                f"bounded sample: 1 block x 1 sample"),
                   "global_batch": args.batch, "seq_len": seq, "parallelism": "cpu"},
        "step_is_sample": True,
        "extrapolated_x": extrapolated,
        "full_step_ms_extrapolated": per_sample * extrapolated * 1e3,
        "wall_s": wall,
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": result["threads"], "kind": "port",
                         "sample": (f"each step: 1 of {DEPTH} blocks x 1 of {args.batch} samples, checkpointed "
                                    f"fwd + recompute + bwd, median of {steps} after {args.warmup} warm-ups; "
                                    f"value = {seq} tokens / ({DEPTH} x the sample time); "
                                    f"cpu={cpu_step.cpu_model_name()}")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- kernel-only modes
def run_comfy_load(args: argparse.Namespace) -> None:
    """Load one block's worth of Comfy int8_tensorwise linears: dense decode + re-quantise
    (what a decode-only loader leads to) against keeping the stored codes."""
    import torch

    from moss_image_b200.comfy_weights import decode_comfy_state, split_comfy_state
    from moss_image_b200.quantization import FrozenInt8Linear

    dev = torch.device("cuda", 0)
    shapes = {"q": (DIM, DIM), "k": (DIM, DIM), "v": (DIM, DIM), "o": (DIM, DIM), "up": (MLP, DIM),
              "down": (DIM, MLP), "adaln": (6 * DIM, DIM)}
    gen = torch.Generator().manual_seed(0)
    marker = torch.tensor(list(b'{"format": "int8_tensorwise"}'), dtype=torch.uint8)
    state = {}
    for name, (n, k) in shapes.items():
        state[f"{name}.weight"] = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
        state[f"{name}.weight_scale"] = (torch.rand(n, 1, generator=gen) * 2e-4 + 1e-4).float()
        state[f"{name}.comfy_quant"] = marker
    nbytes = sum(n * k for n, k in shapes.values())

    def via_dense():
        dense = decode_comfy_state(state, torch.bfloat16)
        out = {}
        for name in shapes:
            linear = torch.nn.Linear(1, 1, bias=False)
            linear.weight = torch.nn.Parameter(dense[f"{name}.weight"].to(dev), requires_grad=False)
            linear.in_features, linear.out_features = shapes[name][1], shapes[name][0]
            out[name] = FrozenInt8Linear(linear)
        torch.cuda.synchronize()
        return out

    def direct():
        quantized, _ = split_comfy_state(state)
        out = {name: FrozenInt8Linear.from_codes(w.codes.to(dev), w.scale.reshape(-1).to(dev))
               for name, w in quantized.items()}
        torch.cuda.synchronize()
        return out

    results = {}
    for label, fn in (("decode_requantize", via_dense), ("direct", direct)):
        fn()
        times = []
        for _ in range(max(1, args.steps)):
            t0 = time.perf_counter()
            modules = fn()
            times.append(time.perf_counter() - t0)
        results[label] = {"ms": 1e3 * statistics.median(times)}
        moved = sum(int((modules[n].weight_int8.cpu() != state[f"{n}.weight"]).sum()) for n in shapes)
        results[label]["codes_changed_frac"] = moved / nbytes
    print(json.dumps({"kernel": "comfy_load", "block_linears": len(shapes), "int8_bytes": nbytes,
                      "threads": torch.get_num_threads(), **results,
                      "speedup": results["decode_requantize"]["ms"] / results["direct"]["ms"]}), flush=True)


def run_kernel(args: argparse.Namespace) -> None:
    import torch

    from moss_image_b200 import quant_kernels as qk

    if args.kernel == "comfy_load":
        run_comfy_load(args)
        return

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    m, k, n = args.m, args.k, args.n
    gen = torch.Generator(device=dev).manual_seed(0)
    w = torch.randn(n, k, device=dev, generator=gen) * 0.02
    q, s = qk.quantize_weight(w)
    del w
    if args.kernel == "gemm_fwd":
        x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
        fn = lambda: qk.int8_linear_forward(x, q, s, None, torch.bfloat16, torch.bfloat16)  # noqa: E731
    elif args.kernel == "hadamard":
        x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
        y = torch.empty_like(x)
        fn = lambda: qk.hadamard_transform(x, args.group, out=y)  # noqa: E731
    elif args.kernel == "convrot_fwd":
        x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
        fn = lambda: qk.convrot_forward(x, q, s, None, torch.bfloat16, torch.bfloat16, args.group)  # noqa: E731
    elif args.kernel in ("convrot_dx", "convrot_dx_separate"):
        dy = torch.randn(m, n, device=dev, generator=gen).to(torch.bfloat16)
        if args.kernel == "convrot_dx":  # rotation in the grad-input GEMM's epilogue where it applies
            fn = lambda: qk.convrot_backward(dy, q, s, torch.Size((m, k)), torch.bfloat16,  # noqa: E731
                                             torch.bfloat16, args.group)
        else:  # the GEMM, then the rotation kernel over its output
            def fn():
                dx = qk.int8_linear_backward(dy, q, s, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)
                return qk.hadamard_transform(dx, args.group, out=dx)
    elif args.kernel in ("rmsnorm", "rmsnorm_bwd"):
        from moss_image_b200.norms import rms_norm

        x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16).requires_grad_(args.kernel == "rmsnorm_bwd")
        wn = torch.ones(k, device=dev, dtype=torch.bfloat16)
        if args.kernel == "rmsnorm":
            fn = lambda: rms_norm(x, wn)  # noqa: E731
        else:
            yn = rms_norm(x, wn)
            dyn = torch.randn_like(yn)
            fn = lambda: torch.autograd.grad(yn, x, dyn, retain_graph=True)  # noqa: E731
    elif args.kernel in ("segment_modulate", "segment_gate"):
        from moss_image_b200 import packed

        x = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
        u = torch.randn(m, k, device=dev, generator=gen).to(torch.bfloat16)
        modulation = torch.randn(2, 6, k, device=dev, generator=gen).to(torch.bfloat16)
        offsets = packed.cumulative_lengths([m // 2, m - m // 2], dev)
        if args.kernel == "segment_modulate":
            fn = lambda: packed.segment_modulate(x, modulation[:, 1], modulation[:, 0], offsets)  # noqa: E731
        else:
            fn = lambda: packed.segment_gate(x, u, modulation[:, 2], offsets)  # noqa: E731
    else:
        dy = torch.randn(m, n, device=dev, generator=gen).to(torch.bfloat16)
        fn = lambda: qk.int8_linear_backward(dy, q, s, torch.Size((m, k)), torch.bfloat16, torch.bfloat16)  # noqa: E731
    for _ in range(max(args.warmup, 1)):
        fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        fn()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / args.steps
    qk.check_device_status(dev)
    line = {"kernel": args.kernel, "m": m, "k": k, "n": n, "us": ms * 1e3}
    if args.kernel == "hadamard":
        line["gbs"] = 2.0 * m * k * 2 / ms / 1e6  # one bf16 read and one write
        line["group"] = args.group
    elif args.kernel.startswith("segment_") or args.kernel.startswith("rmsnorm"):
        # bf16 rows read + written: modulate and norm forward 2, gate and norm backward 3
        streams = 2 if args.kernel in ("segment_modulate", "rmsnorm") else 3
        line["gbs"] = streams * m * k * 2 / ms / 1e6
    else:
        line["tflops"] = 2.0 * m * n * k / ms / 1e9
    print(json.dumps(line), flush=True)


def graph_time_us(calls, device, reps: int | None = None) -> float:
    """Device time per launch of back-to-back launches: every call in `calls` enqueues one
    launch on the current stream; they are captured once in a CUDA graph (no host work between
    launches) and the graph is replayed after warm-up, timed with CUDA events."""
    import torch

    stream = torch.cuda.Stream(device)
    # the inputs were produced on the current stream, and freed temporaries of that stream may
    # back the outputs: the side stream starts only after that work
    torch.cuda.synchronize(device)
    with torch.cuda.stream(stream):
        for call in calls:  # one-time set-up (attributes, symbol lookups) outside the capture
            call()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for call in calls:
            call()
    graph.replay()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if reps is None:
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        once = max(start.elapsed_time(end), 1e-3)
        reps = int(min(10, max(2, 30.0 / once)))
    for _ in range(2):
        graph.replay()
    start.record()
    for _ in range(reps):
        graph.replay()
    end.record()
    end.synchronize()
    us = start.elapsed_time(end) * 1e3 / (reps * len(calls))
    del graph
    return us


def reference_triton_kernels():
    """The reference's own Triton W8A16 kernels (training/quant_kernels.py:294-373), imported
    from the reference package installed under baseline/_ref (pip --target, no deps). Returns
    (module, None), or (None, why) when the install or Triton is missing."""
    ref_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "baseline", "_ref")
    if not os.path.isfile(os.path.join(ref_dir, "training", "quant_kernels.py")):
        return None, "reference package not installed under baseline/_ref"
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        from training import quant_kernels as ref_qk
    except Exception as error:  # the comparator is optional; the sweep still runs without it
        return None, f"reference quant_kernels import failed: {error}"
    if getattr(ref_qk, "triton", None) is None:
        return None, "Triton is not importable"
    return ref_qk, None


def run_sweep(args: argparse.Namespace) -> None:
    """The W8A16 GEMM sweep (M x (K, N), forward and grad-input), one JSON line per shape.

    Four implementations on the same GPU, each timed as back-to-back launches captured in a
    CUDA graph (device time only, no host launch latency):
    * ``ours``: this library's kernels through the C ABI, preallocated buffers and workspace;
    * ``ref_triton``: the reference's own Triton kernels (``triton_int8_linear_forward`` /
      ``_backward``, training/quant_kernels.py:294-373, 32 x 32 x 32 tiles), when the
      reference package is installed under baseline/_ref, with preallocated outputs;
    * ``eager_gpu``: the reference's eager algorithm (decode ``q.to(bf16) * s.to(bf16)[:, None]``
      then ``F.linear`` / ``matmul`` on cuBLAS, training/quantization.py:23-24,43,61-64);
    * ``cublas_bf16``: a plain bf16 cuBLAS GEMM on a dense bf16 weight (the ceiling).
    Every launch reads its own copy of the weight, with enough copies that the weights touched
    by one graph exceed twice the 126 MB L2: the weight stream is measured from HBM. Each cell
    also reports the relative Frobenius difference between our output and the reference
    Triton kernel's on the same inputs.
    """
    import ctypes

    import torch
    import torch.nn.functional as F

    from moss_image_b200 import _lib
    from moss_image_b200 import quant_kernels as qk

    peaks, peak_kind = measured_peaks()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.library()
    status = qk.status_buffer(dev)
    l2_cover = 320 << 20
    grid_m = [int(v) for v in args.sweep_m.split(",")] if args.sweep_m else [128, 512, 2048, 8192, 32768]
    ref_qk, ref_missing = reference_triton_kernels()
    if ref_missing:
        print(json.dumps({"ref_triton": "unavailable", "why": ref_missing}), flush=True)
    for k, n in [(3072, 3072), (3072, 9216), (3072, 12288), (12288, 3072), (3072, 18432)]:
        copies = max(1, -(-l2_cover // (n * k)))
        dense_copies = max(1, -(-l2_cover // (2 * n * k)))
        gen = torch.Generator(device=dev).manual_seed(0)
        qs = [torch.randint(-127, 128, (n, k), generator=gen, device=dev, dtype=torch.int8) for _ in range(copies)]
        ss = [torch.rand(n, generator=gen, device=dev) * 4e-4 + 1e-4 for _ in range(copies)]
        dense = [(qs[i % copies].to(torch.bfloat16) * ss[i % copies].to(torch.bfloat16)[:, None])
                 for i in range(dense_copies)]
        for m in grid_m:
            x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
            dy = torch.randn(m, n, generator=gen, device=dev).to(torch.bfloat16)
            y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
            dx = torch.empty(m, k, device=dev, dtype=torch.bfloat16)
            res = {"m": m, "k": k, "n": n, "weight_copies": copies}
            flops = 2.0 * m * n * k
            for kind in ("fwd", "dx"):
                n_out, k_red = (n, k) if kind == "fwd" else (k, n)
                size = ctypes.c_size_t()
                _lib.check(lib.moss_w8a16_gemm_workspace_bytes(m, n_out, k_red, ctypes.byref(size)), "workspace")
                ws_owner = torch.empty(size.value + 256, dtype=torch.uint8, device=dev)
                ws = (ws_owner.data_ptr() + 255) // 256 * 256

                def ours(i, kind=kind, size=size, ws=ws):
                    stream = torch.cuda.current_stream(dev).cuda_stream
                    if kind == "fwd":
                        rc = lib.moss_w8a16_gemm_fwd(x.data_ptr(), 1, m, k, qs[i].data_ptr(), ss[i].data_ptr(), 1, n,
                                                     None, 0, None, None, 0, 0, 1.0, y.data_ptr(), 1, ws, size.value,
                                                     status.data_ptr(), stream)
                    else:
                        rc = lib.moss_w8a16_gemm_dx(dy.data_ptr(), 1, m, n, qs[i].data_ptr(), ss[i].data_ptr(), 1, k,
                                                    None, None, 0, 0, 1.0, dx.data_ptr(), 1, ws, size.value,
                                                    status.data_ptr(), stream)
                    _lib.check(rc, "gemm")

                def eager(i, kind=kind):
                    w = qs[i].to(torch.bfloat16) * ss[i].to(torch.bfloat16)[:, None]
                    return F.linear(x, w) if kind == "fwd" else dy.matmul(w)

                def cublas(i, kind=kind):
                    return F.linear(x, dense[i]) if kind == "fwd" else dy.matmul(dense[i])

                ref_out = torch.empty(m, n_out, device=dev, dtype=torch.bfloat16)

                def ref_triton(i, kind=kind, ref_out=ref_out):
                    if kind == "fwd":
                        return ref_qk.triton_int8_linear_forward(x, qs[i], ss[i], None, torch.bfloat16, torch.bfloat16,
                                                                 out=ref_out)
                    return ref_qk.triton_int8_linear_backward(dy, qs[i], ss[i], torch.Size((m, k)), torch.bfloat16,
                                                              torch.bfloat16, out=ref_out)

                nbytes = n * k + 4 * n + 2 * m * k + 2 * m * n
                t_roof = max(flops / (peaks["bf16_tflops"] * 1e12), nbytes / (peaks["hbm_gbs"] * 1e9))
                entry = {}
                impls = [("ours", ours, copies), ("eager_gpu", eager, copies), ("cublas_bf16", cublas, dense_copies)]
                if ref_qk is not None:
                    impls.insert(1, ("ref_triton", ref_triton, copies))
                for label, fn, count in impls:
                    us = graph_time_us([lambda i=i, fn=fn: fn(i) for i in range(count)], dev)
                    entry[label] = {"us": us, "tflops": flops / us / 1e6}
                entry["ours"].update({"gbs": nbytes / entry["ours"]["us"] / 1e3,
                                      "roofline_frac": t_roof / (entry["ours"]["us"] * 1e-6)})
                entry["speedup_vs_eager_gpu"] = entry["eager_gpu"]["us"] / entry["ours"]["us"]
                entry["frac_of_cublas_bf16"] = entry["cublas_bf16"]["us"] / entry["ours"]["us"]
                if ref_qk is not None:
                    entry["speedup_vs_ref_triton"] = entry["ref_triton"]["us"] / entry["ours"]["us"]
                    ours(0)
                    ref_triton(0)
                    mine = (y if kind == "fwd" else dx).float()
                    theirs = ref_out.float()
                    entry["rel_diff_vs_ref_triton"] = float((mine - theirs).norm() / theirs.norm().clamp_min(1e-30))
                res[kind] = entry
                del ws_owner
            res["roofline_peaks"] = f"max(flops / bf16_tflops, bytes / hbm_gbs) ({peak_kind})"
            del x, dy, y, dx
            torch.cuda.empty_cache()
            print(json.dumps(res), flush=True)
        del qs, ss, dense
        torch.cuda.empty_cache()
    qk.check_device_status(dev)


def swap_in_reference_modules(model, device) -> dict:
    """Replace this library's hot-path modules in `model` with the reference's own, from the
    reference package installed under baseline/_ref: every FrozenInt8Linear becomes
    training.quantization.FrozenInt8Linear with the Triton backend (same int8 codes and scales,
    copied), every LoRALinear becomes training.lora.LoRALinear (same adapter values), and the
    stack's activation offload context becomes training.activation_offload.activation_cpu_offload.
    The rest of the harness (norms, attention, elementwise) is unchanged."""
    import torch
    from torch import nn

    ref_qk, missing = reference_triton_kernels()
    if missing:
        raise RuntimeError(f"reference modules unavailable: {missing}")
    from training import activation_offload as ref_ao
    from training.lora import LoRALinear as RefLoRA
    from training.quantization import FrozenInt8Linear as RefInt8

    from moss_image_b200 import dit
    from moss_image_b200.lora import LoRALinear as OurLoRA
    from moss_image_b200.quantization import FrozenInt8Linear as OurInt8

    def ref_int8(mod):
        dtype = mod.compute_dtype
        linear = nn.Linear(mod.in_features, mod.out_features, bias=mod.bias is not None, device=device, dtype=dtype)
        with torch.no_grad():
            linear.weight.zero_()
            if linear.bias is not None:
                linear.bias.copy_(mod.bias)
        linear.requires_grad_(False)
        ref = RefInt8(linear, backend="triton")
        with torch.no_grad():
            ref.weight_int8.copy_(mod.weight_int8)
            ref.weight_scale.copy_(mod.weight_scale)
        return ref

    # collect first (a LoRA wrapper's base is replaced together with the wrapper), then swap
    targets = []
    for parent in model.modules():
        if isinstance(parent, OurLoRA):
            continue
        for child_name, child in parent.named_children():
            if isinstance(child, OurLoRA) and isinstance(child.base, OurInt8):
                targets.append((parent, child_name, child, True))
            elif isinstance(child, OurInt8):
                targets.append((parent, child_name, child, False))
    counts = {"int8": 0, "lora": 0}
    for parent, child_name, child, is_lora in targets:
        if is_lora:
            wrapped = RefLoRA(ref_int8(child.base), child.rank, child.alpha).to(device)
            with torch.no_grad():
                wrapped.lora_A.copy_(child.lora_A)
                wrapped.lora_B.copy_(child.lora_B)
            setattr(parent, child_name, wrapped)
            counts["lora"] += 1
        else:
            setattr(parent, child_name, ref_int8(child))
        counts["int8"] += 1
    dit.activation_cpu_offload = ref_ao.activation_cpu_offload
    return counts


def time_reference_modules(args: argparse.Namespace, steps: int, warmup: int) -> dict:
    """The benchmark's config-3 training step (same model, inputs, optimizer and offload setting as the
    default run) with the reference's own hot-path modules swapped in, timed the same way
    (CUDA events over `steps` after `warmup`, 1 GPU). Returns the measurement."""
    import torch

    sys.path.insert(0, str(REPO))
    from moss_image_b200 import dit
    from moss_image_b200.activation_offload import activation_cpu_offload as ours_offload
    from moss_image_b200.dit import build_lora_model, flow_matching_loss

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    model = build_lora_model(args.depth, device=dev, dim=DIM, heads=HEADS, mlp_dim=MLP, rank=RANK, seed=0,
                             full_qkvo=args.full_qkvo)
    try:
        swapped = swap_in_reference_modules(model, dev)
        model.train()
        model.activation_offload = not args.no_offload
        params = [p for p in model.parameters() if p.requires_grad]
        opt = torch.optim.AdamW(params, lr=1e-4, fused=True)
        img_tokens, txt_tokens = args.img_tokens, args.txt_tokens
        gen = torch.Generator(device=dev).manual_seed(1234)
        latents = torch.randn(args.batch, img_tokens, DIM, device=dev, generator=gen).to(torch.bfloat16)
        text = torch.randn(args.batch, txt_tokens, DIM, device=dev, generator=gen).to(torch.bfloat16)
        noise = torch.randn(args.batch, img_tokens, DIM, device=dev, generator=gen).to(torch.bfloat16)
        t = torch.rand(args.batch, device=dev, generator=gen)

        def step() -> torch.Tensor:
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = flow_matching_loss(model, latents, text, t, noise)
            loss.backward()
            opt.step()
            opt.zero_grad(set_to_none=True)
            return loss.detach()

        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        props = torch.cuda.get_device_properties(dev)
        clocks = ClockSampler(f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0")
        clocks.start()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            loss = step()
        end.record()
        torch.cuda.synchronize()
        clock_info = clocks.stop()
    finally:
        dit.activation_cpu_offload = ours_offload
    ms = start.elapsed_time(end) / steps
    tokens = args.batch * (img_tokens + txt_tokens)
    return {
        "value": tokens / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps, "warmup": warmup,
        "loss": float(loss.item()), "swapped": swapped, "offload": not args.no_offload, "clocks": clock_info,
        "note": "training.quantization.FrozenInt8Linear (backend triton), training.lora.LoRALinear and "
                "training.activation_offload from baseline/_ref in place of this library's modules; "
                "the rest of the synthetic model, the inputs and AdamW are the default run's",
    }


def run_train_ref_modules(args: argparse.Namespace) -> None:
    """One JSON line: `time_reference_modules` at `--steps` after `--warmup`."""
    result = time_reference_modules(args, args.steps, args.warmup)
    print(json.dumps({"impl": "reference_gpu_modules",
                      "metric": "INT8-W DiT train tokens/s (reference modules on the same GPU)", **result}),
          flush=True)


def run_packed(args: argparse.Namespace) -> None:
    """One training step over a heterogeneous batch: packed into one traversal (every GEMM sees
    all tokens, variable-length attention) versus one traversal per sample (what a batch of
    unequal samples costs without packing). Same model, samples, optimizer and offload."""
    import torch

    sys.path.insert(0, str(REPO))
    from moss_image_b200 import quant_kernels as qk
    from moss_image_b200.dit import build_lora_model, flow_matching_loss, packed_flow_matching_loss

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec = [tuple(int(v) for v in item.split(":")) for item in args.packed.split(",")]
    model = build_lora_model(args.depth, device=dev, dim=DIM, heads=HEADS, mlp_dim=MLP, rank=RANK, seed=0)
    model.train()
    model.activation_offload = not args.no_offload
    model.activation_offload_defer_bytes = args.offload_defer_mb << 20
    opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=1e-4, fused=True)
    gen = torch.Generator(device=dev).manual_seed(99)
    latents = [torch.randn(i, DIM, device=dev, generator=gen).to(torch.bfloat16) for i, _ in spec]
    text = [torch.randn(t, DIM, device=dev, generator=gen).to(torch.bfloat16) for _, t in spec]
    noise = [torch.randn(i, DIM, device=dev, generator=gen).to(torch.bfloat16) for i, _ in spec]
    times = torch.rand(len(spec), device=dev, generator=gen)
    total = sum(i + t for i, t in spec)

    def packed_step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = packed_flow_matching_loss(model, latents, text, times, noise)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    def serial_step():
        for k in range(len(spec)):
            with torch.autocast("cuda", dtype=torch.bfloat16):
                loss = flow_matching_loss(model, latents[k][None], text[k][None], times[k:k + 1], noise[k][None])
            (loss / len(spec)).backward()
        opt.step()
        opt.zero_grad(set_to_none=True)

    result = {}
    for label, fn in (("packed", packed_step), ("serial", serial_step)):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(args.steps):
            fn()
        b.record()
        b.synchronize()
        ms = a.elapsed_time(b) / args.steps
        result[label] = {"ms_per_step": ms, "tokens_per_s": total / (ms * 1e-3)}
    qk.check_device_status(dev)
    print(json.dumps({"metric": "packed heterogeneous-batch train tokens/s", "value": result["packed"]["tokens_per_s"],
                      "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
                      "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": f"{args.depth}-block synthetic DiT int8-W LoRA step, samples (img:txt) "
                                             f"{args.packed}, activation offload {'off' if args.no_offload else 'on'}",
                                 "tokens_per_step": total},
                      **result, "speedup_vs_serial": result["serial"]["ms_per_step"] / result["packed"]["ms_per_step"]}),
          flush=True)


# ----------------------------------------------------------------------------- training step
def run_train(args: argparse.Namespace) -> None:
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(REPO))
    from moss_image_b200 import activation_offload as ao
    from moss_image_b200 import quant_kernels as qk
    from moss_image_b200.dit import build_lora_model, flow_matching_loss
    from moss_image_b200.dp import GradAllReducer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    # each rank's pinned offload ring on the NUMA node of its GPU (host-DRAM traffic of N offload streams)
    numa_cpus = ao.bind_to_device_numa_node(dev) if not args.no_numa_bind else None
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))

    model = build_lora_model(args.depth, device=dev, dim=DIM, heads=HEADS, mlp_dim=MLP, rank=RANK, seed=0,
                             full_qkvo=args.full_qkvo)
    model.train()
    streamer = None
    if args.blocks_to_swap:
        from moss_image_b200.memory import place_model

        place_model(model, dev, args.blocks_to_swap, block_swap_mode="async")
        streamer = model.block_swap_manager
        torch.cuda.empty_cache()
    model.activation_offload = not args.no_offload
    model.activation_offload_defer_bytes = args.offload_defer_mb << 20
    params = [p for p in model.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)
    reducer = GradAllReducer(params, timing=True)

    img_tokens, txt_tokens = args.img_tokens, args.txt_tokens
    seq = img_tokens + txt_tokens
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    latents = torch.randn(args.batch, img_tokens, DIM, device=dev, generator=gen).to(torch.bfloat16)
    text = torch.randn(args.batch, txt_tokens, DIM, device=dev, generator=gen).to(torch.bfloat16)
    noise = torch.randn(args.batch, img_tokens, DIM, device=dev, generator=gen).to(torch.bfloat16)
    t = torch.rand(args.batch, device=dev, generator=gen)
    host = [x.cpu().pin_memory() for x in (latents, text, noise, t)]
    h2d_bytes = sum(x.numel() * x.element_size() for x in host)

    def step(inputs) -> torch.Tensor:
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = flow_matching_loss(model, *inputs)
        loss.backward()
        reducer.finish()
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss.detach()

    inputs = (latents, text, t, noise)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step(inputs)
    qk.check_device_status(dev)
    ring = ao.offload_ring(dev)
    stats0 = ring.stats()
    swap0 = streamer.copy_statistics() if streamer is not None else None

    timer = GemmTimer()
    qk.set_launch_observer(timer)
    props = torch.cuda.get_device_properties(dev)
    clocks = ClockSampler(f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0")
    from moss_image_b200 import _lib as moss_lib

    counts0 = dict(moss_lib.launch_counts)
    barrier()
    clocks.start()
    timer.active = True
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step(inputs)
    end.record()
    barrier()
    timer.active = False
    clock_info = clocks.stop()
    elapsed_ms = start.elapsed_time(end)
    stats1 = ring.stats()
    other_launches = {name: count - counts0.get(name, 0) for name, count in moss_lib.launch_counts.items()}
    swap1 = streamer.copy_statistics() if streamer is not None else None
    gemm = timer.summary()

    # e2e: inputs copied from pinned host buffers each step, loss read back each step
    dev_bufs = [torch.empty_like(x, device=dev) for x in host]
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    losses = []
    for _ in range(args.steps):
        for d, h in zip(dev_bufs, host):
            d.copy_(h, non_blocking=True)
        loss = step((dev_bufs[0], dev_bufs[1], dev_bufs[3], dev_bufs[2]))
        losses.append(float(loss.item()))
    e_end.record()
    barrier()
    e2e_ms = e_start.elapsed_time(e_end)
    qk.check_device_status(dev)

    # Offload on against off in the same process: alternating arms of `arm_steps` steps, each
    # after one untimed step, so slow drift (clocks, host) hits both arms alike. The copy
    # engines are timed (an event pair per copy) only during the offload-on arms.
    offload_ab = None
    if not args.no_offload and args.offload_pairs > 0:
        arm_steps = max(1, args.offload_arm_steps)
        arms = {True: [], False: []}
        d2h_ms = h2d_ms = 0.0
        d2h_b = h2d_b = moved = 0
        for _ in range(args.offload_pairs):
            for enabled in (False, True):
                model.activation_offload = enabled
                ring.set_timing(enabled)
                step(inputs)
                barrier()
                if enabled:  # the untimed step's copies are left out of the copy-engine figures
                    c0, b0 = ring.copy_time(), ring.stats()
                a_ev, b_ev = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a_ev.record()
                for _ in range(arm_steps):
                    step(inputs)
                b_ev.record()
                barrier()
                arms[enabled].append(a_ev.elapsed_time(b_ev) / arm_steps)
                if enabled:
                    c1, b1 = ring.copy_time(), ring.stats()
                    d2h_ms += c1["d2h_ms"] - c0["d2h_ms"]
                    h2d_ms += c1["h2d_ms"] - c0["h2d_ms"]
                    d2h_b += c1["d2h_bytes"] - c0["d2h_bytes"]
                    h2d_b += c1["h2d_bytes"] - c0["h2d_bytes"]
                    moved += (b1["d2h_bytes"] - b0["d2h_bytes"]) + (b1["h2d_bytes"] - b0["h2d_bytes"])
        ring.set_timing(False)
        model.activation_offload = True
        on_ms, off_ms = statistics.mean(arms[True]), statistics.mean(arms[False])
        link = host_link_gbs(dev)
        offload_ab = {
            "ms_per_step_on": on_ms, "ms_per_step_off": off_ms, "overhead": on_ms / off_ms - 1.0,
            "arms": {"on": arms[True], "off": arms[False]}, "steps_per_arm": arm_steps,
            "d2h_copy_engine_gbs": d2h_b / (d2h_ms * 1e-3) / 1e9 if d2h_ms > 0 else None,
            "h2d_copy_engine_gbs": h2d_b / (h2d_ms * 1e-3) / 1e9 if h2d_ms > 0 else None,
            "host_link_gbs": link,
            "d2h_busy_frac_of_step": d2h_ms / (on_ms * arm_steps * args.offload_pairs),
            "h2d_busy_frac_of_step": h2d_ms / (on_ms * arm_steps * args.offload_pairs),
            "bytes_per_step": moved / (arm_steps * args.offload_pairs),
            "note": ("offload on vs off alternated in this run (one untimed step before each arm); copy-engine GB/s = "
                     "bytes / summed CUDA-event time of the ring's copies; host_link_gbs = best plain 256 MiB "
                     "pinned->device copy on the idle GPU"),
        }
    exchange = None
    if world > 1:
        waits = []
        for _ in range(2):
            step(inputs)
            waits.append(reducer.last_wait_ms())
        exchange = {"buckets": len(reducer.buckets), "bucket_bytes": reducer.bucket_bytes,
                    "grad_bytes_per_step": sum(reducer.bucket_bytes),
                    "buckets_sent_during_backward": reducer.last_sent_from_hooks,
                    "finish_wait_ms": waits,
                    "note": "finish_wait_ms: device time the compute stream waited in the all-reduce after backward"}

    times = torch.tensor([elapsed_ms, e2e_ms], device=dev)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    elapsed_ms, e2e_ms = float(times[0]), float(times[1])
    tokens = world * args.batch * seq * args.steps
    value = tokens / (elapsed_ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)

    if rank == 0:
        peaks, peak_kind = measured_peaks()
        dominant = max(gemm, key=lambda kind: gemm[kind]["total_ms"]) if gemm else None
        roofline = None
        if dominant is not None:
            d = gemm[dominant]
            per_launch_flops = d["flops"] / d["launches"]
            achieved = per_launch_flops / (d["avg_us"] * 1e-6) / 1e12
            peak = peaks["bf16_tflops_sustained"]
            traffic = load_traffic(dominant)
            roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak, "traffic": traffic,
                        "kernel": f"w8a16_gemm_{dominant}", "peak_source": f"bf16_tflops_sustained ({peak_kind})",
                        "launches_timed": d["launches"], "avg_launch_us": d["avg_us"],
                        "algorithmic_flops_per_launch": per_launch_flops,
                        "algorithmic_bytes_per_launch": d["bytes"] / d["launches"]}
        offload_bytes = (stats1["d2h_bytes"] - stats0["d2h_bytes"]) + (stats1["h2d_bytes"] - stats0["h2d_bytes"])
        gemm_tflops = {k: v["flops"] / (v["total_ms"] * 1e-3) / 1e12 for k, v in gemm.items()}
        launches = sum(v["launches"] for v in gemm.values())
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": (f"{args.depth}-block synthetic DiT int8-W {'full-q/k/v/o' if args.full_qkvo else 'LoRA'} "
                                    f"training step per GPU (batch "
                                    f"{args.batch} x ({img_tokens} img + {txt_tokens} txt) tokens, width {DIM}, MLP {MLP} "
                                    f"GELU, per-block adaLN {DIM}->{6 * DIM}, "
                                    + ("q/k/v/o trained in full (bf16 masters), " if args.full_qkvo
                                       else f"LoRA r{RANK} q/k/v/o, ") + "grad checkpointing, "
                                    f"activation offload {'on' if model.activation_offload else 'off'}"
                                    + (f", int8 blocks streamed from pinned host: last {args.blocks_to_swap}"
                                       if args.blocks_to_swap else "") + ")"),
                       "global_batch": world * args.batch, "seq_len": seq, "parallelism": f"dp{world}",
                       "l2": "no flush: per-step working set (GBs of weights/activations) exceeds the 126 MB L2"},
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d_bytes,
                    "d2h_bytes_per_step": 4},
            "roofline": roofline,
            "gemm_tflops": gemm_tflops,
            "offload": {"bytes_per_step": offload_bytes / args.steps, "defer_bytes": args.offload_defer_mb << 20,
                        "gbs_over_step": offload_bytes / (elapsed_ms * 1e-3) / 1e9,
                        "pinned_bytes": stats1["pinned_bytes"]},
            "clocks": clock_info,
            "host_binding": {"cpus": len(numa_cpus) if numa_cpus else None,
                             "note": "rank 0's CPU affinity: the cores NVML reports local to its GPU (None: not bound)"},
            "gpu_launches": launches + sum(other_launches.values()),
            "gpu_launches_by_kind": {"int8_gemm": launches, **other_launches},
            "gpu_launches_note": ("libmoss_w8.so kernel launches in the timed region: int8 GEMM calls (fwd + dx; "
                                  "a split-K call's extra reduction launch is not counted), per-sample "
                                  "conditioning, offload gather/scatter"),
            "loss_last": losses[-1] if losses else None,
        }
        if offload_ab is not None:
            line["offload"]["ab"] = offload_ab
        if exchange is not None:
            line["grad_exchange"] = exchange
        if streamer is not None:
            line["config"]["blocks_to_swap"] = args.blocks_to_swap
            line["block_swap"] = block_swap_summary(swap0, swap1, args.steps, elapsed_ms, dev)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_sample()
        if world == 1 and not args.no_ref_gpu_arm:
            # The same step with the reference's own modules on this GPU (after this run's
            # model is freed); a failure is recorded, not raised.
            del model, opt, params, reducer
            torch.cuda.empty_cache()
            try:
                ref = time_reference_modules(args, steps=2, warmup=1)
                line["reference_gpu_modules"] = ref
                line["speedup_vs_reference_gpu_modules"] = line["value"] / ref["value"]
            except Exception as error:
                line["reference_gpu_modules"] = {"unavailable": f"{type(error).__name__}: {error}"[:300]}
        print(json.dumps(line), flush=True)
    qk.set_launch_observer(None)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    elif args.packed:
        run_packed(args)
    elif args.kernel:
        run_kernel(args)
    elif args.sweep:
        run_sweep(args)
    elif args.ref_gpu_modules:
        run_train_ref_modules(args)
    else:
        run_train(args)


if __name__ == "__main__":
    main()

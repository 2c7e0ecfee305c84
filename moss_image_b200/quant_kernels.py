"""Backend selection, validation and launchers for the sm_100a weight-only int8 linear.

Mirrors the host interface of ``training/quant_kernels.py`` (backend strings, validation
messages and exception types, autocast dtype rule, ``out=`` buffers) so callers of the
reference switch without edits. The error texts are the reference's own, including the
"Triton quantized backend is unavailable: <reason>." prefix of its explicit-backend check
(training/quant_kernels.py:78), so code and tests that match on them keep working.

Deliberate differences, all of them refusals where the reference would compute on another
device or in another precision (there is no CPU and no eager fallback):

* every accepted backend string (``auto``, ``eager``, ``triton``) executes the sm_100a
  kernels of ``libmoss_w8.so``; where the reference resolves ``auto``/``eager`` to its
  dense-decode path (training/quant_kernels.py:64-79), an input the kernels cannot run
  raises ``RuntimeError`` with the reference's message - CPU tensors included;
* the compute dtype must be float16 or bfloat16 (tcgen05 ``kind::f16``); a float32
  compute dtype (an fp32 module outside autocast) raises ``RuntimeError``. The trainer never
  reaches it on CUDA: LoRA mode casts the model to bfloat16 (training/train.py:579-580);
* non-contiguous inputs and empty matrices, which the reference's Triton launcher refuses
  (training/quant_kernels.py:58-61), are accepted (copied contiguous / shaped results).
"""

from __future__ import annotations

import ctypes
from typing import Literal

import torch

from . import _lib

QuantizedBackend = Literal["auto", "eager", "triton"]

_BACKENDS = {"auto", "eager", "triton"}

# Prefix of every "cannot run this here" error (the reference's text, training/quant_kernels.py:78).
UNAVAILABLE = "Triton quantized backend is unavailable"

_status_buffers: dict[tuple[str, int | None], torch.Tensor] = {}
# host-visible copies of the status bits (moss_status_mirror), by device index
_status_mirrors: dict[int, "ctypes._Pointer"] = {}
_backward_polls: set[int] = set()

# Optional launch observer (benchmarks): called as observer(kind, m, n, k, device) before a
# GEMM launch and returns a callable invoked right after it.
_launch_observer = None


def set_launch_observer(observer) -> None:
    """Install (or clear with ``None``) a callback wrapped around every GEMM launch."""
    global _launch_observer
    _launch_observer = observer


def validate_quantized_backend(backend: str) -> QuantizedBackend:
    """Reference: training/quant_kernels.py:30-33 (same accepted strings and message)."""
    if backend not in _BACKENDS:
        raise ValueError("quantized backend must be auto, eager or triton.")
    return backend  # type: ignore[return-value]


def kernels_are_available() -> bool:
    """Whether the CUDA library loads and a CUDA device is visible."""
    return _lib.is_available() and torch.cuda.is_available()


# Reference name (training/quant_kernels.py:36-38); here it reports the B200 kernels.
triton_is_available = kernels_are_available


def _unsupported_reason(tokens: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor) -> str | None:
    """Reference: training/quant_kernels.py:41-61, adapted to the sm_100a kernels."""
    if not _lib.is_available():
        try:
            _lib.library()
        except RuntimeError as error:
            return f"the sm_100a kernel library is not installed ({error})"
    if tokens.device.type != "cuda":
        return "the input is not on CUDA"
    if weight.device != tokens.device or scale.device != tokens.device:
        return "the quantized weight and scale are not on the input CUDA device"
    if tokens.dtype not in {torch.float16, torch.bfloat16, torch.float32}:
        return f"input dtype {tokens.dtype} is unsupported"
    if weight.dtype != torch.int8 or scale.dtype != torch.float32:
        return "weights must be int8 and scales must be float32"
    if tokens.ndim < 1 or tokens.shape[-1] != weight.shape[1]:
        return "input and weight dimensions do not match"
    if not weight.is_contiguous() or not scale.is_contiguous():
        return "weight and scale must be contiguous"
    return None


def resolve_quantized_backend(
    backend: str,
    tokens: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
) -> QuantizedBackend:
    """Validate the backend string and that the sm_100a kernels can run these tensors.

    Reference: training/quant_kernels.py:64-79, with its message. Unlike the reference,
    ``auto`` and ``eager`` do not fall back to a CPU or dequantise-then-cuBLAS path: an
    input the kernels cannot run raises ``RuntimeError`` for every backend string.
    """
    selected = validate_quantized_backend(backend)
    reason = _unsupported_reason(tokens, weight, scale)
    if reason is not None:
        raise RuntimeError(f"{UNAVAILABLE}: {reason}.")
    return selected


def autocast_compute_dtype(tokens: torch.Tensor, module_dtype: torch.dtype) -> torch.dtype:
    """Match CUDA autocast's output dtype for a linear operation.

    Reference: training/quant_kernels.py:82-95.
    """
    if tokens.device.type != "cuda":
        return module_dtype
    if not torch.is_autocast_enabled("cuda"):
        return module_dtype
    return torch.get_autocast_dtype("cuda")


def _device_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def status_buffer(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR their MOSS_STATUS_* bits into.

    Creating it also sets up the device's host-visible copy of those bits
    (``moss_status_mirror``), which ``poll_device_status`` reads without a device sync.
    """
    key = ("cuda", _device_index(device))
    buf = _status_buffers.get(key)
    if buf is None:
        dev = torch.device("cuda", key[1])
        buf = torch.zeros(1, dtype=torch.int32, device=dev)
        word = ctypes.POINTER(ctypes.c_int)()
        with torch.cuda.device(dev):
            _lib.check(_lib.library().moss_status_mirror(ctypes.byref(word)), "moss_status_mirror")
        _status_mirrors[key[1]] = word
        _status_buffers[key] = buf
    return buf


def poll_device_status(device: torch.device) -> int:
    """Raise if a kernel on ``device`` has reported a pipeline timeout; never synchronises.

    Reads the host-visible copy of the status bits, which a failed launch writes when it
    completes. The failure is sticky: every later GEMM call on the device raises until
    ``check_device_status`` (or ``reset_device_status``) clears it.
    """
    word = _status_mirrors.get(_device_index(device))
    value = 0 if word is None else int(word[0])
    if value & _lib.STATUS_TIMEOUT_MASK:
        raise RuntimeError(f"sm_100a int8 kernel reported a pipeline timeout (status 0x{value:x}); its output "
                           "is invalid. Clear with quant_kernels.reset_device_status() after handling it.")
    return value


def reset_device_status(device: torch.device) -> None:
    """Clear the device status word and its host-visible copy."""
    buf = status_buffer(device)
    buf.zero_()
    torch.cuda.synchronize(buf.device)
    word = _status_mirrors.get(_device_index(device))
    if word is not None:
        word[0] = 0


def check_device_status(device: torch.device | None = None, *, reset: bool = True) -> int:
    """Synchronise on the status word and raise if a kernel reported a failure."""
    devices = [device] if device is not None else [torch.device("cuda", k[1]) for k in _status_buffers]
    worst = 0
    for dev in devices:
        buf = status_buffer(dev)
        value = int(buf.item())
        word = _status_mirrors.get(_device_index(dev))
        if word is not None:
            value |= int(word[0])
        if reset and value:
            reset_device_status(dev)
        worst |= value
    if worst & _lib.STATUS_TIMEOUT_MASK:
        raise RuntimeError(f"sm_100a int8 kernel reported a pipeline timeout (status 0x{worst:x}).")
    return worst


def _poll_after_backward(device: torch.device) -> None:
    """Queue a status poll for the end of the running backward pass (once per pass)."""
    index = _device_index(device)
    if index in _backward_polls:
        return
    _backward_polls.add(index)

    def _poll() -> None:
        _backward_polls.discard(index)
        poll_device_status(torch.device("cuda", index))

    try:
        torch.autograd.Variable._execution_engine.queue_callback(_poll)
    except RuntimeError:  # not inside a backward pass (direct launcher call)
        _backward_polls.discard(index)


def _compute_kind(dtype: torch.dtype) -> int:
    if dtype not in (torch.float16, torch.bfloat16):
        raise RuntimeError(
            f"{UNAVAILABLE}: compute dtype {dtype} is unsupported "
            "(the sm_100a kernels compute in float16 or bfloat16; use autocast or a half-precision module)."
        )
    return _lib.DTYPE_CODES[dtype]


def _workspace(m: int, n_out: int, k_red: int, device: torch.device) -> tuple[torch.Tensor | None, int | None, int]:
    """Scratch for split launches from torch's caching allocator: small-M split-K, and the
    CTA-pair kernel's split of a partly empty last round of tiles.

    Returns (owner tensor, 256-byte aligned address, bytes); the caller keeps the owner alive
    until the launch is enqueued (later reuse is ordered by the stream).
    """
    size = ctypes.c_size_t()
    _lib.check(_lib.library().moss_w8a16_gemm_workspace_bytes(m, n_out, k_red, ctypes.byref(size)),
               "moss_w8a16_gemm_workspace_bytes")
    if size.value == 0:
        return None, None, 0
    buf = torch.empty(size.value + 256, dtype=torch.uint8, device=device)
    return buf, (buf.data_ptr() + 255) // 256 * 256, size.value


def _matrix_view(tokens: torch.Tensor) -> torch.Tensor:
    rows = 1
    for size in tokens.shape[:-1]:
        rows *= size
    return tokens.reshape(rows, tokens.shape[-1])


def int8_linear_forward(
    tokens: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None,
    output_dtype: torch.dtype,
    weight_dtype: torch.dtype,
    *,
    out: torch.Tensor | None = None,
    lora_xa: torch.Tensor | None = None,
    lora_b: torch.Tensor | None = None,
    lora_scale: float = 1.0,
) -> torch.Tensor:
    """Y = X dec(W)^T (+ bias) (+ lora_scale * lora_xa lora_b^T) on the sm_100a kernel.

    Reference: ``triton_int8_linear_forward``, training/quant_kernels.py:294-334 (same
    arguments and ``out=`` contract). ``tokens`` is cast to ``output_dtype`` (as the
    reference's kernel casts its tile loads) and made contiguous if needed.
    """
    v_kind = _compute_kind(output_dtype)
    if tokens.is_cuda:
        status_buffer(tokens.device)
        poll_device_status(tokens.device)
    matrix = _matrix_view(tokens)
    if matrix.dtype != output_dtype:
        matrix = matrix.to(output_dtype)
    if not matrix.is_contiguous():
        matrix = matrix.contiguous()
    rows, in_features = matrix.shape
    out_features = weight.shape[0]
    if out is None:
        output = torch.empty((rows, out_features), device=tokens.device, dtype=output_dtype)
    else:
        output = out.reshape(rows, out_features)
        if output.dtype != output_dtype or not output.is_contiguous():
            raise ValueError("Triton output buffer has the wrong dtype or is not contiguous.")
    if bias is not None and (bias.device != tokens.device or not bias.is_contiguous()):
        raise RuntimeError("Triton quantized bias must be contiguous and on the input device.")
    rank = 0
    if lora_xa is not None:
        if lora_b is None:
            raise ValueError("lora_xa needs lora_b")
        lora_xa = lora_xa.reshape(rows, -1)
        if lora_xa.dtype != output_dtype or not lora_xa.is_contiguous():
            lora_xa = lora_xa.to(output_dtype).contiguous()
        rank = lora_xa.shape[1]
        if lora_b.shape != (out_features, rank):
            raise ValueError(f"lora_b must be [{out_features}, {rank}], got {tuple(lora_b.shape)}")
        lora_b = lora_b.contiguous()
    lib = _lib.library()
    status = status_buffer(tokens.device)  # before the workspace: never carved out of it
    ws_owner, ws, ws_bytes = _workspace(rows, out_features, in_features, tokens.device)
    done = _launch_observer("fwd", rows, out_features, in_features, tokens.device) if _launch_observer else None
    rc = lib.moss_w8a16_gemm_fwd(
        _lib.ptr(matrix), v_kind, rows, in_features,
        _lib.ptr(weight), _lib.ptr(scale), _lib.dtype_code(weight_dtype), out_features,
        _lib.ptr(bias), _lib.DTYPE_CODES.get(bias.dtype, -1) if bias is not None else 0,
        _lib.ptr(lora_xa), _lib.ptr(lora_b), _lib.DTYPE_CODES.get(lora_b.dtype, -1) if lora_b is not None else 0,
        rank, float(lora_scale),
        _lib.ptr(output), _lib.DTYPE_CODES[output_dtype], ws, ws_bytes,
        _lib.ptr(status), _lib.stream_handle(tokens.device),
    )
    if done is not None:
        done()
    del ws_owner
    _lib.check(rc, "moss_w8a16_gemm_fwd")
    return output.reshape(*tokens.shape[:-1], out_features)


def int8_linear_backward(
    gradient: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    input_shape: torch.Size,
    input_dtype: torch.dtype,
    weight_dtype: torch.dtype,
    *,
    out: torch.Tensor | None = None,
    compute_dtype: torch.dtype | None = None,
    lora_dyb: torch.Tensor | None = None,
    lora_a: torch.Tensor | None = None,
    lora_scale: float = 1.0,
    rotate_group: int = 1,
) -> torch.Tensor:
    """dX = dY dec(W) (+ lora_scale * lora_dyb lora_a) on the sm_100a kernel.

    Reference: ``triton_int8_linear_backward``, training/quant_kernels.py:337-373. The
    product is rounded to the gradient's compute dtype and stored as ``input_dtype``.
    The int8 weight is consumed in its ``[N, K]`` storage order (no transpose copy).
    With ``rotate_group`` > 1 (ConvRot, no LoRA term) each row of dX is then rotated by the
    grouped Hadamard transform (``moss_w8a16_gemm_dx_rotated``: in the GEMM's epilogue when the
    CTA-pair kernel runs, else by the rotation kernel right after it).
    """
    compute_dtype = gradient.dtype if compute_dtype is None else compute_dtype
    v_kind = _compute_kind(compute_dtype)
    if gradient.is_cuda:
        status_buffer(gradient.device)
        poll_device_status(gradient.device)
        _poll_after_backward(gradient.device)
    matrix = _matrix_view(gradient)
    if matrix.dtype != compute_dtype:
        matrix = matrix.to(compute_dtype)
    if not matrix.is_contiguous():
        matrix = matrix.contiguous()
    rows, out_features = matrix.shape
    in_features = weight.shape[1]
    if out is None:
        grad_input = torch.empty((rows, in_features), device=gradient.device, dtype=input_dtype)
    else:
        grad_input = out.reshape(rows, in_features)
        if grad_input.dtype != input_dtype or not grad_input.is_contiguous():
            raise ValueError("Triton input-gradient buffer has the wrong dtype or is not contiguous.")
    rank = 0
    if lora_dyb is not None:
        if lora_a is None:
            raise ValueError("lora_dyb needs lora_a")
        lora_dyb = lora_dyb.reshape(rows, -1)
        if lora_dyb.dtype != compute_dtype or not lora_dyb.is_contiguous():
            lora_dyb = lora_dyb.to(compute_dtype).contiguous()
        rank = lora_dyb.shape[1]
        if lora_a.shape != (rank, in_features):
            raise ValueError(f"lora_a must be [{rank}, {in_features}], got {tuple(lora_a.shape)}")
        lora_a = lora_a.contiguous()
    lib = _lib.library()
    status = status_buffer(gradient.device)
    ws_owner, ws, ws_bytes = _workspace(rows, in_features, out_features, gradient.device)
    done = _launch_observer("dx", rows, in_features, out_features, gradient.device) if _launch_observer else None
    if rotate_group > 1:
        if lora_dyb is not None:
            raise ValueError("a rotated grad-input takes no LoRA term")
        rc = lib.moss_w8a16_gemm_dx_rotated(
            _lib.ptr(matrix), v_kind, rows, out_features,
            _lib.ptr(weight), _lib.ptr(scale), _lib.dtype_code(weight_dtype), in_features, int(rotate_group),
            _lib.ptr(grad_input), _lib.dtype_code(input_dtype), ws, ws_bytes,
            _lib.ptr(status), _lib.stream_handle(gradient.device),
        )
        what = "moss_w8a16_gemm_dx_rotated"
    else:
        rc = lib.moss_w8a16_gemm_dx(
            _lib.ptr(matrix), v_kind, rows, out_features,
            _lib.ptr(weight), _lib.ptr(scale), _lib.dtype_code(weight_dtype), in_features,
            _lib.ptr(lora_dyb), _lib.ptr(lora_a), _lib.DTYPE_CODES.get(lora_a.dtype, -1) if lora_a is not None else 0,
            rank, float(lora_scale),
            _lib.ptr(grad_input), _lib.dtype_code(input_dtype), ws, ws_bytes,
            _lib.ptr(status), _lib.stream_handle(gradient.device),
        )
        what = "moss_w8a16_gemm_dx"
    if done is not None:
        done()
    del ws_owner
    _lib.check(rc, what)
    return grad_input.reshape(input_shape)


# Reference launcher names (training/quant_kernels.py:294, :337): same contract, B200 kernel.
triton_int8_linear_forward = int8_linear_forward
triton_int8_linear_backward = int8_linear_backward


def quantize_weight(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel symmetric int8 codes and f32 scales, bit-exact with the reference.

    Reference: ``FrozenInt8Linear.__init__``, training/quantization.py:87-91. Runs on the
    weight's CUDA device; a CPU weight is staged through the current CUDA device and the
    results are returned on the weight's device. Raises ``ValueError`` for non-finite input.
    """
    if weight.ndim != 2:
        raise ValueError("weight must be 2-D [out_features, in_features]")
    if not torch.cuda.is_available():
        raise RuntimeError("int8 quantization needs a CUDA device (the sm_100a quantiser has no CPU fallback).")
    source_device = weight.device
    work = weight.detach()
    if work.device.type != "cuda":
        work = work.to(torch.device("cuda", torch.cuda.current_device()))
    if work.dtype not in _lib.DTYPE_CODES:
        work = work.float()
    work = work.contiguous()
    n, k = work.shape
    codes = torch.empty((n, k), dtype=torch.int8, device=work.device)
    scale = torch.empty((n,), dtype=torch.float32, device=work.device)
    status = torch.zeros(1, dtype=torch.int32, device=work.device)
    rc = _lib.library().moss_w8_quantize(
        _lib.ptr(work), _lib.DTYPE_CODES[work.dtype], n, k, _lib.ptr(codes), _lib.ptr(scale),
        _lib.ptr(status), _lib.stream_handle(work.device),
    )
    _lib.check(rc, "moss_w8_quantize")
    if int(status.item()) & _lib.STATUS_NONFINITE_WEIGHT:
        raise ValueError("Cannot quantize non-finite linear weights.")
    if source_device != work.device:
        codes = codes.to(source_device)
        scale = scale.to(source_device)
    return codes, scale


def dequantize_weight(weight: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Transient decoded weight ``round_d(q * round_d(s))`` (reference quantization.py:23-24)."""
    if weight.device.type != "cuda":
        raise RuntimeError(f"{UNAVAILABLE}: the weight is not on CUDA.")
    out = torch.empty(weight.shape, dtype=dtype, device=weight.device)
    rc = _lib.library().moss_w8_dequantize(
        _lib.ptr(weight), _lib.ptr(scale), weight.shape[0], weight.shape[1], _lib.dtype_code(dtype),
        _lib.ptr(out), _lib.stream_handle(weight.device),
    )
    _lib.check(rc, "moss_w8_dequantize")
    return out


# ------------------------------------------------------------------ ConvRot (grouped Hadamard)
# Rows rotated per call of the ConvRot launchers: bounds the temporary rotated activations at
# 32 Mi elements whatever the token count (one chunk for any step of the benchmark).
_CONVROT_WORKSPACE_ELEMENTS = 32 << 20


def hadamard_transform(
    tokens: torch.Tensor,
    group_size: int,
    *,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
) -> torch.Tensor:
    """Grouped normalised Hadamard rotation of a contiguous CUDA matrix in one pass.

    Reference: ``triton_hadamard_transform``, training/quant_kernels.py:387-426 (same
    arguments and errors; ``workspace`` is accepted for compatibility and unused: all
    stages run on chip). ``out`` may be ``tokens`` itself (in place).
    """
    if tokens.ndim != 2 or not tokens.is_contiguous():
        raise ValueError("Triton Hadamard input must be a contiguous matrix.")
    if tokens.shape[1] % group_size:
        raise ValueError("Input width must be divisible by Hadamard group size.")
    if out is None:
        out = torch.empty_like(tokens)
    if out.shape != tokens.shape or out.dtype != tokens.dtype or not out.is_contiguous():
        raise ValueError("Triton Hadamard output must match its contiguous input.")
    if tokens.device.type != "cuda":
        raise RuntimeError(f"{UNAVAILABLE}: the input is not on CUDA.")
    rc = _lib.library().moss_hadamard_rotate(
        _lib.ptr(tokens), _lib.dtype_code(tokens.dtype), tokens.shape[0], tokens.shape[1], int(group_size),
        _lib.ptr(out), _lib.stream_handle(tokens.device),
    )
    _lib.check(rc, "moss_hadamard_rotate")
    return out


def _convrot_chunk_rows(in_features: int, rows: int) -> int:
    return min(rows, max(1, _CONVROT_WORKSPACE_ELEMENTS // in_features))


def convrot_forward(
    tokens: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    bias: torch.Tensor | None,
    output_dtype: torch.dtype,
    weight_dtype: torch.dtype,
    group_size: int,
) -> torch.Tensor:
    """ConvRot forward ``(x H) dec(W H)^T + b``: rotate the activations, then the int8 GEMM.

    Reference: ``triton_convrot_forward``, training/quant_kernels.py:433-466. The rotation
    is one on-chip pass per chunk of rows (the reference runs one kernel per radix stage).
    """
    matrix = _matrix_view(tokens)
    if not matrix.is_contiguous():
        matrix = matrix.contiguous()
    rows, in_features = matrix.shape
    out_features = weight.shape[0]
    output = torch.empty((rows, out_features), device=tokens.device, dtype=output_dtype)
    if rows == 0:
        return output.reshape(*tokens.shape[:-1], out_features)
    chunk_rows = _convrot_chunk_rows(in_features, rows)
    rotated = torch.empty((chunk_rows, in_features), device=tokens.device, dtype=matrix.dtype)
    for start in range(0, rows, chunk_rows):
        count = min(chunk_rows, rows - start)
        rotated_chunk = rotated[:count]
        hadamard_transform(matrix[start : start + count], group_size, out=rotated_chunk)
        gemm_input = rotated_chunk if rotated_chunk.dtype == weight_dtype else rotated_chunk.to(weight_dtype)
        int8_linear_forward(gemm_input, weight, scale, bias, output_dtype, weight_dtype,
                            out=output[start : start + count])
    return output.reshape(*tokens.shape[:-1], out_features)


def convrot_backward(
    gradient: torch.Tensor,
    weight: torch.Tensor,
    scale: torch.Tensor,
    input_shape: torch.Size,
    input_dtype: torch.dtype,
    weight_dtype: torch.dtype,
    group_size: int,
) -> torch.Tensor:
    """ConvRot input gradient ``H (dY dec(W H))`` (H is symmetric and orthonormal): one call of
    ``moss_w8a16_gemm_dx_rotated``, which rotates the GEMM's output rows in the CTA-pair
    epilogue (group 256) or runs the rotation kernel on them right after the GEMM.

    Reference: ``triton_convrot_backward``, training/quant_kernels.py:469-504 (same roundings:
    the GEMM output in the input dtype, then every radix stage).
    """
    matrix = _matrix_view(gradient.contiguous())
    rows = matrix.shape[0]
    in_features = weight.shape[1]
    grad_input = int8_linear_backward(matrix, weight, scale, torch.Size((rows, in_features)), input_dtype,
                                      weight_dtype, rotate_group=group_size)
    return grad_input.reshape(input_shape)


def convrot_workspace_bound_bytes(in_features: int, dtype: torch.dtype) -> int:
    """Upper bound for the temporary rotated activations of one ConvRot forward call.

    Reference: training/quant_kernels.py:507-513 (the reference bounds two stage buffers;
    here only the rotated chunk exists, for a larger chunk).
    """
    if in_features < 1:
        raise ValueError("input width must be positive")
    element_size = torch.empty((), dtype=dtype).element_size()
    rows = max(1, _CONVROT_WORKSPACE_ELEMENTS // in_features)
    return rows * in_features * element_size


triton_hadamard_transform = hadamard_transform
triton_convrot_forward = convrot_forward
triton_convrot_backward = convrot_backward

"""ctypes binding of the C ABI in ``include/moss_w8.h`` (``libmoss_w8.so``).

The product path has no fallback: if the shared library is missing or fails to load,
every entry point raises ``RuntimeError`` with the loader's message. Loading needs no GPU,
so CPU-only processes can still import the package and inspect the exported symbols.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "libmoss_w8.so"

DTYPE_CODES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}

MOSS_OK = 0
MOSS_ERR_INVALID_ARGUMENT = 1
MOSS_ERR_UNSUPPORTED = 2
MOSS_ERR_CUDA = 3
MOSS_ERR_RING_FULL = 4
MOSS_ERR_NOT_FOUND = 5
MOSS_ERR_BUSY = 6

NOALLOC_SCRATCH_BYTES = 4 << 20  # MOSS_W8A16_NOALLOC_SCRATCH_BYTES

STATUS_NONFINITE_WEIGHT = 0x1
STATUS_TIMEOUT_MASK = 0x2 | 0x4 | 0x8 | 0x10 | 0x20

# name -> (restype, argtypes); mirrors include/moss_w8.h exactly.
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int
_f32 = ctypes.c_float
_sz = ctypes.c_size_t
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "moss_version": (_i32, []),
    "moss_last_error": (ctypes.c_char_p, []),
    "moss_status_mirror": (_i32, [ctypes.POINTER(ctypes.POINTER(ctypes.c_int))]),
    "moss_debug_stall_next_gemm": (_i32, []),
    "moss_w8_quantize": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _vp, _vp]),
    "moss_w8_dequantize": (_i32, [_vp, _vp, _i64, _i64, _i32, _vp, _vp]),
    "moss_w8a16_gemm_workspace_bytes": (_i32, [_i64, _i64, _i64, ctypes.POINTER(_sz)]),
    "moss_w8a16_gemm_fwd": (
        _i32,
        [_vp, _i32, _i64, _i64, _vp, _vp, _i32, _i64, _vp, _i32, _vp, _vp, _i32, _i64, _f32, _vp, _i32, _vp, _sz,
         _vp, _vp],
    ),
    "moss_w8a16_gemm_fwd_noalloc": (
        _i32,
        [_vp, _i32, _i64, _i64, _vp, _vp, _i32, _i64, _vp, _i32, _vp, _vp, _i32, _i64, _f32, _vp, _i32, _vp, _vp],
    ),
    "moss_w8a16_gemm_dx": (
        _i32,
        [_vp, _i32, _i64, _i64, _vp, _vp, _i32, _i64, _vp, _vp, _i32, _i64, _f32, _vp, _i32, _vp, _sz, _vp, _vp],
    ),
    "moss_w8a16_gemm_dx_rotated": (
        _i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i32, _i64, _i64, _vp, _i32, _vp, _sz, _vp, _vp]),
    "moss_hadamard_rotate": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _vp]),
    "moss_segment_modulate": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i32, _i64, _vp, _i64, _vp, _vp]),
    "moss_segment_modulate_bwd": (
        _i32, [_vp, _vp, _i32, _i64, _i64, _vp, _i32, _i64, _vp, _i64, _vp, _vp, _vp, _vp]),
    "moss_segment_gate": (_i32, [_vp, _vp, _i32, _i64, _i64, _vp, _i32, _i64, _vp, _i64, _vp, _vp]),
    "moss_segment_gate_bwd": (_i32, [_vp, _vp, _i32, _i64, _i64, _vp, _i32, _i64, _vp, _i64, _vp, _vp, _vp]),
    "moss_rmsnorm_fwd": (_i32, [_vp, _i32, _i64, _i64, _vp, _i32, _f32, _vp, _vp, _vp]),
    "moss_rmsnorm_bwd": (_i32, [_vp, _vp, _i32, _i64, _i64, _vp, _i32, _vp, _vp, _vp]),
    "moss_strided_gather": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp]),
    "moss_strided_scatter": (_i32, [_vp, _i64, _i32, _vp, _vp, _vp, _vp]),
    "moss_offload_ring_create": (_i32, [_i32, _sz, _sz, _vp, _vp, ctypes.POINTER(_vp)]),
    "moss_offload_ring_destroy": (_i32, [_vp]),
    "moss_offload_pack": (_i32, [_vp, _vp, _sz, _vp, ctypes.POINTER(_i64)]),
    "moss_offload_prefetch": (_i32, [_vp, _i64, _vp]),
    "moss_offload_wait": (_i32, [_vp, _i64, _vp]),
    "moss_offload_release": (_i32, [_vp, _i64]),
    "moss_offload_host_ptr": (_i32, [_vp, _i64, ctypes.POINTER(_vp)]),
    "moss_offload_stats": (
        _i32,
        [_vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_i64),
         ctypes.POINTER(ctypes.c_uint64)],
    ),
    "moss_offload_set_timing": (_i32, [_vp, _i32]),
    "moss_offload_copy_time": (
        _i32,
        [_vp, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint64),
         ctypes.POINTER(ctypes.c_uint64)],
    ),
    "moss_block_stager_create": (_i32, [_i32, _i32, _vp, ctypes.POINTER(_vp)]),
    "moss_block_stager_destroy": (_i32, [_vp, _i32]),
    "moss_block_stager_add_block": (_i32, [_vp, _vp, _sz, ctypes.POINTER(_i64)]),
    "moss_block_stager_set_slot": (_i32, [_vp, _i32, _vp, _sz]),
    "moss_block_stager_select": (_i32, [_vp, _i64, ctypes.POINTER(_i64), _i32, ctypes.POINTER(_i32)]),
    "moss_block_stager_stage": (_i32, [_vp, _i64, _i32, ctypes.POINTER(ctypes.c_uint64)]),
    "moss_block_stager_lease": (_i32, [_vp, _i32, _vp, ctypes.POINTER(ctypes.c_uint64)]),
    "moss_block_stager_hold": (_i32, [_vp, _i32]),
    "moss_block_stager_release": (_i32, [_vp, _i32, _i64, ctypes.c_uint64, _vp]),
    "moss_block_stager_slot_info": (
        _i32, [_vp, _i32, ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_i32)]),
    "moss_block_stager_stats": (
        _i32,
        [_vp, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(_i32),
         ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_uint64)],
    ),
}

# Kernel launches issued through this binding by the ops that do not go through the GEMM
# launch observer (segment conditioning, offload gather/scatter); benchmarks read the deltas.
launch_counts: dict[str, int] = {}


def count_launch(name: str) -> None:
    launch_counts[name] = launch_counts.get(name, 0) + 1


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None
_load_error: str | None = None


def library() -> ctypes.CDLL:
    """Load (once) and return the C-ABI library, raising if it is unavailable."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if _load_error is not None:
            raise RuntimeError(_load_error)
        path = Path(os.environ.get("MOSS_W8_LIB", LIB_PATH))
        if not path.exists():
            _load_error = (
                f"moss_image_b200 CUDA library not found at {path}; build it with "
                "`python -m moss_image_b200.build` (there is no CPU fallback)."
            )
            raise RuntimeError(_load_error)
        try:
            lib = ctypes.CDLL(str(path))
        except OSError as error:
            _load_error = f"failed to load {path}: {error}"
            raise RuntimeError(_load_error) from error
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def is_available() -> bool:
    try:
        library()
    except RuntimeError:
        return False
    return True


def last_error() -> str:
    return library().moss_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    """Raise for a non-zero C-ABI return code."""
    if rc == MOSS_OK:
        return
    message = last_error()
    if rc in (MOSS_ERR_INVALID_ARGUMENT, MOSS_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {message}")
    raise RuntimeError(f"{what} failed (code {rc}): {message}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return DTYPE_CODES[dtype]
    except KeyError:
        raise TypeError(f"int8 kernels do not support {dtype}.") from None


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream

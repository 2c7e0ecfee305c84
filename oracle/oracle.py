"""numpy front end of the CPU oracle - TEST INFRASTRUCTURE ONLY.

Two independent restatements of the reference quantiser (numpy and C) plus the decode
rounding, fp64-accumulated reference GEMMs and the offload payload-view rule. Every
function cites the reference line it restates (paths inside the MOSS-Image repository).
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "_build" / "liboracle.so"

F16, BF16, F32 = 0, 1, 2
KIND_OF = {"float16": F16, "bfloat16": BF16, "float32": F32}

_lib: ctypes.CDLL | None = None


def build() -> Path:
    """Compile the C oracle (make)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (ORACLE_DIR / "w8_oracle.c").stat().st_mtime:
            build()
        L = ctypes.CDLL(str(LIB_PATH))
        vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.oracle_quantize.argtypes = [vp, i64, i64, vp, vp]
        L.oracle_quantize.restype = i32
        L.oracle_dequantize.argtypes = [vp, vp, i64, i64, i32, vp]
        L.oracle_gemm_fwd.argtypes = [vp, i64, i64, vp, vp, i64, i32, i32, vp, vp, vp, i64, f32, vp]
        L.oracle_gemm_dx.argtypes = [vp, i64, i64, vp, vp, i64, i32, i32, vp, vp, i64, f32, vp]
        L.oracle_offload_view.argtypes = [i32, vp, vp, vp]
        L.oracle_offload_view.restype = i32
        L.oracle_gather.argtypes = [vp, i64, i32, vp, vp, vp]
        L.oracle_round.argtypes = [f32, i32]
        L.oracle_hadamard.argtypes = [vp, i64, i64, i64, i32, vp]
        L.oracle_round.restype = f32
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------------------- rounding
def round_bf16(x: np.ndarray) -> np.ndarray:
    """f32 -> bf16 -> f32, round to nearest even (torch's bf16 cast)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    out = u.astype(np.uint32).view(np.float32).copy()
    out[nan] = np.nan
    return out


def round_kind(x: np.ndarray, kind: int) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    if kind == BF16:
        return round_bf16(x)
    if kind == F16:
        return x.astype(np.float16).astype(np.float32)
    return x


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return (round_bf16(x).view(np.uint32) >> 16).astype(np.uint16)


def from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


# ----------------------------------------------------------------------------- quantiser
def quantize_np(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """numpy restatement of training/quantization.py:87-90 (f32 math, half-to-even)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    scale = (np.abs(w).max(axis=1) if w.shape[1] else np.zeros(w.shape[0], np.float32)) / np.float32(127)
    scale = scale.astype(np.float32)
    scale = np.where(scale == 0, np.float32(1), scale).astype(np.float32)
    with np.errstate(invalid="ignore"):
        q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def quantize(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, bool]:
    """C restatement of training/quantization.py:82-90; returns (codes, scales, nonfinite)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty((n,), np.float32)
    nonfinite = lib().oracle_quantize(_p(w), n, k, _p(q), _p(s))
    return q, s, bool(nonfinite)


def dequantize(q: np.ndarray, s: np.ndarray, w_kind: int) -> np.ndarray:
    """training/quantization.py:23-24: round_w(q * round_w(s)) as f32 values."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.float32)
    out = np.empty(q.shape, np.float32)
    lib().oracle_dequantize(_p(q), _p(s), q.shape[0], q.shape[1], w_kind, _p(out))
    return out


# ----------------------------------------------------------------------------- GEMMs
def gemm_fwd(x: np.ndarray, q: np.ndarray, s: np.ndarray, *, w_kind: int, v_kind: int,
             bias: np.ndarray | None = None, lora_xa: np.ndarray | None = None,
             lora_b: np.ndarray | None = None, lora_scale: float = 1.0) -> np.ndarray:
    """fp64-accumulated y = round_v(x) dec(q)^T + round_v(bias) (+ LoRA); unrounded.

    Restates training/quant_kernels.py:125-158 (decode :138-149, bias :152-158) and the
    eager training/quantization.py:43. The LoRA term restates training/lora.py:85-86 with the
    adapter factors as given (already in the compute dtype).
    """
    x = round_kind(np.ascontiguousarray(x, np.float32), v_kind)
    m, k = x.shape
    n = q.shape[0]
    q = np.ascontiguousarray(q, np.int8)
    s = np.ascontiguousarray(s, np.float32)
    y = np.empty((m, n), np.float64)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    xa = None if lora_xa is None else np.ascontiguousarray(lora_xa, np.float32)
    lb = None if lora_b is None else np.ascontiguousarray(lora_b, np.float32)
    r = 0 if xa is None else xa.shape[1]
    lib().oracle_gemm_fwd(_p(x), m, k, _p(q), _p(s), n, w_kind, v_kind, _p(b), _p(xa), _p(lb), r,
                          float(lora_scale), _p(y))
    return y


def gemm_dx(dy: np.ndarray, q: np.ndarray, s: np.ndarray, *, w_kind: int, v_kind: int,
            lora_dyb: np.ndarray | None = None, lora_a: np.ndarray | None = None,
            lora_scale: float = 1.0) -> np.ndarray:
    """fp64-accumulated dx = round_v(dy) dec(q) (+ LoRA); unrounded.

    Restates training/quant_kernels.py:193-218 and the eager training/quantization.py:61-64.
    """
    dy = round_kind(np.ascontiguousarray(dy, np.float32), v_kind)
    m, n = dy.shape
    k = q.shape[1]
    dx = np.empty((m, k), np.float64)
    dyb = None if lora_dyb is None else np.ascontiguousarray(lora_dyb, np.float32)
    a = None if lora_a is None else np.ascontiguousarray(lora_a, np.float32)
    r = 0 if dyb is None else dyb.shape[1]
    lib().oracle_gemm_dx(_p(dy), m, n, _p(np.ascontiguousarray(q, np.int8)), _p(np.ascontiguousarray(s, np.float32)),
                         k, w_kind, v_kind, _p(dyb), _p(a), r, float(lora_scale), _p(dx))
    return dx


def rel_fro(actual: np.ndarray, expected: np.ndarray) -> float:
    """Relative Frobenius error ||a - e|| / ||e|| (0 if both are zero)."""
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    denom = np.linalg.norm(e)
    num = np.linalg.norm(a - e)
    if denom == 0:
        return float(num)
    return float(num / denom)


# ----------------------------------------------------------------------------- offload
def offload_view(shape: tuple[int, ...], stride: tuple[int, ...]) -> tuple[int, ...] | None:
    """training/activation_offload.py:32-61: payload shape, or None if it stays resident."""
    nd = len(shape)
    sh = (ctypes.c_int64 * max(1, nd))(*shape)
    st = (ctypes.c_int64 * max(1, nd))(*stride)
    out = (ctypes.c_int64 * max(1, nd))()
    rc = lib().oracle_offload_view(nd, ctypes.cast(sh, ctypes.c_void_p), ctypes.cast(st, ctypes.c_void_p),
                                   ctypes.cast(out, ctypes.c_void_p))
    return None if rc else tuple(out[i] for i in range(nd))


def gather(storage: np.ndarray, esize: int, shape: tuple[int, ...], stride: tuple[int, ...],
           offset: int = 0) -> bytes:
    """Dense row-major payload bytes of a strided view (what pack() copies to the host)."""
    raw = np.ascontiguousarray(storage).view(np.uint8)
    total = int(np.prod(shape)) if shape else 1
    out = np.empty(total * esize, np.uint8)
    nd = len(shape)
    sh = (ctypes.c_int64 * max(1, nd))(*shape)
    st = (ctypes.c_int64 * max(1, nd))(*stride)
    base = raw[offset * esize:]
    lib().oracle_gather(base.ctypes.data_as(ctypes.c_void_p), esize, nd, ctypes.cast(sh, ctypes.c_void_p),
                        ctypes.cast(st, ctypes.c_void_p), out.ctypes.data_as(ctypes.c_void_p))
    return out.tobytes()


def hadamard(x: np.ndarray, group: int, kind: int) -> np.ndarray:
    """Grouped normalised Hadamard rotation of the last dimension, each stage rounded to
    ``kind`` (w8_oracle.c: oracle_hadamard; reference training/quant_kernels.py:231-277,
    :376-426)."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    cols = a.shape[-1]
    rows = a.size // cols if cols else 0
    out = np.empty_like(a)
    lib().oracle_hadamard(_p(a), rows, cols, group, kind, _p(out))
    return out

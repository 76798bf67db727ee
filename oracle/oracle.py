"""CPU oracle for the W4A16 decode GEMV -- TEST INFRASTRUCTURE ONLY.

This module is the parity checker and the timed CPU baseline.  It is imported
only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm.  The library (decode-kernel_b200/) never imports it and has no CPU
fallback.

Two restatements of RohanDisa/decode-kernel's reference path live here:

* ``libdk_oracle.so`` (dk_oracle.c), plain C, scalar: the bit-exact quantizer
  (python/decode_kernel/quantize.py:26-51), unpack (:54-63), dequantize
  (:66-78) and an fp32 dequantize-then-dot with a double accumulator
  (python/decode_kernel/reference.py:17-26).  Used for parity at small sizes
  and on sampled rows of large matrices.
* numpy versions of the same functions (``*_np``): vectorised, and
  ``linear_fp32_np`` keeps the reference's shape of work -- materialise the
  fp32 dequantized matrix, then one fp32 BLAS matmul -- so it is what the CPU
  baseline times.

Both are pinned against vectors produced by the reference itself
(tests/golden/make_golden.py).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

GROUP_SIZE = 128
NIBBLES_PER_WORD = 8
QMIN, QMAX = -7, 7

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "libdk_oracle.so"
_lib = None


def build() -> Path:
    """Compile dk_oracle.c with the committed Makefile (gcc, no fast-math)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        L = ctypes.CDLL(str(_LIB_PATH))
        i64, p = ctypes.c_int64, ctypes.c_void_p
        L.dko_quantize_pack.argtypes = [p, i64, i64, p, p]
        L.dko_quantize_pack.restype = ctypes.c_int
        L.dko_unpack_to_int.argtypes = [p, i64, i64, p]
        L.dko_dequantize.argtypes = [p, p, i64, i64, p]
        L.dko_linear_fp32.argtypes = [p, p, p, i64, i64, i64, p]
        L.dko_linear_fp32_rows.argtypes = [p, p, p, i64, i64, i64, i64, i64, p]
        L.dko_f32_to_f16.argtypes = [ctypes.c_float]
        L.dko_f32_to_f16.restype = ctypes.c_uint16
        L.dko_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.dko_f16_to_f32.restype = ctypes.c_float
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# --------------------------------------------------------------------------
# C restatement (scalar, exact)
# --------------------------------------------------------------------------


def quantize_and_pack(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """W fp32 [M, K] -> (packed int32 [M, K/8], scales as fp16 bit patterns
    uint16 [M, K/128]).  Bit-exact with quantize.py:26-51 on CPU."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("weight must be [M, K]")
    m, k = w.shape
    if k % GROUP_SIZE:
        raise ValueError(f"K={k} is not divisible by group_size={GROUP_SIZE}")
    packed = np.empty((m, k // NIBBLES_PER_WORD), dtype=np.int32)
    scales = np.empty((m, k // GROUP_SIZE), dtype=np.uint16)
    rc = lib().dko_quantize_pack(_ptr(w), m, k, _ptr(packed), _ptr(scales))
    if rc != 0:
        raise ValueError("dko_quantize_pack rejected the shape")
    return packed, scales


def unpack_to_int(packed: np.ndarray) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    m, words = packed.shape
    q = np.empty((m, words * NIBBLES_PER_WORD), dtype=np.int8)
    lib().dko_unpack_to_int(_ptr(packed), m, words * NIBBLES_PER_WORD, _ptr(q))
    return q


def dequantize(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    m, words = packed.shape
    k = words * NIBBLES_PER_WORD
    w = np.empty((m, k), dtype=np.float32)
    lib().dko_dequantize(_ptr(packed), _ptr(scales), m, k, _ptr(w))
    return w


def linear_fp32(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
                rows: tuple[int, int] | None = None) -> np.ndarray:
    """y fp32 [B, M] = x[B, K] . dequant(W)^T (reference.py:17-26).

    ``x`` is fp16 (np.float16 or its uint16 bit pattern), 1-D or [B, K].
    ``rows=(m0, m1)`` computes only those output rows (the rest are NaN).
    """
    xb = _as_f16_bits(x)
    if xb.ndim == 1:
        xb = xb[None, :]
    packed = np.ascontiguousarray(packed, dtype=np.int32)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    m, words = packed.shape
    k = words * NIBBLES_PER_WORD
    b = xb.shape[0]
    if xb.shape[1] != k:
        raise ValueError("x.shape[1] must equal K")
    y = np.full((b, m), np.nan, dtype=np.float32)
    m0, m1 = rows if rows is not None else (0, m)
    lib().dko_linear_fp32_rows(_ptr(xb), _ptr(packed), _ptr(scales), m, k, b,
                               m0, m1, _ptr(y))
    return y


def f32_to_f16_bits(v: float) -> int:
    return int(lib().dko_f32_to_f16(float(v)))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().dko_f16_to_f32(int(h)))


def _as_f16_bits(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x)
    if x.dtype == np.float16:
        x = x.view(np.uint16)
    if x.dtype != np.uint16:
        raise TypeError("x must be float16 or its uint16 bit pattern")
    return np.ascontiguousarray(x)


# --------------------------------------------------------------------------
# numpy restatement (vectorised; same arithmetic)
# --------------------------------------------------------------------------


def quantize_and_pack_np(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Vectorised twin of ``quantize_and_pack`` (IEEE fp32 division,
    np.rint = round half to even, fp16 RNE)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    m, k = w.shape
    if k % GROUP_SIZE:
        raise ValueError(f"K={k} is not divisible by group_size={GROUP_SIZE}")
    g = w.reshape(m, k // GROUP_SIZE, GROUP_SIZE)
    amax = np.abs(g).max(axis=-1)
    scale = np.maximum(amax / np.float32(QMAX), np.float32(1e-8)).astype(np.float32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        q = np.clip(np.rint(g / scale[..., None]), QMIN, QMAX)
    q = np.nan_to_num(q, nan=0.0).astype(np.int32).reshape(m, k // NIBBLES_PER_WORD,
                                                           NIBBLES_PER_WORD)
    nib = (q & 0xF).astype(np.uint32)
    shifts = (4 * np.arange(NIBBLES_PER_WORD, dtype=np.uint32))
    packed = np.bitwise_or.reduce(nib << shifts, axis=-1).view(np.int32)
    with np.errstate(over="ignore"):
        scales = scale.astype(np.float16).view(np.uint16)
    return np.ascontiguousarray(packed), np.ascontiguousarray(scales)


def unpack_to_int_np(packed: np.ndarray) -> np.ndarray:
    p = np.ascontiguousarray(packed).view(np.uint32)
    m, words = p.shape
    shifts = (4 * np.arange(NIBBLES_PER_WORD, dtype=np.uint32))
    nib = ((p[:, :, None] >> shifts) & 0xF).astype(np.int8)
    nib = np.where(nib >= 8, nib - 16, nib).astype(np.int8)
    return nib.reshape(m, words * NIBBLES_PER_WORD)


def dequantize_np(packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    q = unpack_to_int_np(packed).astype(np.float32)
    m, k = q.shape
    s = np.ascontiguousarray(scales, dtype=np.uint16).view(np.float16).astype(np.float32)
    return (q.reshape(m, k // GROUP_SIZE, GROUP_SIZE) * s[..., None]).reshape(m, k)


def linear_fp32_np(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
                   threads: int | None = None) -> np.ndarray:
    """The reference's CPU path restated in numpy: materialise fp32 W, then an
    fp32 matmul (reference.py:17-26).  The rows are split over ``threads``
    host threads (default: every core this process may run on); each thread
    dequantizes its row block and multiplies it with one-thread BLAS, so the
    whole host works on the dequantisation, which dominates at small batch."""
    xf = _as_f16_bits(x).view(np.float16).astype(np.float32)
    if xf.ndim == 1:
        xf = xf[None, :]
    m = packed.shape[0]
    n = max(1, min(threads or cpu_threads(), m // 64 or 1))
    if n == 1:
        return xf @ dequantize_np(packed, scales).T
    from concurrent.futures import ThreadPoolExecutor

    from threadpoolctl import threadpool_limits

    out = np.empty((xf.shape[0], m), dtype=np.float32)
    bounds = [m * i // n for i in range(n + 1)]

    def work(i: int) -> None:
        a, b = bounds[i], bounds[i + 1]
        out[:, a:b] = xf @ dequantize_np(packed[a:b], scales[a:b]).T

    with threadpool_limits(1, user_api="blas"), ThreadPoolExecutor(n) as ex:
        list(ex.map(work, range(n)))
    return out


def cpu_threads() -> int:
    """Host threads linear_fp32_np uses by default: the cores this process may
    run on."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1

"""W4A16 decode GEMV for NVIDIA B200 (sm_100a).

Drop-in for RohanDisa/decode-kernel's Python API (python/decode_kernel/
__init__.py:11-83): ``gemv``, ``w4a16_linear``, ``cuda_available``,
``quantize_and_pack``, ``dequantize``, ``GROUP_SIZE``, backed by this
repository's CUDA library (``libdk_b200.so``, C ABI in include/dk_w4a16.h)
through the torch extension ``decode_kernel._cuda``.

There is no CPU fallback: when the extension or a GPU is missing these
functions raise.
"""

from __future__ import annotations

from typing import Optional

import torch

from .quantize import GROUP_SIZE, dequantize, quantize_and_pack, quantize_and_pack_cuda

__all__ = [
    "GROUP_SIZE",
    "cuda_available",
    "dequantize",
    "gemv",
    "gemv_out",
    "quantize_and_pack",
    "quantize_and_pack_cuda",
    "w4a16_linear",
]


def cuda_available() -> bool:
    """True when a CUDA device is visible and the extension imports."""
    if not torch.cuda.is_available():
        return False
    try:
        from . import _cuda  # noqa: F401

        return True
    except Exception:
        return False


def gemv(
    packed: torch.Tensor,
    scales: torch.Tensor,
    x: torch.Tensor,
    version: int = 5,
    split_k: int = 4,
    reuse_weights: bool = False,
    warps_per_row: int = 1,
) -> torch.Tensor:
    """Y[B, M] = dequant(W)[M, K] . X[B, K]^T in one kernel launch.

    packed: int32 [M, K/8]; scales: fp16 [M, K/128]; x: fp16 [B, K] or [K].
    ``version`` 0..5 picks a member of the kernel family (5, the default, is
    the persistent bulk-copy pipeline); ``reuse_weights`` the batch path.
    """
    from . import _cuda

    if x.dim() == 1:
        x = x.unsqueeze(0)
    return _cuda.w4a16_gemv(
        packed, scales, x, int(version), int(split_k), bool(reuse_weights), int(warps_per_row)
    )


def gemv_out(
    packed: torch.Tensor,
    scales: torch.Tensor,
    x: torch.Tensor,
    y: torch.Tensor,
    version: int = 5,
    reuse_weights: bool = False,
    pdl: bool = False,
) -> torch.Tensor:
    """``gemv`` into a preallocated fp16 ``y`` [B, M].

    ``pdl=True`` launches with programmatic dependent launch: the kernel may
    begin while the previous kernel on the stream finishes and streams its
    weights early.  Only valid when that previous kernel does not write
    ``packed`` or ``scales``.
    """
    from . import _cuda

    if x.dim() == 1:
        x = x.unsqueeze(0)
    if y.dim() == 1:
        y = y.unsqueeze(0)
    _cuda.w4a16_gemv_out(packed, scales, x, y, int(version), 4, bool(reuse_weights), 1, bool(pdl))
    return y


def w4a16_linear(
    x: torch.Tensor,
    packed: torch.Tensor,
    scales: torch.Tensor,
    version: int = 5,
    split_k: Optional[int] = None,
    reuse_weights: Optional[bool] = None,
) -> torch.Tensor:
    """Bias-free quantized ``F.linear``: returns x . dequant(W)^T, [B, M]."""
    if split_k is None:
        split_k = 4 if version == 4 else 1
    if reuse_weights is None:
        reuse_weights = x.dim() == 2 and x.size(0) > 1
    return gemv(
        packed,
        scales,
        x,
        version=version,
        split_k=split_k,
        reuse_weights=reuse_weights,
        warps_per_row=1,
    )

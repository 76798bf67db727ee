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
    "W4A16Linear",
    "cuda_available",
    "gemv_multi",
    "gemv_silu_mul",
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


def gemv_multi(weights, x: torch.Tensor, pdl: bool = False, reuse_weights: bool = False):
    """Several matrices that share ``x`` (q/k/v, gate/up) in one launch.

    ``weights``: up to 4 ``(packed, scales)`` pairs with the same K.  Returns
    one fp16 [B, M_i] tensor per pair, each bit-identical to ``gemv`` of that
    pair (the streaming kernel runs over the concatenated row tiles).
    """
    from . import capi

    if x.dim() == 1:
        x = x.unsqueeze(0)
    if not weights or len(weights) > capi.DK_MAX_SEGMENTS:
        raise RuntimeError(f"gemv_multi takes 1..{capi.DK_MAX_SEGMENTS} weight pairs")
    K = x.shape[1]
    if x.dtype != torch.float16 or not x.is_cuda or not x.is_contiguous():
        raise RuntimeError("x must be a contiguous CUDA fp16 tensor")
    for p, s in weights:
        if p.dtype != torch.int32 or s.dtype != torch.float16 or not (p.is_cuda and s.is_cuda):
            raise RuntimeError("packed must be CUDA int32 and scales CUDA fp16")
        if p.device != x.device or s.device != x.device:
            raise RuntimeError("packed and scales must be on x's device")
        if p.shape[1] * 8 != K or s.shape != (p.shape[0], K // GROUP_SIZE):
            raise RuntimeError("every matrix must be [M, K/8] with scales [M, K/128] for x's K")
        if not (p.is_contiguous() and s.is_contiguous()):
            raise RuntimeError("packed and scales must be contiguous")
    ys = [torch.empty((x.shape[0], p.shape[0]), dtype=torch.float16, device=x.device)
          for p, _ in weights]
    flags = capi.DK_FLAG_PDL if pdl else 0
    cfg = capi.default_config(reuse_weights=int(bool(reuse_weights)), flags=flags)
    with torch.cuda.device(x.device):  # the C ABI launches on the current device
        capi.check(capi.gemv_multi([p.data_ptr() for p, _ in weights],
                                   [s.data_ptr() for _, s in weights],
                                   [p.shape[0] for p, _ in weights], [y.data_ptr() for y in ys],
                                   x.data_ptr(), K, x.shape[0], cfg,
                                   torch.cuda.current_stream(x.device).cuda_stream),
                   "dk_w4a16_gemv_multi")
    return ys


def _check_pair(packed: torch.Tensor, scales: torch.Tensor, K: int, device: torch.device) -> None:
    if packed.dtype != torch.int32 or scales.dtype != torch.float16 or not (
            packed.is_cuda and scales.is_cuda):
        raise RuntimeError("packed must be CUDA int32 and scales CUDA fp16")
    if packed.device != device or scales.device != device:
        raise RuntimeError("packed and scales must be on x's device")
    if packed.dim() != 2 or packed.shape[1] * 8 != K or scales.shape != (packed.shape[0],
                                                                          K // GROUP_SIZE):
        raise RuntimeError("every matrix must be [M, K/8] with scales [M, K/128] for x's K")
    if not (packed.is_contiguous() and scales.is_contiguous()):
        raise RuntimeError("packed and scales must be contiguous")


def gemv_silu_mul(gate, up, x: torch.Tensor, pdl: bool = False, reuse_weights: bool = False):
    """The gate/up pair of a gated MLP with its SiLU-mul epilogue, one launch.

    ``gate`` and ``up``: ``(packed, scales)`` of two [M, K] matrices.  Returns
    fp16 [B, M] ``h = silu(gemv(gate, x)) * gemv(up, x)`` with the roundings of
    that unfused fp16 sequence (``torch.nn.functional.silu`` then ``*``).
    """
    from . import capi

    if x.dim() == 1:
        x = x.unsqueeze(0)
    if x.dtype != torch.float16 or not x.is_cuda or not x.is_contiguous() or x.dim() != 2:
        raise RuntimeError("x must be a contiguous 2-D CUDA fp16 tensor")
    K = x.shape[1]
    _check_pair(*gate, K, x.device)
    _check_pair(*up, K, x.device)
    if gate[0].shape != up[0].shape:
        raise RuntimeError("gate and up must have the same shape")
    M = gate[0].shape[0]
    h = torch.empty((x.shape[0], M), dtype=torch.float16, device=x.device)
    flags = capi.DK_FLAG_PDL if pdl else 0
    cfg = capi.default_config(reuse_weights=int(bool(reuse_weights)), flags=flags)
    with torch.cuda.device(x.device):  # the C ABI launches on the current device
        capi.check(capi.gemv_silu_mul(gate[0].data_ptr(), gate[1].data_ptr(), up[0].data_ptr(),
                                      up[1].data_ptr(), x.data_ptr(), h.data_ptr(), M, K,
                                      x.shape[0], cfg,
                                      torch.cuda.current_stream(x.device).cuda_stream),
                   "dk_w4a16_gemv_silu_mul")
    return h


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


from .ops import W4A16Linear  # noqa: E402  (registers torch.ops.decode_kernel.w4a16_linear)

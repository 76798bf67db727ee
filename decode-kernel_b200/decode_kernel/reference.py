"""fp32 dequantize-then-matmul, the accuracy yardstick of the reference's API.

Kept because code written against RohanDisa/decode-kernel imports it
(``python/decode_kernel/reference.py:17-30``; its GPU tests compare every
kernel to it at max-abs 1e-2).  It is a test helper: no GEMV in this package
calls it, and there is no CPU fallback -- ``decode_kernel.gemv`` always runs
the CUDA kernels or raises.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from .quantize import dequantize


def linear_fp32(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Y[B, M] = X . dequant(W)^T in fp32 on the CPU; x may be [K] or [B, K]."""
    w = dequantize(packed.cpu(), scales.cpu(), dtype=torch.float32)
    xf = x.detach().cpu().float()
    if xf.dim() == 1:
        xf = xf.unsqueeze(0)
    return F.linear(xf, w)


def max_abs_err(y_kernel: torch.Tensor, y_ref: torch.Tensor) -> float:
    return (y_kernel.float().cpu() - y_ref.float().cpu()).abs().max().item()

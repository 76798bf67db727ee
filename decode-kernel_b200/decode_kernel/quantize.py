"""The W4A16 weight format: symmetric signed int4, one fp16 scale per 128
weights along K, eight values per int32 word, low nibble first.

Same functions, signatures and results as RohanDisa/decode-kernel's
``python/decode_kernel/quantize.py``:

* ``quantize_and_pack`` (reference :26-51) -- torch ops, so on any device it
  produces exactly what the reference produces on that device:
  ``scale = max(amax / 7, 1e-8)`` in fp32, ``q = round_half_even(w / scale)``
  clamped to [-7, 7], nibble ``q & 0xF`` at bit ``4 * (k % 8)``, scale stored
  as fp16.  (-8 decodes but is never produced.)
* ``unpack_to_int`` (:54-63), ``dequantize`` (:66-78).

``quantize_and_pack_cuda`` runs the same quantizer as one CUDA kernel of this
library; it matches the CPU result bit for bit (or the torch-on-CUDA result
with ``torch_cuda_scale=True``).
"""

from __future__ import annotations

import torch

GROUP_SIZE = 128
NIBBLES_PER_WORD = 8
QMIN, QMAX = -7, 7

_SHIFTS = tuple(4 * n for n in range(NIBBLES_PER_WORD))


def _check_shape(weight: torch.Tensor, group_size: int) -> tuple[int, int]:
    if weight.dim() != 2:
        raise ValueError("weight must be [M, K]")
    m, k = weight.shape
    if k % group_size != 0:
        raise ValueError(f"K={k} is not divisible by group_size={group_size}")
    if k % NIBBLES_PER_WORD != 0:
        raise ValueError(f"K={k} is not divisible by {NIBBLES_PER_WORD}")
    return m, k


def quantize_and_pack(
    weight: torch.Tensor, group_size: int = GROUP_SIZE
) -> tuple[torch.Tensor, torch.Tensor]:
    """W[M, K] -> (packed int32 [M, K/8], fp16 scales [M, K/group_size])."""
    m, k = _check_shape(weight, group_size)
    per_group = weight.float().reshape(m, k // group_size, group_size)
    scale = (per_group.abs().amax(dim=-1) / float(QMAX)).clamp(min=1e-8)
    q = (per_group / scale[..., None]).round().clamp(QMIN, QMAX).to(torch.int32)
    # Nibble n of a word sits at bit 4n; the fields are disjoint, so a sum of
    # shifted nibbles is their OR.  Summed in int64, then folded to the int32
    # bit pattern.
    nib = (q.reshape(m, k // NIBBLES_PER_WORD, NIBBLES_PER_WORD) & 0xF).to(torch.int64)
    shifts = torch.tensor(_SHIFTS, dtype=torch.int64, device=nib.device)
    word = (nib << shifts).sum(dim=-1)
    packed = ((word ^ 0x80000000) - 0x80000000).to(torch.int32)
    return packed.contiguous(), scale.half().contiguous()


def unpack_to_int(packed: torch.Tensor) -> torch.Tensor:
    """Packed int32 words -> signed q values in [-8, 7], int32 [M, K]."""
    m, words = packed.shape
    shifts = torch.tensor(_SHIFTS, dtype=torch.int32, device=packed.device)
    nib = (packed.unsqueeze(-1) >> shifts) & 0xF
    q = nib - ((nib & 0x8) << 1)  # two's complement of the 4-bit field
    return q.reshape(m, words * NIBBLES_PER_WORD).to(torch.int32)


def dequantize(
    packed: torch.Tensor,
    scales: torch.Tensor,
    group_size: int = GROUP_SIZE,
    dtype: torch.dtype = torch.float32,
) -> torch.Tensor:
    """Materialise q * scale as a dense [M, K] matrix (tests and tools only;
    the GEMV kernels never build it)."""
    q = unpack_to_int(packed).to(dtype)
    m, k = q.shape
    s = scales.to(dtype).reshape(m, k // group_size, 1)
    return (q.reshape(m, k // group_size, group_size) * s).reshape(m, k)


def quantize_and_pack_cuda(
    weight: torch.Tensor, torch_cuda_scale: bool = False
) -> tuple[torch.Tensor, torch.Tensor]:
    """``quantize_and_pack`` as one CUDA kernel (dk_quantize_pack).

    Bit-exact with ``quantize_and_pack`` evaluated on the CPU; with
    ``torch_cuda_scale=True``, bit-exact with it evaluated on a CUDA tensor.
    """
    from . import _cuda

    _check_shape(weight, GROUP_SIZE)
    w = weight if weight.is_cuda else weight.cuda()
    packed, scales = _cuda.quantize_pack(w.float().contiguous(), bool(torch_cuda_scale))
    return packed, scales

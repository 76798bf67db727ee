"""Import and export of GPTQ-format int4 checkpoints.

GPTQ checkpoints are the usual input of the Marlin W4A16 kernels (vLLM's
``gptq_marlin_repack`` takes them).  Their 4-bit symmetric form holds the
same numbers as this library's format, laid out differently:

================  ====================================  ===========================
tensor            GPTQ (sym, group 128, no act-order)   this library
================  ====================================  ===========================
quantized values  ``qweight`` int32 ``[K/8, N]``:       ``packed`` int32 ``[M, K/8]``:
                  nibble i of word ``[r, n]`` is         nibble i of word ``[m, r]``
                  ``u = q + 8`` of ``k = 8r + i``        is ``q & 0xF`` of ``k = 8r + i``
scales            fp16 ``[K/128, N]``                    fp16 ``[M, K/128]``
zero points       ``qzeros`` int32 ``[K/128, N/8]``,     none (symmetric)
                  8 in every nibble (7 in the older
                  serialisation that stores zero - 1)
group index       ``g_idx[k] = k // 128``                implied
================  ====================================  ===========================

Both decode to ``w = q * scale`` with ``q`` in [-8, 7].  Since ``(q & 0xF) ^ 8
== q + 8`` for every 4-bit ``q``, a word converts with one XOR of 0x88888888,
and the matrices are transposes of each other (N = M output rows).  The
conversion is exact in both directions.  Checkpoints that this format cannot
hold are rejected with ``ValueError``: group sizes other than 128,
asymmetric zero points, and act-order (``desc_act``) checkpoints whose
``g_idx`` permutes K.

These are offline tools for loading and exporting weights, written in torch
ops, so they run on whatever device the tensors are on.  The GEMV kernels
read only the library's own layout.
"""

from __future__ import annotations

from typing import NamedTuple, Optional

import torch

from .quantize import GROUP_SIZE, NIBBLES_PER_WORD

# 0x88888888 and 0x77777777 as int32 bit patterns.
_XOR_BIAS = 0x88888888 - (1 << 32)
_ZEROS_8 = 0x88888888 - (1 << 32)
_ZEROS_7 = 0x77777777


class GPTQWeights(NamedTuple):
    """One linear layer's tensors under the GPTQ checkpoint names."""

    qweight: torch.Tensor  # int32 [K/8, N]
    qzeros: torch.Tensor   # int32 [K/128, ceil(N/8)]
    scales: torch.Tensor   # fp16 [K/128, N]
    g_idx: torch.Tensor    # int32 [K]


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _group_index(k: int, device) -> torch.Tensor:
    return torch.arange(k, dtype=torch.int32, device=device) // GROUP_SIZE


def to_gptq(packed: torch.Tensor, scales: torch.Tensor, *,
            zeros_minus_one: bool = False) -> GPTQWeights:
    """This library's ``(packed [M, K/8], scales [M, K/128])`` as GPTQ tensors.

    GPTQ's N is this library's M.  ``qzeros`` carries the symmetric zero
    point 8 in every nibble, or 7 with ``zeros_minus_one=True`` (the
    serialisation that stores zero - 1); when M % 8 != 0 the unused nibbles of
    each row's last ``qzeros`` word hold the same value.
    """
    _check(packed.dtype == torch.int32 and packed.dim() == 2, "packed must be int32 [M, K/8]")
    _check(scales.dtype == torch.float16 and scales.dim() == 2, "scales must be fp16 [M, K/128]")
    m, words = packed.shape
    k = words * NIBBLES_PER_WORD
    _check(k % GROUP_SIZE == 0, f"K={k} is not divisible by {GROUP_SIZE}")
    _check(tuple(scales.shape) == (m, k // GROUP_SIZE),
           f"scales must be [{m}, {k // GROUP_SIZE}], got {list(scales.shape)}")
    qweight = torch.bitwise_xor(packed, _XOR_BIAS).t().contiguous()
    zword = _ZEROS_7 if zeros_minus_one else _ZEROS_8
    qzeros = torch.full((k // GROUP_SIZE, (m + 7) // 8), zword, dtype=torch.int32,
                        device=packed.device)
    return GPTQWeights(qweight, qzeros, scales.t().contiguous(), _group_index(k, packed.device))


def from_gptq(qweight: torch.Tensor, scales: torch.Tensor,
              qzeros: Optional[torch.Tensor] = None, g_idx: Optional[torch.Tensor] = None, *,
              zeros_minus_one: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """GPTQ tensors -> this library's ``(packed int32 [N, K/8], scales fp16 [N, K/128])``.

    ``qzeros`` (optional) must hold 8 in every nibble of the N real columns,
    or 7 with ``zeros_minus_one=True``.  ``g_idx`` (optional) must be the
    identity grouping ``k // 128``.  The result may contain q = -8 (GPTQ's
    u = 0), which the kernels decode although this library's quantizer,
    like the reference's, never produces it.
    """
    _check(qweight.dtype == torch.int32 and qweight.dim() == 2, "qweight must be int32 [K/8, N]")
    _check(scales.dim() == 2 and scales.dtype == torch.float16,
           "scales must be fp16 [K/group, N]")
    words, n = qweight.shape
    k = words * NIBBLES_PER_WORD
    _check(scales.shape[1] == n, f"scales must have {n} columns, got {scales.shape[1]}")
    _check(scales.shape[0] > 0 and k % scales.shape[0] == 0,
           f"K={k} is not a whole number of scale groups ({scales.shape[0]})")
    group = k // scales.shape[0]
    _check(group == GROUP_SIZE, f"group size {group} is not {GROUP_SIZE}")
    if qzeros is not None:
        _check(qzeros.dtype == torch.int32 and tuple(qzeros.shape) == (k // GROUP_SIZE, (n + 7) // 8),
               f"qzeros must be int32 [{k // GROUP_SIZE}, {(n + 7) // 8}]")
        shifts = torch.arange(0, 32, 4, dtype=torch.int32, device=qzeros.device)
        z = ((qzeros.unsqueeze(-1) >> shifts) & 0xF).reshape(qzeros.shape[0], -1)[:, :n]
        want = 7 if zeros_minus_one else 8
        _check(bool((z == want).all()),
               f"zero points must all be {want} (symmetric int4); asymmetric checkpoints "
               "cannot be represented in this format")
    if g_idx is not None:
        _check(g_idx.dim() == 1 and g_idx.numel() == k, f"g_idx must have K={k} entries")
        _check(bool(torch.equal(g_idx.to(torch.int64).cpu(),
                                _group_index(k, "cpu").to(torch.int64))),
               "g_idx is not k // 128: act-order (desc_act) checkpoints permute K and "
               "cannot be represented in this format")
    packed = torch.bitwise_xor(qweight, _XOR_BIAS).t().contiguous()
    return packed, scales.t().contiguous()

"""The W4A16 GEMV as a PyTorch operator and module.

``torch.ops.decode_kernel.w4a16_linear(x, packed, scales) -> y`` is a
``torch.library`` custom op around this package's CUDA kernel (the caller
side of the reference's ``w4a16_linear``, python/decode_kernel/__init__.py:
62-83): it has a fake (meta) implementation, so code that traces or captures
-- torch.fx, ``torch.cuda.CUDAGraph`` capture of a decode step -- sees a
proper operator with a known output shape instead of an opaque Python call.
``W4A16Linear`` is a bias-free ``nn.Linear`` replacement holding the packed
weights and scales as buffers.  ``torch.ops.decode_kernel.w4a16_silu_mul(x,
packed_gate, scales_gate, packed_up, scales_up)`` is a gated MLP's gate/up
pair with its SiLU-mul epilogue in one launch.

There is no CPU implementation: the op raises on CPU tensors, like the rest of
the package.
"""

from __future__ import annotations

from typing import Optional

import torch

from .quantize import GROUP_SIZE, quantize_and_pack_cuda

__all__ = ["W4A16Linear", "w4a16_linear_op", "w4a16_silu_mul_op"]


@torch.library.custom_op("decode_kernel::w4a16_linear", mutates_args=())
def w4a16_linear_op(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """y[..., M] = x[..., K] . dequant(W)^T (fp16), any number of leading dims."""
    from . import gemv

    if not x.is_cuda:
        raise RuntimeError("decode_kernel::w4a16_linear runs on CUDA tensors only")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    y = gemv(packed, scales, x2)
    return y.reshape(*lead, packed.shape[0])


@w4a16_linear_op.register_fake
def _(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    torch._check(x.shape[-1] == packed.shape[1] * 8, lambda: "x.shape[-1] must equal K")
    torch._check(x.dtype == torch.float16, lambda: "x must be fp16")
    return x.new_empty((*x.shape[:-1], packed.shape[0]), dtype=torch.float16)


@torch.library.custom_op("decode_kernel::w4a16_silu_mul", mutates_args=())
def w4a16_silu_mul_op(x: torch.Tensor, packed_gate: torch.Tensor, scales_gate: torch.Tensor,
                      packed_up: torch.Tensor, scales_up: torch.Tensor) -> torch.Tensor:
    """h[..., M] = silu(x . Wg^T) * (x . Wu^T) (fp16), one launch for both GEMVs."""
    from . import gemv_silu_mul

    if not x.is_cuda:
        raise RuntimeError("decode_kernel::w4a16_silu_mul runs on CUDA tensors only")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    h = gemv_silu_mul((packed_gate, scales_gate), (packed_up, scales_up), x2)
    return h.reshape(*lead, packed_gate.shape[0])


@w4a16_silu_mul_op.register_fake
def _(x, packed_gate, scales_gate, packed_up, scales_up):
    torch._check(x.shape[-1] == packed_gate.shape[1] * 8, lambda: "x.shape[-1] must equal K")
    torch._check(packed_up.shape[0] == packed_gate.shape[0], lambda: "gate and up rows differ")
    torch._check(x.dtype == torch.float16, lambda: "x must be fp16")
    return x.new_empty((*x.shape[:-1], packed_gate.shape[0]), dtype=torch.float16)


class W4A16Linear(torch.nn.Module):
    """Bias-free linear layer with symmetric int4 weights (group 128 along K,
    fp16 scales), computed by the B200 GEMV kernels."""

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor):
        super().__init__()
        if packed.dtype != torch.int32 or scales.dtype != torch.float16:
            raise ValueError("packed must be int32 [M, K/8] and scales fp16 [M, K/128]")
        if scales.shape != (packed.shape[0], packed.shape[1] * 8 // GROUP_SIZE):
            raise ValueError("scales shape must be [M, K/128]")
        self.register_buffer("packed", packed.contiguous())
        self.register_buffer("scales", scales.contiguous())

    @property
    def in_features(self) -> int:
        return self.packed.shape[1] * 8

    @property
    def out_features(self) -> int:
        return self.packed.shape[0]

    @classmethod
    def from_linear(cls, linear: torch.nn.Linear, device: Optional[torch.device] = None) -> "W4A16Linear":
        """Quantize an ``nn.Linear``'s weight (the reference quantizer's
        arithmetic, on the GPU); a bias is refused."""
        if linear.bias is not None:
            raise ValueError("W4A16Linear has no bias")
        w = linear.weight.detach().to(device or "cuda", torch.float32)
        packed, scales = quantize_and_pack_cuda(w)
        return cls(packed, scales)

    @classmethod
    def from_gptq(cls, qweight: torch.Tensor, scales: torch.Tensor,
                  qzeros: Optional[torch.Tensor] = None, g_idx: Optional[torch.Tensor] = None, *,
                  zeros_minus_one: bool = False) -> "W4A16Linear":
        """A layer from a symmetric 4-bit GPTQ checkpoint's tensors (group 128,
        no act-order), converted exactly by ``decode_kernel.gptq.from_gptq``;
        the buffers stay on the tensors' device."""
        from .gptq import from_gptq

        packed, s = from_gptq(qweight, scales, qzeros, g_idx, zeros_minus_one=zeros_minus_one)
        return cls(packed, s)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return torch.ops.decode_kernel.w4a16_linear(x, self.packed, self.scales)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bits=4, group={GROUP_SIZE}"

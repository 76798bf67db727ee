"""Exact properties of every GEMV path at the full BASELINE and 70B shapes,
checked on every output row.

At these sizes the oracle runs on sampled rows only (test_gemv_gpu.py).
The properties below need no oracle and hold bit for bit, because every
operation in the kernels is sign-symmetric and exact under scaling by two:
the int4 unpack, fp16 x, products, fp32 sums with round-to-nearest, and the
final fp16 rounding.

* determinism: two calls return the same bits (fixed reduction order, no
  atomics);
* odd symmetry: y(-x) == -y(x);
* homogeneity: y(2x) == 2 y(x), and doubling every group scale doubles y.
  Outputs in fp16's subnormal range, whose rounding grid is fixed, are left
  out of this check.

The weights are random packed words, so every nibble value occurs, -8
included (the reference's quantizer never writes -8; its kernels decode it,
quantize.py:10-11).
"""

from __future__ import annotations

import pytest
import torch

from dkhelpers import capi_gemv

pytestmark = pytest.mark.gpu

SHAPES = [(4096, 4096), (11008, 4096), (4096, 11008), (28672, 8192), (8192, 28672)]
MIN_NORMAL = 2.0 ** -14


def _problem(M, K, B, seed):
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(seed)
    packed = torch.randint(-2**31, 2**31 - 1, (M, K // 8), generator=g, device=dev,
                           dtype=torch.int32)
    scales = (torch.rand(M, K // 128, generator=g, device=dev) * 0.02 + 0.001).half()
    x = torch.randn(B, K, generator=g, device=dev).half()
    return packed, scales, x


def _configs(B):
    from decode_kernel import capi

    out = [("v5", capi.default_config()), ("reuse", capi.default_config(reuse_weights=1))]
    if B <= 8:
        out += [("v3", capi.default_config(version=3)),
                ("v4", capi.default_config(version=4, split_k=4))]
    return out


def _doubled(y2, y):
    """y2 == 2 y wherever y is a normal fp16 number."""
    keep = y.float().abs() >= MIN_NORMAL
    return torch.equal(y2[keep], (2 * y)[keep])


@pytest.mark.slow
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("batch", [1, 8, 32])
def test_exact_properties_full_size(shape, batch, cuda_device):
    from decode_kernel import capi

    M, K = shape
    packed, scales, x = _problem(M, K, batch, seed=M + K + batch)
    for name, c in _configs(batch):
        y = capi_gemv(packed, scales, x, c)
        assert torch.isfinite(y).all(), name
        assert torch.equal(capi_gemv(packed, scales, x, c), y), f"{name}: not deterministic"
        assert torch.equal(capi_gemv(packed, scales, -x, c), -y), f"{name}: y(-x) != -y(x)"
        assert _doubled(capi_gemv(packed, scales, 2 * x, c), y), f"{name}: y(2x) != 2y(x)"
        assert _doubled(capi_gemv(packed, 2 * scales, x, c), y), f"{name}: 2 scales != 2y"
    assert capi.load().dk_device_error(-1, 0) == 0

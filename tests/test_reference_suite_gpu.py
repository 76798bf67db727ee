"""RohanDisa/decode-kernel's own GPU correctness suite (tests/test_correctness.py)
restated against this package's drop-in API: same shapes, versions, batches,
seeds (1000+i, 1, 2, 4, 3), weight scale (randn * 0.05 on the GPU, quantized
by ``quantize_and_pack`` on the GPU), oracle (``linear_fp32``) and
tolerances.  It runs through ``decode_kernel.gemv`` -> ``decode_kernel._cuda``
-> the C ABI, exactly as a user of the reference would call it."""

from __future__ import annotations

import os

import pytest
import torch

pytestmark = pytest.mark.gpu

SHAPES = [(256, 256), (4096, 4096)]
if os.environ.get("DK_FULL_SHAPES") == "1":
    SHAPES += [(4096, 11008), (4096, 14336)]
VERSIONS = [0, 1, 2, 3, 4, 5]
MAX_ABS = 1e-2
N_RANDOM = int(os.environ.get("DK_N_RANDOM", "3"))
if os.environ.get("DK_FULL_TEST") == "1":
    N_RANDOM = 100


def _run(m, k, batch, version, seed, reuse=False):
    from decode_kernel import gemv
    from decode_kernel.quantize import quantize_and_pack
    from decode_kernel.reference import linear_fp32, max_abs_err

    torch.manual_seed(seed)
    w = torch.randn(m, k, device="cuda") * 0.05
    x = torch.randn(batch, k, device="cuda", dtype=torch.float16)
    packed, scales = quantize_and_pack(w)
    y = gemv(packed, scales, x, version=version, split_k=4 if version == 4 else 1,
             reuse_weights=reuse)
    err = max_abs_err(y, linear_fp32(x, packed, scales))
    assert err < MAX_ABS, f"max abs err {err:.4e} for v{version} M={m} K={k} B={batch} seed={seed}"
    return err


@pytest.mark.parametrize("version", VERSIONS)
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("batch", [1, 4])
def test_versions_against_fp32_reference(version, shape, batch, cuda_device):
    m, k = shape
    for i in range(N_RANDOM):
        _run(m, k, batch, version, seed=1000 + i)


def test_reuse_weights_matches_streaming(cuda_device):
    from decode_kernel import gemv
    from decode_kernel.quantize import quantize_and_pack

    torch.manual_seed(1)
    m, k, b = 256, 512, 8
    w = torch.randn(m, k, device="cuda") * 0.05
    x = torch.randn(b, k, device="cuda", dtype=torch.float16)
    packed, scales = quantize_and_pack(w)
    y_stream = gemv(packed, scales, x, version=5, reuse_weights=False)
    y_reuse = gemv(packed, scales, x, version=5, reuse_weights=True)
    assert (y_stream.float() - y_reuse.float()).abs().max().item() < 1e-3


def test_splitk_matches_v3(cuda_device):
    from decode_kernel import gemv
    from decode_kernel.quantize import quantize_and_pack

    torch.manual_seed(2)
    m, k = 256, 1024
    w = torch.randn(m, k, device="cuda") * 0.05
    x = torch.randn(1, k, device="cuda", dtype=torch.float16)
    packed, scales = quantize_and_pack(w)
    y3 = gemv(packed, scales, x, version=3)
    y4 = gemv(packed, scales, x, version=4, split_k=4)
    assert (y3.float() - y4.float()).abs().max().item() < 1e-3


def test_kernel_stamps_are_distinct(cuda_device):
    from decode_kernel import _cuda, gemv
    from decode_kernel.quantize import quantize_and_pack

    torch.manual_seed(4)
    m, k = 256, 512
    w = torch.randn(m, k, device="cuda") * 0.05
    x = torch.randn(1, k, device="cuda", dtype=torch.float16)
    packed, scales = quantize_and_pack(w)
    seen = {}
    for v in range(6):
        gemv(packed, scales, x, version=v, split_k=4 if v == 4 else 1)
        seen[v] = int(_cuda.last_kernel_stamp())
    assert seen == {0: 0, 1: 1, 2: 2, 3: 3, 4: 4, 5: 5}, seen
    gemv(packed, scales, x, version=5, reuse_weights=True)
    assert int(_cuda.last_kernel_stamp()) == 15


def test_v1_multiwarp_matches_v1(cuda_device):
    from decode_kernel import _cuda, gemv
    from decode_kernel.quantize import quantize_and_pack

    torch.manual_seed(3)
    m, k = 256, 1024
    w = torch.randn(m, k, device="cuda") * 0.05
    x = torch.randn(1, k, device="cuda", dtype=torch.float16)
    packed, scales = quantize_and_pack(w)
    y1 = gemv(packed, scales, x, version=1, warps_per_row=1)
    s1 = int(_cuda.last_kernel_stamp())
    y2 = gemv(packed, scales, x, version=1, warps_per_row=2)
    s2 = int(_cuda.last_kernel_stamp())
    y4 = gemv(packed, scales, x, version=1, warps_per_row=4)
    s4 = int(_cuda.last_kernel_stamp())
    assert s1 == 1 and s2 == 12 and s4 == 14, (s1, s2, s4)
    assert (y1.float() - y2.float()).abs().max().item() < 1e-2
    assert (y1.float() - y4.float()).abs().max().item() < 1e-2


def test_w4a16_linear_dropin(cuda_device):
    from decode_kernel import w4a16_linear
    from decode_kernel.quantize import quantize_and_pack
    from decode_kernel.reference import linear_fp32, max_abs_err

    torch.manual_seed(9)
    w = torch.randn(512, 2048, device="cuda") * 0.05
    packed, scales = quantize_and_pack(w)
    for b in (1, 3, 16):
        x = torch.randn(b, 2048, device="cuda", dtype=torch.float16)
        assert max_abs_err(w4a16_linear(x, packed, scales), linear_fp32(x, packed, scales)) < 1e-2
    x1 = torch.randn(2048, device="cuda", dtype=torch.float16)
    assert w4a16_linear(x1, packed, scales).shape == (1, 512)


def test_binding_rejects_like_reference(cuda_device):
    from decode_kernel import gemv

    packed = torch.zeros(64, 32, dtype=torch.int32, device="cuda")
    scales = torch.zeros(64, 2, dtype=torch.float16, device="cuda")
    x = torch.zeros(1, 256, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="x must be fp16"):
        gemv(packed, scales, x.float())
    with pytest.raises(RuntimeError, match=r"scales shape must be \[M, K/128\]"):
        gemv(packed, scales[:, :1].contiguous(), x)
    with pytest.raises(RuntimeError, match="x.shape\\[1\\] must equal K"):
        gemv(packed, scales, x[:, :128].contiguous())
    with pytest.raises(RuntimeError, match="warps_per_row > 1"):
        gemv(packed, scales, x, version=5, warps_per_row=2)

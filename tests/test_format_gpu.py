"""GPU format kernels (dk_quantize_pack / dk_unpack_to_int / dk_dequantize)
and the STREAM probes, checked against the oracle and the golden vectors."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

GQ = np.load(Path(__file__).resolve().parent / "golden" / "golden_quant.npz")
QCASES = sorted({k.split("/")[0] for k in GQ.files})


@pytest.mark.parametrize("case", QCASES)
def test_gpu_quantizer_matches_reference_golden(case, cuda_device):
    from decode_kernel import _cuda

    w = torch.from_numpy(GQ[f"{case}/w"]).cuda()
    packed, scales = _cuda.quantize_pack(w, False)
    np.testing.assert_array_equal(packed.cpu().numpy(), GQ[f"{case}/packed"])
    np.testing.assert_array_equal(scales.cpu().view(torch.int16).numpy().view(np.uint16),
                                  GQ[f"{case}/scales"])
    np.testing.assert_array_equal(_cuda.unpack_to_int(packed).cpu().numpy(), GQ[f"{case}/q"])
    if f"{case}/dequant" in GQ.files:
        np.testing.assert_array_equal(_cuda.dequantize(packed, scales).cpu().numpy(),
                                      GQ[f"{case}/dequant"])


@pytest.mark.parametrize("shape,std", [((4096, 4096), 0.02), ((512, 11008), 0.05)])
def test_gpu_quantizer_matches_oracle_large(shape, std, cuda_device):
    from decode_kernel.quantize import quantize_and_pack_cuda

    rng = np.random.default_rng(3)
    w = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    p_ref, s_ref = O.quantize_and_pack(w)
    packed, scales = quantize_and_pack_cuda(torch.from_numpy(w))
    np.testing.assert_array_equal(packed.cpu().numpy(), p_ref)
    np.testing.assert_array_equal(scales.cpu().view(torch.int16).numpy().view(np.uint16), s_ref)


def test_torch_cuda_scale_mode_matches_torch_on_cuda(cuda_device):
    # The same torch quantizer evaluated on a CUDA tensor divides by the host
    # scalar 7 as a reciprocal multiply; the flag reproduces those bits.
    from decode_kernel.quantize import quantize_and_pack, quantize_and_pack_cuda

    torch.manual_seed(1000)
    w = torch.randn(2048, 4096, device="cuda") * 0.05
    p_t, s_t = quantize_and_pack(w)
    p_k, s_k = quantize_and_pack_cuda(w, torch_cuda_scale=True)
    assert torch.equal(p_t, p_k) and torch.equal(s_t.view(torch.int16), s_k.view(torch.int16))


def test_stream_probes(cuda_device):
    from decode_kernel import _cuda

    n = 64 << 20
    src = torch.ones(n // 4, dtype=torch.float32, device="cuda")
    blocks = _cuda.stream_recommended_blocks()
    assert blocks == min(8192, max(1024, 32 * torch.cuda.get_device_properties(0).multi_processor_count))
    partials = torch.empty(blocks, dtype=torch.float32, device="cuda")
    _cuda.stream_read(src, partials)
    assert float(partials.double().sum()) == pytest.approx(n / 4, rel=1e-6)
    dst = torch.zeros_like(src)
    _cuda.stream_write(dst)
    assert bool((dst == 1.0).all())
    src2 = torch.randn(n // 4 + 4, device="cuda")
    dst2 = torch.empty_like(src2)
    _cuda.d2d_copy(src2, dst2)
    assert torch.equal(src2, dst2)

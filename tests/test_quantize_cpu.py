"""The package's format helpers on the CPU: bit-exact with the reference's
golden vectors, plus the reference's own CPU tests (tests/test_quantize.py)
restated against this package."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from decode_kernel.quantize import GROUP_SIZE, dequantize, quantize_and_pack, unpack_to_int

GQ = np.load(Path(__file__).resolve().parent / "golden" / "golden_quant.npz")
QCASES = sorted({k.split("/")[0] for k in GQ.files})


@pytest.mark.parametrize("case", QCASES)
def test_package_quantizer_matches_reference_bits(case):
    packed, scales = quantize_and_pack(torch.from_numpy(GQ[f"{case}/w"]))
    np.testing.assert_array_equal(packed.numpy(), GQ[f"{case}/packed"])
    np.testing.assert_array_equal(scales.view(torch.int16).numpy().view(np.uint16),
                                  GQ[f"{case}/scales"])
    np.testing.assert_array_equal(unpack_to_int(packed).numpy(), GQ[f"{case}/q"])
    if f"{case}/dequant" in GQ.files:
        np.testing.assert_array_equal(dequantize(packed, scales).numpy(), GQ[f"{case}/dequant"])


# --- tests/test_quantize.py of the reference, same shapes and seeds ---------

@pytest.mark.parametrize("shape", [(8, 128), (16, 256), (32, 512)])
def test_pack_unpack_q_roundtrip(shape):
    torch.manual_seed(0)
    w = torch.randn(*shape)
    packed, scales = quantize_and_pack(w)
    q = unpack_to_int(packed)
    assert int(q.min()) >= -7 and int(q.max()) <= 7
    recon = dequantize(packed, scales)
    scale = scales.float().repeat_interleave(GROUP_SIZE, dim=1)
    assert torch.allclose(recon, q.float() * scale, atol=1e-6)


@pytest.mark.parametrize("shape", [(8, 128), (16, 256)])
def test_reconstruction_within_half_step(shape):
    torch.manual_seed(0)
    w = torch.randn(*shape)
    packed, scales = quantize_and_pack(w)
    recon = dequantize(packed, scales)
    scale = scales.float().repeat_interleave(GROUP_SIZE, dim=1)
    assert torch.all((recon - w.float()).abs() <= 0.5 * scale + 1e-3)


def test_pack_layout_low_nibble_first():
    w = torch.zeros(1, 128)
    w[0, 0] = 7.0
    w[0, 1] = -7.0
    packed, scales = quantize_and_pack(w)
    word = int(packed[0, 0].item()) & 0xFFFFFFFF
    assert word & 0xF == 7
    assert (word >> 4) & 0xF == 9
    assert scales.shape == (1, 1)
    assert abs(float(scales[0, 0]) - 1.0) < 1e-3


def test_zero_group_does_not_nan():
    packed, scales = quantize_and_pack(torch.zeros(2, 128))
    assert torch.isfinite(dequantize(packed, scales)).all()
    assert torch.isfinite(scales.float()).all()


# --- format edges ------------------------------------------------------------

def test_minus_eight_decodes():
    # The quantizer never emits -8 but the format (and every kernel) decodes it.
    packed = torch.tensor([[0x88888888 - (1 << 32)] * 16], dtype=torch.int32)
    assert (unpack_to_int(packed) == -8).all()


def test_top_nibble_sign_bit_round_trips():
    w = torch.zeros(1, 128)
    w[0, 7] = -7.0  # nibble 7 lives in the word's sign bit
    w[0, 0] = 7.0
    packed, _ = quantize_and_pack(w)
    assert int(packed[0, 0]) < 0
    assert unpack_to_int(packed)[0, 7].item() == -7


@pytest.mark.parametrize("bad", [(2, 100), (3,)])
def test_shape_errors(bad):
    with pytest.raises(ValueError):
        quantize_and_pack(torch.zeros(*bad))


def test_agrees_with_oracle_on_baseline_distribution():
    from oracle import oracle as O

    rng = np.random.default_rng(5)
    w = (rng.standard_normal((96, 4096), dtype=np.float32) * np.float32(0.02))
    p_ref, s_ref = O.quantize_and_pack(w)
    packed, scales = quantize_and_pack(torch.from_numpy(w))
    np.testing.assert_array_equal(packed.numpy(), p_ref)
    np.testing.assert_array_equal(scales.view(torch.int16).numpy().view(np.uint16), s_ref)

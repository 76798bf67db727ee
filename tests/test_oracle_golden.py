"""Pin the oracle to the reference: every golden vector the reference itself
produced (tests/golden/make_golden.py) must be reproduced -- the quantizer bit
for bit, the fp32 linear within 1e-4."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"
GQ = np.load(GOLDEN / "golden_quant.npz")
GL = np.load(GOLDEN / "golden_linear.npz")
QCASES = sorted({k.split("/")[0] for k in GQ.files})
LCASES = sorted({k.split("/")[0] for k in GL.files})


def test_golden_cases_present():
    assert "kat_low_nibble_first" in QCASES and "zero_groups" in QCASES
    assert len(QCASES) >= 10 and len(LCASES) >= 6


@pytest.mark.parametrize("case", QCASES)
def test_c_quantizer_bit_exact(case):
    packed, scales = O.quantize_and_pack(GQ[f"{case}/w"])
    np.testing.assert_array_equal(packed, GQ[f"{case}/packed"])
    np.testing.assert_array_equal(scales, GQ[f"{case}/scales"])


@pytest.mark.parametrize("case", QCASES)
def test_numpy_quantizer_bit_exact(case):
    packed, scales = O.quantize_and_pack_np(GQ[f"{case}/w"])
    np.testing.assert_array_equal(packed, GQ[f"{case}/packed"])
    np.testing.assert_array_equal(scales, GQ[f"{case}/scales"])


@pytest.mark.parametrize("case", QCASES)
def test_unpack_and_dequantize(case):
    packed, scales = GQ[f"{case}/packed"], GQ[f"{case}/scales"]
    np.testing.assert_array_equal(O.unpack_to_int(packed), GQ[f"{case}/q"])
    np.testing.assert_array_equal(O.unpack_to_int_np(packed), GQ[f"{case}/q"])
    if f"{case}/dequant" in GQ.files:
        ref = GQ[f"{case}/dequant"]
        np.testing.assert_array_equal(O.dequantize(packed, scales), ref)
        np.testing.assert_array_equal(O.dequantize_np(packed, scales), ref)


@pytest.mark.parametrize("case", LCASES)
def test_linear_matches_reference(case):
    x, packed, scales = GL[f"{case}/x"], GL[f"{case}/packed"], GL[f"{case}/scales"]
    ref = GL[f"{case}/y"]
    assert np.abs(O.linear_fp32(x, packed, scales) - ref).max() <= 1e-4
    assert np.abs(O.linear_fp32_np(x, packed, scales) - ref).max() <= 1e-4


def test_linear_row_sampling_matches_full():
    case = LCASES[0]
    x, packed, scales = GL[f"{case}/x"], GL[f"{case}/packed"], GL[f"{case}/scales"]
    full = O.linear_fp32(x, packed, scales)
    part = O.linear_fp32(x, packed, scales, rows=(5, 17))
    np.testing.assert_array_equal(part[:, 5:17], full[:, 5:17])
    assert np.isnan(part[:, :5]).all()


def test_kat_low_nibble_first():
    # test_quantize.py:41-53: w[0,0]=7, w[0,1]=-7 -> nibbles 7 and 9, scale 1.
    w = np.zeros((1, 128), np.float32)
    w[0, 0], w[0, 1] = 7.0, -7.0
    packed, scales = O.quantize_and_pack(w)
    word = int(packed[0, 0]) & 0xFFFFFFFF
    assert word & 0xF == 7 and (word >> 4) & 0xF == 9
    assert scales.shape == (1, 1) and O.f16_bits_to_f32(scales[0, 0]) == 1.0


def test_fp16_conversions_exhaustive():
    # Every binary16 value round-trips; random fp32 values round like numpy.
    bits = np.arange(1 << 16, dtype=np.uint32)
    lib = O.lib()
    vals = np.array([lib.dko_f16_to_f32(int(b)) for b in bits[::97]], np.float32)
    ref = bits[::97].astype(np.uint16).view(np.float16).astype(np.float32)
    np.testing.assert_array_equal(np.isnan(vals), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_array_equal(vals[ok], ref[ok])
    rng = np.random.default_rng(0)
    f = np.concatenate([rng.standard_normal(3000).astype(np.float32) * s
                        for s in (1e-7, 1e-5, 1e-3, 1.0, 1e3, 7e4)])
    with np.errstate(over="ignore"):
        want = f.astype(np.float16).view(np.uint16)
    got = np.array([lib.dko_f32_to_f16(float(v)) for v in f], np.uint16)
    np.testing.assert_array_equal(got, want)


def test_quantizer_rejects_bad_shapes():
    with pytest.raises(ValueError):
        O.quantize_and_pack(np.zeros((2, 100), np.float32))

"""GPTQ-format import/export (decode_kernel.gptq) on the CPU.

Pinned to vLLM's own GPTQ packing helpers through tests/golden/golden_gptq.npz
(made by tests/golden/make_gptq_golden.py): to_gptq must reproduce vLLM's
qweight/qzeros bit for bit, and from_gptq must turn them back into this
library's layout.  Round trips run over the reference quantizer's golden
outputs, and the rejected checkpoint kinds are checked.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from decode_kernel.gptq import from_gptq, to_gptq
from decode_kernel.quantize import dequantize, unpack_to_int

GOLDEN = Path(__file__).resolve().parent / "golden"
GG = np.load(GOLDEN / "golden_gptq.npz")
GCASES = sorted({k.split("/")[0] for k in GG.files})
GQ = np.load(GOLDEN / "golden_quant.npz")
QCASES = sorted({k.split("/")[0] for k in GQ.files})


def pack_library(q: np.ndarray) -> np.ndarray:
    """Signed q [M, K] in [-8, 7] -> int32 [M, K/8], nibble k % 8 at bit 4 (k % 8)."""
    nib = q.astype(np.int64) & 0xF
    words = np.zeros((q.shape[0], q.shape[1] // 8), dtype=np.int64)
    for i in range(8):
        words |= nib[:, i::8] << (4 * i)
    return words.astype(np.uint32).view(np.int32)


def golden(case: str):
    q = GG[f"{case}/q"]
    s = torch.from_numpy(GG[f"{case}/scales"].view(np.float16).copy())
    return q, s, torch.from_numpy(GG[f"{case}/qweight"]), torch.from_numpy(GG[f"{case}/qzeros"])


def gptq_dequant(qweight: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """w[k, n] = (u - 8) * scales[k // 128, n], straight from the GPTQ definition."""
    words, n = qweight.shape
    shifts = torch.arange(0, 32, 4, dtype=torch.int32)
    u = ((qweight.unsqueeze(1) >> shifts.view(1, 8, 1)) & 0xF).reshape(words * 8, n)
    return (u - 8).float() * scales.float().repeat_interleave(128, dim=0)


@pytest.mark.parametrize("case", GCASES)
def test_to_gptq_matches_vllm_packing(case):
    q, s, qweight, qzeros = golden(case)
    out = to_gptq(torch.from_numpy(pack_library(q)), s)
    assert torch.equal(out.qweight, qweight)
    assert torch.equal(out.qzeros, qzeros)
    assert torch.equal(out.scales, s.t())
    assert torch.equal(out.g_idx, torch.arange(q.shape[1], dtype=torch.int32) // 128)


@pytest.mark.parametrize("case", GCASES)
def test_from_gptq_gives_the_library_layout(case):
    q, s, qweight, qzeros = golden(case)
    g_idx = torch.arange(q.shape[1], dtype=torch.int32) // 128
    packed, scales = from_gptq(qweight, s.t().contiguous(), qzeros, g_idx)
    np.testing.assert_array_equal(packed.numpy(), pack_library(q))
    assert torch.equal(scales, s)
    np.testing.assert_array_equal(unpack_to_int(packed).numpy(), q.astype(np.int32))
    # Both layouts decode to the same matrix.
    assert torch.equal(dequantize(packed, scales).t(), gptq_dequant(qweight, s.t()))


@pytest.mark.parametrize("case", QCASES)
def test_round_trip_over_reference_quantizer_outputs(case):
    packed = torch.from_numpy(GQ[f"{case}/packed"])
    scales = torch.from_numpy(GQ[f"{case}/scales"].view(np.float16).copy())
    g = to_gptq(packed, scales)
    back, s2 = from_gptq(g.qweight, g.scales, g.qzeros, g.g_idx)
    assert torch.equal(back, packed)
    assert torch.equal(s2, scales)
    assert torch.equal(dequantize(packed, scales).t(), gptq_dequant(g.qweight, g.scales))


def test_zeros_minus_one_serialisation():
    q, s, qweight, _ = golden("m24_k384")
    out = to_gptq(torch.from_numpy(pack_library(q)), s, zeros_minus_one=True)
    assert bool((out.qzeros == 0x77777777).all())
    packed, _ = from_gptq(out.qweight, out.scales, out.qzeros, zeros_minus_one=True)
    np.testing.assert_array_equal(packed.numpy(), pack_library(q))
    with pytest.raises(ValueError, match="zero points"):
        from_gptq(out.qweight, out.scales, out.qzeros)  # 7 read as the zero point itself


def test_rows_not_a_multiple_of_eight():
    rng = np.random.default_rng(5)
    q = rng.integers(-8, 8, size=(20, 256)).astype(np.int8)
    s = torch.rand(20, 2).half()
    g = to_gptq(torch.from_numpy(pack_library(q)), s)
    assert tuple(g.qzeros.shape) == (2, 3) and bool((g.qzeros == -0x77777778).all())
    packed, s2 = from_gptq(g.qweight, g.scales, g.qzeros, g.g_idx)
    np.testing.assert_array_equal(packed.numpy(), pack_library(q))
    assert torch.equal(s2, s)


def test_rejects_what_the_format_cannot_hold():
    q, s, qweight, qzeros = golden("m24_k384")
    st = s.t().contiguous()
    # group 64: six scale rows for K = 384
    with pytest.raises(ValueError, match="group size 64"):
        from_gptq(qweight, st.repeat_interleave(2, dim=0))
    # an asymmetric zero point in one column
    bad = qzeros.clone()
    bad[1, 0] = bad[1, 0] ^ 0x3
    with pytest.raises(ValueError, match="zero points"):
        from_gptq(qweight, st, bad)
    # act-order: g_idx permutes K
    g_idx = torch.arange(384, dtype=torch.int32) // 128
    with pytest.raises(ValueError, match="act-order"):
        from_gptq(qweight, st, qzeros, g_idx.flip(0))
    with pytest.raises(ValueError, match="g_idx"):
        from_gptq(qweight, st, qzeros, g_idx[:-1])
    # dtypes and shapes
    with pytest.raises(ValueError, match="qweight"):
        from_gptq(qweight.to(torch.int64), st)
    with pytest.raises(ValueError, match="scales"):
        from_gptq(qweight, st.float())
    with pytest.raises(ValueError, match="columns"):
        from_gptq(qweight, st[:, :-1])
    with pytest.raises(ValueError, match="qzeros"):
        from_gptq(qweight, st, qzeros[:, :-1])
    with pytest.raises(ValueError, match="packed"):
        to_gptq(torch.from_numpy(pack_library(q)).to(torch.int64), s)
    with pytest.raises(ValueError, match="scales"):
        to_gptq(torch.from_numpy(pack_library(q)), s[:, :-1])


def test_linear_module_from_gptq_checkpoint():
    from decode_kernel import W4A16Linear

    q, s, qweight, qzeros = golden("m40_k1024")
    g_idx = torch.arange(q.shape[1], dtype=torch.int32) // 128
    layer = W4A16Linear.from_gptq(qweight, s.t().contiguous(), qzeros, g_idx)
    assert (layer.out_features, layer.in_features) == q.shape
    np.testing.assert_array_equal(layer.packed.numpy(), pack_library(q))
    assert torch.equal(layer.scales, s)
    with pytest.raises(ValueError, match="zero points"):
        W4A16Linear.from_gptq(qweight, s.t().contiguous(), qzeros, zeros_minus_one=True)

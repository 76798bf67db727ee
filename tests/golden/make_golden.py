"""Generate golden vectors by running RohanDisa/decode-kernel's own Python code.

Run once, in a container where the reference checkout is present:

    DK_REFERENCE=/path/to/decode-kernel python tests/golden/make_golden.py

It imports the reference package (``python/decode_kernel``), feeds it seeded
inputs and writes ``tests/golden/golden_quant.npz`` and
``tests/golden/golden_linear.npz``.  The GPU box never runs this script and
never needs the reference: the committed .npz files are the fixtures.

Reference functions exercised:
  quantize_and_pack  python/decode_kernel/quantize.py:26-51
  unpack_to_int      python/decode_kernel/quantize.py:54-63
  dequantize         python/decode_kernel/quantize.py:66-78
  linear_fp32        python/decode_kernel/reference.py:17-26

Every case is on CPU, as the reference's CPU tests and BASELINE inputs are.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def _load_reference():
    root = os.environ.get("DK_REFERENCE")
    if not root:
        raise SystemExit("set DK_REFERENCE to the decode-kernel checkout")
    sys.path.insert(0, str(Path(root) / "python"))
    os.environ.setdefault("DK_SKIP_CUDA", "1")
    from decode_kernel.quantize import dequantize, quantize_and_pack, unpack_to_int
    from decode_kernel.reference import linear_fp32

    return quantize_and_pack, unpack_to_int, dequantize, linear_fp32


def quant_cases(torch):
    """(name, W fp32) pairs.  Shapes and seeds of tests/test_quantize.py plus
    the edge cases the format has: zero groups, exact .5 ties, fp16 scale
    underflow / subnormal / overflow, a group count that is not a power of 2,
    and the BASELINE weight distribution N(0, 0.02)."""
    cases = []
    for shape in [(8, 128), (16, 256), (32, 512)]:  # test_quantize.py:16-25
        torch.manual_seed(0)
        cases.append((f"randn_seed0_{shape[0]}x{shape[1]}", torch.randn(*shape)))
    w = torch.zeros(1, 128)  # test_quantize.py:41-53
    w[0, 0] = 7.0
    w[0, 1] = -7.0
    cases.append(("kat_low_nibble_first", w))
    cases.append(("zero_groups", torch.zeros(2, 128)))  # test_quantize.py:56-61
    # amax = 7 -> scale = 1, so w/scale hits the .5 ties exactly.
    t = torch.zeros(2, 128)
    t[:, 0] = 7.0
    ties = torch.tensor([0.5, 1.5, 2.5, 3.5, 4.5, 5.5, 6.5, -0.5, -1.5, -2.5, -3.5,
                         -4.5, -5.5, -6.5, 7.5, -7.5])
    t[0, 1:17] = ties
    t[1, 1:17] = -ties
    cases.append(("round_half_even_ties", t))
    g = torch.Generator().manual_seed(7)
    mixed = torch.randn(4, 512, generator=g) * 0.02
    mixed[0, 128:256] = 0.0                       # a zero group inside a row
    mixed[1, 0:128] *= 1e-4                       # fp16 subnormal scale
    mixed[1, 128:256] *= 1e-7                     # scale clamps to 1e-8 -> fp16 0
    mixed[2, 256:384] *= 1e6                      # scale overflows fp16 -> inf
    mixed[3, :] = torch.randn(512, generator=g) * 3000.0  # large, finite scales
    cases.append(("scale_edges", mixed))
    g = torch.Generator().manual_seed(11)
    cases.append(("baseline_dist_64x1024", torch.randn(64, 1024, generator=g) * 0.02))
    g = torch.Generator().manual_seed(12)
    cases.append(("ref_test_dist_48x384", torch.randn(48, 384, generator=g) * 0.05))
    g = torch.Generator().manual_seed(13)
    cases.append(("k11008_3rows", torch.randn(3, 11008, generator=g) * 0.02))
    return cases


def linear_cases(torch):
    """(name, M, K, B, weight std, seed) -- small enough for the scalar C
    oracle to finish in well under a second each."""
    return [
        ("m64_k256_b1", 64, 256, 1, 0.05, 1000),
        ("m33_k384_b3", 33, 384, 3, 0.05, 1001),
        ("m128_k1024_b8", 128, 1024, 8, 0.02, 1002),
        ("m16_k11008_b1", 16, 11008, 1, 0.02, 1003),
        ("m40_k4096_b32", 40, 4096, 32, 0.02, 1004),
        ("m8_k8192_b2", 8, 8192, 2, 0.02, 1005),
    ]


def main():
    import torch

    torch.set_num_threads(1)
    quantize_and_pack, unpack_to_int, dequantize, linear_fp32 = _load_reference()

    q_out = {}
    for name, w in quant_cases(torch):
        w = w.float().contiguous()
        packed, scales = quantize_and_pack(w)
        q_out[f"{name}/w"] = w.numpy()
        q_out[f"{name}/packed"] = packed.numpy()
        q_out[f"{name}/scales"] = scales.view(torch.int16).numpy().view(np.uint16)
        q_out[f"{name}/q"] = unpack_to_int(packed).numpy().astype(np.int8)
        if w.numel() <= 1 << 15:  # larger cases are covered through packed/scales
            q_out[f"{name}/dequant"] = dequantize(packed, scales).numpy()
    np.savez_compressed(OUT / "golden_quant.npz", **q_out)

    l_out = {}
    for name, m, k, b, std, seed in linear_cases(torch):
        g = torch.Generator().manual_seed(seed)
        w = torch.randn(m, k, generator=g) * std
        x = torch.randn(b, k, generator=g).half()
        packed, scales = quantize_and_pack(w)
        y = linear_fp32(x, packed, scales)
        l_out[f"{name}/packed"] = packed.numpy()
        l_out[f"{name}/scales"] = scales.view(torch.int16).numpy().view(np.uint16)
        l_out[f"{name}/x"] = x.view(torch.int16).numpy().view(np.uint16)
        l_out[f"{name}/y"] = y.numpy()
    np.savez_compressed(OUT / "golden_linear.npz", **l_out)
    for f in ("golden_quant.npz", "golden_linear.npz"):
        print(f, (OUT / f).stat().st_size, "bytes")


if __name__ == "__main__":
    main()

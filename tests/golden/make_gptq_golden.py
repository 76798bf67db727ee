"""Generate the GPTQ-layout golden vectors with vLLM's own packing code.

Run once, in a container where vLLM is installed:

    python tests/golden/make_gptq_golden.py

It packs seeded signed int4 values with vLLM's reference helpers
(``vllm.model_executor.layers.quantization.utils.quant_utils``: ``gptq_pack``
for ``qweight``, packing along K; ``pack_cols`` for ``qzeros``, packing along
N) in the symmetric "uint4b8" convention (stored value q + 8, zero point 8),
and writes ``tests/golden/golden_gptq.npz``.  The tests read only the .npz, so
neither the GPU box nor the CPU suite needs vLLM.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent / "golden_gptq.npz"


def cases():
    """(name, q int8 [M, K] in [-8, 7], scales fp16 [M, K/128])."""
    out = []
    for name, (m, k, seed) in {"m24_k384": (24, 384, 11), "m16_k128": (16, 128, 12),
                               "m40_k1024": (40, 1024, 13)}.items():
        rng = np.random.default_rng(seed)
        q = rng.integers(-8, 8, size=(m, k)).astype(np.int8)
        s = (rng.random((m, k // 128)) * 0.05 + 1e-3).astype(np.float16)
        out.append((name, q, s))
    # Every 4-bit value at every nibble position of a word.
    q = np.array([[((r + i) % 16) - 8 for i in range(128)] for r in range(8)], dtype=np.int8)
    out.append(("kat_all_nibbles", q, np.ones((8, 1), dtype=np.float16)))
    return out


def main() -> None:
    import torch
    from vllm.model_executor.layers.quantization.utils.quant_utils import gptq_pack, pack_cols

    arrays = {}
    for name, q, s in cases():
        m, k = q.shape
        u = torch.from_numpy((q.astype(np.int32) + 8).T.copy())  # [K, N], uint4b8
        qweight = gptq_pack(u, 4, k, m).numpy()
        zeros = torch.full((k // 128, m), 8, dtype=torch.int32)
        qzeros = pack_cols(zeros, 4, k // 128, m).numpy()
        arrays[f"{name}/q"] = q
        arrays[f"{name}/scales"] = s.view(np.uint16)
        arrays[f"{name}/qweight"] = qweight.astype(np.int32)
        arrays[f"{name}/qzeros"] = qzeros.astype(np.int32)
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({len(arrays)} arrays)")


if __name__ == "__main__":
    main()

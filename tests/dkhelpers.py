"""Helpers shared by the tests: seeded problems, the oracle comparison, and
calls through the C ABI with torch-owned device memory."""

from __future__ import annotations

import numpy as np

from oracle import oracle as O

MAX_ABS = 1e-2  # north-star / reference tolerance (test_correctness.py:29)


def make_problem(M: int, K: int, B: int, seed: int, std: float = 0.02):
    """Seeded W ~ N(0, std) [M, K] fp32 and x ~ N(0, 1) fp16 [B, K]; W is
    quantized by the oracle (bit-exact with the reference's quantizer)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((M, K), dtype=np.float32) * np.float32(std)).astype(np.float32)
    x = rng.standard_normal((B, K), dtype=np.float32).astype(np.float16)
    packed, scales = O.quantize_and_pack(w)
    return packed, scales, x


def oracle_y(x, packed, scales, rows=None) -> np.ndarray:
    """fp32 oracle; the scalar C path for small problems and sampled rows,
    the numpy (BLAS) restatement for large ones."""
    m, words = packed.shape
    k = words * 8
    if rows is None and m * k * x.shape[0] > 64 * 1024 * 1024:
        return O.linear_fp32_np(x, packed, scales)
    return O.linear_fp32(x, packed, scales, rows=rows)


def to_device(packed, scales, x):
    import torch

    dev = torch.device("cuda", 0)
    tp = torch.from_numpy(np.ascontiguousarray(packed)).to(dev)
    ts = torch.from_numpy(np.ascontiguousarray(scales).view(np.int16)).to(dev).view(torch.float16)
    tx = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev).view(torch.float16)
    return tp, ts, tx


def capi_gemv(tp, ts, tx, cfg=None, y=None, poison=True):
    """Run dk_w4a16_gemv through ctypes; returns y (fp16 CUDA tensor [B, M])."""
    import torch
    from decode_kernel import capi

    M = tp.shape[0]
    K = tp.shape[1] * 8
    B = tx.shape[0]
    if y is None:
        y = torch.empty((B, M), dtype=torch.float16, device=tp.device)
        if poison:
            y.fill_(float("nan"))  # rows a kernel fails to write stay NaN
    ws_bytes = capi.workspace_bytes(M, K, B, cfg)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=tp.device)
    stream = torch.cuda.current_stream().cuda_stream
    st = capi.gemv(tp.data_ptr(), ts.data_ptr(), tx.data_ptr(), y.data_ptr(), M, K, B, cfg,
                   ws.data_ptr() if ws_bytes else 0, ws_bytes, stream)
    capi.check(st, "dk_w4a16_gemv")
    return y


def max_err(y_dev, y_ref, rows=None) -> float:
    y = y_dev.float().cpu().numpy()
    if rows is not None:
        y = y[:, rows[0]:rows[1]]
        y_ref = y_ref[:, rows[0]:rows[1]]
    assert np.isfinite(y).all(), "kernel left NaN/inf in the output"
    return float(np.abs(y - y_ref).max()) if y.size else 0.0

"""dk_w4a16_gemv_splitk_noalloc: the split-K GEMV for callers that cannot
allocate device memory where they call it (an allocator callback, a runtime
that owns every buffer, a decode path that must not touch the allocator).

It runs the same split-K kernel as dk_w4a16_gemv(version=4) but keeps its
scratch in a fixed buffer inside the library, so the caller passes only the
inputs and the output.  The GPU test compares it with the ordinary entry point
(which takes a caller workspace) on two calls in a row through the C ABI; the
buffer is shared by every call, so the second call also shows that whatever
the first one left behind does not leak into the result.

This file is named to be collected last.  The GPU test works alone in a fresh
process (it makes the first call on the device, which looks up the buffer's
address) and after all other tests.
"""

from __future__ import annotations

import numpy as np
import pytest

from dkhelpers import MAX_ABS, capi_gemv, make_problem, max_err, oracle_y, to_device


def _noalloc(tp, ts, tx, y, split):
    import torch
    from decode_kernel import capi

    M, K, B = tp.shape[0], tp.shape[1] * 8, tx.shape[0]
    return capi.load().dk_w4a16_gemv_splitk_noalloc(
        tp.data_ptr(), ts.data_ptr(), tx.data_ptr(), y.data_ptr(), M, K, B, split,
        torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_before_touching_the_device():
    from decode_kernel import capi

    lib = capi.load()
    # split_k outside [1, 32], bad K: rejected from the arguments alone.
    assert lib.dk_w4a16_gemv_splitk_noalloc(16, 16, 16, 16, 64, 256, 1, 0, None) == \
        capi.DK_ERR_INVALID_ARG
    assert lib.dk_w4a16_gemv_splitk_noalloc(16, 16, 16, 16, 64, 200, 1, 4, None) == \
        capi.DK_ERR_INVALID_ARG
    # A problem whose split-K scratch exceeds the fixed buffer is refused.
    M, K = 65536, 8192
    need = capi.workspace_bytes(M, K, 1, capi.default_config(version=4, split_k=4))
    assert need > capi.DK_NOALLOC_SCRATCH_BYTES
    assert lib.dk_w4a16_gemv_splitk_noalloc(16, 16, 16, 16, M, K, 1, 4, None) == \
        capi.DK_ERR_WORKSPACE


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice(cuda_device):
    import torch
    from decode_kernel import capi

    M, K, split = 1000, 4096, 4
    for call, (B, seed) in enumerate([(3, 501), (1, 502)]):
        packed, scales, x = make_problem(M, K, B, seed=seed)
        tp, ts, tx = to_device(packed, scales, x)
        want = capi_gemv(tp, ts, tx, capi.default_config(version=4, split_k=split))
        got = torch.full((B, M), float("nan"), dtype=torch.float16, device=cuda_device)
        capi.check(_noalloc(tp, ts, tx, got, split), f"noalloc call {call}")
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert max_err(got, want.float().cpu().numpy()) < MAX_ABS
        assert torch.equal(got, want)  # same kernel, same reduction order
        assert max_err(got, oracle_y(x, packed, scales)) < MAX_ABS
    assert capi.load().dk_device_error(-1, 0) == 0


# (M, K, B, split): batches that run in one pass (B = 1) and in several 8-row
# passes that reuse the shared buffer on one stream (B = 9, 17); a problem
# whose scratch (counters + 8 rows of per-group partials) reaches to within
# 15 KB of the buffer's end; K = 128, where the split clamps to 1 and no
# scratch is used at all.
NOALLOC_CASES = [(1000, 4096, 1, 4), (1000, 4096, 9, 4), (600, 2048, 17, 8),
                 (8176, 4096, 9, 4), (300, 128, 17, 4)]


@pytest.mark.gpu
@pytest.mark.parametrize("M,K,B,split", NOALLOC_CASES)
def test_noalloc_batches_and_limits(M, K, B, split, cuda_device):
    import torch
    from decode_kernel import capi

    cfg4 = capi.default_config(version=4, split_k=split)
    need = capi.workspace_bytes(M, K, B, cfg4)
    assert need <= capi.DK_NOALLOC_SCRATCH_BYTES
    if K == 128:
        assert need == 0
    packed, scales, x = make_problem(M, K, B, seed=M + K + B)
    tp, ts, tx = to_device(packed, scales, x)
    want = capi_gemv(tp, ts, tx, cfg4)
    for call in range(2):
        got = torch.full((B, M), float("nan"), dtype=torch.float16, device=cuda_device)
        capi.check(_noalloc(tp, ts, tx, got, split), f"noalloc call {call}")
        torch.cuda.synchronize()
        assert torch.equal(got, want), call
    assert max_err(got, oracle_y(x, packed, scales)) < MAX_ABS
    assert capi.load().dk_device_error(-1, 0) == 0

"""This library against the reference's own CUDA kernels, on the same GPU and
the same device buffers.

The reference's csrc/gemv_w4a16.cu is compiled unmodified for sm_100a from
its checkout (oracle/Makefile ``ref``) and called through oracle/ref_cuda.py.
For every kernel version the reference dispatches (v0..v5, split-K, the
warps-per-row variants of v1, the batch weight-reuse path; gemv_w4a16.cu:
427-591) both libraries run the same configuration on identical inputs:

* each output is within the north-star tolerance (max-abs < 1e-2,
  test_correctness.py:29) of the fp32 oracle, and the two outputs are within
  that tolerance of each other;
* both write the same dispatch stamp (gemv_w4a16.cu:18-25, 553-564).

The two are not bit-identical: the reference sums in a per-lane fp32 order
with warp shuffles (and fp32 atomics for split-K), this library in its own
canonical order, both then round to fp16.
"""

from __future__ import annotations

import numpy as np
import pytest

from dkhelpers import MAX_ABS, capi_gemv, make_problem, max_err, oracle_y, to_device

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    from oracle import ref_cuda

    if not ref_cuda.available():
        pytest.skip("oracle/_ref/libdkref.so not built (no reference checkout at build time)")
    return ref_cuda


def _pair(ref, tp, ts, tx, **cfg):
    """Run the reference kernel and this library with one configuration;
    return (ours, theirs, our stamp, their stamp)."""
    import torch
    from decode_kernel import capi

    B, M = tx.shape[0], tp.shape[0]
    theirs = torch.full((B, M), float("nan"), dtype=torch.float16, device=tp.device)
    ws = None
    if cfg.get("version", 5) == 4 and not cfg.get("reuse_weights", False):
        ws = torch.zeros((B, M), dtype=torch.float32, device=tp.device)
    assert ref.gemv(tp, ts, tx, theirs, workspace=ws, **cfg) == 0
    their_stamp = ref.lib().dkref_last_kernel_stamp()  # synchronizes
    ours = capi_gemv(tp, ts, tx, capi.default_config(**{k: int(v) for k, v in cfg.items()}))
    torch.cuda.synchronize()
    our_stamp = capi.load().dk_last_kernel_stamp(-1)
    return ours, theirs, our_stamp, their_stamp


CONFIGS = [dict(version=v, split_k=4 if v == 4 else 1) for v in range(6)] + [
    dict(version=4, split_k=16),
    dict(version=1, warps_per_row=2),
    dict(version=1, warps_per_row=4),
    dict(version=5, reuse_weights=True),
]


def _cfg_id(c):
    return "-".join(f"{k}{int(v)}" for k, v in c.items())


@pytest.mark.parametrize("cfg", CONFIGS, ids=_cfg_id)
@pytest.mark.parametrize("shape", [(256, 256), (4096, 4096)])
@pytest.mark.parametrize("batch", [1, 4])
def test_every_reference_kernel_agrees(ref, cfg, shape, batch, cuda_device):
    M, K = shape
    packed, scales, x = make_problem(M, K, batch, seed=7000 + M + batch, std=0.05)
    tp, ts, tx = to_device(packed, scales, x)
    ours, theirs, s_ours, s_theirs = _pair(ref, tp, ts, tx, **cfg)
    want = oracle_y(x, packed, scales)
    assert max_err(ours, want) < MAX_ABS
    assert max_err(theirs, want) < MAX_ABS
    assert max_err(ours, theirs.float().cpu().numpy()) < MAX_ABS
    assert s_ours == s_theirs, f"stamp {s_ours} vs the reference's {s_theirs}"


@pytest.mark.parametrize("shape", [(11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("version", [1, 5])
def test_baseline_shapes_agree(ref, shape, version, cuda_device):
    """The BASELINE 7B MLP shapes at B=1 with the reference's best (v1) and
    default (v5) kernels, weights N(0, 0.02) as in the benchmark."""
    M, K = shape
    packed, scales, x = make_problem(M, K, 1, seed=7100 + version)
    tp, ts, tx = to_device(packed, scales, x)
    ours, theirs, s_ours, s_theirs = _pair(ref, tp, ts, tx, version=version)
    want = oracle_y(x, packed, scales)
    assert max_err(ours, want) < MAX_ABS
    assert max_err(theirs, want) < MAX_ABS
    assert s_ours == s_theirs


def test_reuse_batch_sweep_agrees(ref, cuda_device):
    """The reference's batch path (weight reuse) over its sweep's batches at
    4096^2 (bench.py --sweep of the reference: B in 1..32)."""
    packed, scales, _ = make_problem(4096, 4096, 1, seed=7200)
    rng = np.random.default_rng(7201)
    for B in (2, 8, 16, 32):
        x = rng.standard_normal((B, 4096), dtype=np.float32).astype(np.float16)
        tp, ts, tx = to_device(packed, scales, x)
        ours, theirs, s_ours, s_theirs = _pair(ref, tp, ts, tx, version=5, reuse_weights=True)
        want = oracle_y(x, packed, scales)
        assert max_err(ours, want) < MAX_ABS, B
        assert max_err(theirs, want) < MAX_ABS, B
        assert s_ours == s_theirs == 15

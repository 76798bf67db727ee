"""GPU parity of every GEMV kernel, called through the C ABI (dk_w4a16_gemv),
against the CPU oracle: max-abs < 1e-2, plus the
bit-level properties the kernel family guarantees (one canonical reduction
order for v2/v3/v4/v5/reuse up to 8 batch rows, batch- and row-invariance
within each kernel; 17..32 rows on large matrices run on the tensor-core
batch kernel)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from dkhelpers import MAX_ABS, capi_gemv, make_problem, max_err, oracle_y, to_device

pytestmark = pytest.mark.gpu


def cfg(**kw):
    from decode_kernel import capi

    return capi.default_config(**kw)


def stamp():
    from decode_kernel import capi

    return capi.load().dk_last_kernel_stamp(-1)


SHAPES = [(256, 256), (64, 128), (48, 384), (33, 1024), (1, 128), (17, 4096), (300, 640),
          (1000, 2048), (4096, 4096)]


@pytest.mark.parametrize("version", [0, 1, 2, 3, 4, 5])
@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("batch", [1, 4])
def test_versions_vs_oracle(version, shape, batch, cuda_device):
    M, K = shape
    packed, scales, x = make_problem(M, K, batch, seed=1000 + M + K + batch, std=0.05)
    ref = oracle_y(x, packed, scales)
    tp, ts, tx = to_device(packed, scales, x)
    y = capi_gemv(tp, ts, tx, cfg(version=version, split_k=4))
    assert max_err(y, ref) < MAX_ABS
    assert stamp() == version


@pytest.mark.parametrize("batch", [1, 2, 3, 7, 8, 9, 16, 17, 31, 32, 33, 40, 64])
@pytest.mark.parametrize("reuse", [0, 1])
def test_batch_path_vs_oracle(batch, reuse, cuda_device):
    M, K = 200, 1536
    packed, scales, x = make_problem(M, K, batch, seed=77 + batch)
    ref = oracle_y(x, packed, scales)
    tp, ts, tx = to_device(packed, scales, x)
    y = capi_gemv(tp, ts, tx, cfg(version=5, reuse_weights=reuse))
    assert max_err(y, ref) < MAX_ABS
    assert stamp() == (15 if reuse else 5)


@pytest.mark.parametrize("split", [1, 2, 3, 4, 7, 8, 32])
@pytest.mark.parametrize("batch", [1, 5, 9])
def test_split_k_vs_oracle_and_bitwise_v3(split, batch, cuda_device):
    M, K = 300, 4096
    packed, scales, x = make_problem(M, K, batch, seed=5 * split + batch)
    ref = oracle_y(x, packed, scales)
    tp, ts, tx = to_device(packed, scales, x)
    y4 = capi_gemv(tp, ts, tx, cfg(version=4, split_k=split))
    assert stamp() == 4
    y3 = capi_gemv(tp, ts, tx, cfg(version=3))
    assert max_err(y4, ref) < MAX_ABS
    assert torch.equal(y4, y3), "split-K must replay the canonical reduction order"


@pytest.mark.parametrize("wpr", [1, 2, 3, 4, 8])
def test_warps_per_row(wpr, cuda_device):
    M, K = 256, 1024
    packed, scales, x = make_problem(M, K, 3, seed=3)
    ref = oracle_y(x, packed, scales)
    tp, ts, tx = to_device(packed, scales, x)
    y = capi_gemv(tp, ts, tx, cfg(version=1, warps_per_row=wpr))
    assert max_err(y, ref) < MAX_ABS
    assert stamp() == (1 if wpr == 1 else 10 + wpr)


def test_stamp_resets_when_a_call_launches_nothing(cuda_device):
    # The reference clears the stamp before every launch (gemv_w4a16.cu:553-557),
    # so after a call that ran no kernel last_kernel_stamp is -1, not the
    # stamp of the kernel before it.
    from decode_kernel import capi

    lib = capi.load()
    packed, scales, x = make_problem(64, 256, 1, seed=4)
    tp, ts, tx = to_device(packed, scales, x)
    capi_gemv(tp, ts, tx, cfg(version=3))
    assert stamp() == 3
    y = torch.empty(1, 64, dtype=torch.float16, device=cuda_device)
    bad = cfg(version=3)
    st = capi.gemv(tp.data_ptr(), ts.data_ptr(), tx.data_ptr() + 2, y.data_ptr(), 64, 256, 1, bad,
                   0, 0, torch.cuda.current_stream().cuda_stream)  # misaligned x: rejected
    assert st == capi.DK_ERR_INVALID_ARG
    assert stamp() == -1
    capi_gemv(tp, ts, tx, cfg(version=2))
    assert stamp() == 2
    st = capi.gemv(tp.data_ptr(), ts.data_ptr(), tx.data_ptr(), y.data_ptr(), 0, 256, 1, bad, 0,
                   0, torch.cuda.current_stream().cuda_stream)  # M = 0: nothing to launch
    assert st == capi.DK_OK
    assert stamp() == -1
    assert lib.dk_last_kernel_stamp(-1) == -1


def test_tensor_core_family_is_bitwise_identical(cuda_device):
    M, K, B = 777, 11008, 5
    packed, scales, x = make_problem(M, K, B, seed=11)
    tp, ts, tx = to_device(packed, scales, x)
    outs = [capi_gemv(tp, ts, tx, cfg(version=v, split_k=4)) for v in (2, 3, 4, 5)]
    outs.append(capi_gemv(tp, ts, tx, cfg(version=5, reuse_weights=1)))
    for y in outs[1:]:
        assert torch.equal(y, outs[0])


@pytest.mark.parametrize("batch", [1, 3, 8])
def test_uneven_tile_ranges_match_the_family(batch, cuda_device):
    # 9477 x 8192: 593 tiles over 148 CTAs, 4 or 5 each (the 16-warp streaming
    # kernel, two 4096-k chunks per tile); the rows past M fill half of the
    # matrix's last tile.  Bitwise the v3 kernel's outputs, and within the
    # tolerance of the oracle.
    M, K = 9477, 8192
    packed, scales, x = make_problem(M, K, batch, seed=31 + batch)
    tp, ts, tx = to_device(packed, scales, x)
    y5 = capi_gemv(tp, ts, tx, cfg())
    y3 = capi_gemv(tp, ts, tx, cfg(version=3))
    assert torch.equal(y5, y3)
    rows = (M - 300, M)
    assert max_err(y5, oracle_y(x, packed, scales, rows=rows), rows=rows) < MAX_ABS


def test_batch_rows_are_independent(cuda_device):
    # y[b] must not depend on which other rows share the call (bitwise), for
    # each kernel path: 1..8 rows, 9..16 rows and 17..32 rows each run on one
    # kernel; B = 33 is a pass of 32 plus a pass of 1.
    M, K, B = 512, 4096, 33
    packed, scales, x = make_problem(M, K, B, seed=21)
    tp, ts, tx = to_device(packed, scales, x)
    full = capi_gemv(tp, ts, tx, cfg())
    for b in (0, 7, 8, 31):
        # the same row at another position among 8 others (a B = 9 call)
        idx = [(b + 5 + i) % 32 for i in range(4)] + [b] + [(b + 11 + i) % 32 for i in range(4)]
        part = capi_gemv(tp, ts, tx[idx].contiguous(), cfg())
        assert torch.equal(part[4], full[b]), b
    one = capi_gemv(tp, ts, tx[32:33].contiguous(), cfg())
    assert torch.equal(one[0], full[32])
    five = capi_gemv(tp, ts, tx[:5].contiguous(), cfg())
    for b in range(5):
        assert torch.equal(capi_gemv(tp, ts, tx[b:b + 1].contiguous(), cfg())[0], five[b])


def test_row_slices_are_independent(cuda_device):
    # A row shard of W gives exactly the matching slice of y (the property the
    # row-parallel multi-GPU path relies on).
    M, K, B = 4096, 4096, 2
    packed, scales, x = make_problem(M, K, B, seed=22)
    tp, ts, tx = to_device(packed, scales, x)
    full = capi_gemv(tp, ts, tx, cfg())
    for a, b in ((0, 512), (512, 1024), (1000, 1377), (4095, 4096)):
        part = capi_gemv(tp[a:b].contiguous(), ts[a:b].contiguous(), tx, cfg())
        assert torch.equal(part, full[:, a:b])


def test_minus_eight_nibbles(cuda_device):
    # The quantizer never emits -8, but the format decodes it.
    M, K = 32, 256
    packed = np.full((M, K // 8), np.int32(-0x77777778), np.int32)  # 0x88888888
    scales = np.full((M, K // 128), np.float16(0.5)).view(np.uint16)
    x = np.random.default_rng(0).standard_normal((2, K)).astype(np.float16)
    ref = oracle_y(x, packed, scales)
    tp, ts, tx = to_device(packed, scales, x)
    for v in range(6):
        assert max_err(capi_gemv(tp, ts, tx, cfg(version=v)), ref) < MAX_ABS


def test_k_zero_writes_zeros(cuda_device):
    from decode_kernel import capi

    y = torch.full((3, 64), 7.0, dtype=torch.float16, device="cuda")
    st = capi.gemv(16, 16, 16, y.data_ptr(), 64, 0, 3, cfg())
    assert st == capi.DK_OK
    torch.cuda.synchronize()
    assert (y == 0).all()


def test_workspace_too_small_is_reported(cuda_device):
    from decode_kernel import capi

    packed, scales, x = make_problem(64, 1024, 1, seed=1)
    tp, ts, tx = to_device(packed, scales, x)
    y = torch.empty((1, 64), dtype=torch.float16, device="cuda")
    c = cfg(version=4, split_k=4)
    need = capi.workspace_bytes(64, 1024, 1, c)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    st = capi.gemv(tp.data_ptr(), ts.data_ptr(), tx.data_ptr(), y.data_ptr(), 64, 1024, 1, c,
                   ws.data_ptr(), need - 4, 0)
    assert st == capi.DK_ERR_WORKSPACE


def test_pdl_chain_matches_plain(cuda_device):
    # Back-to-back launches with programmatic dependent launch: each GEMV's
    # output feeds the next GEMV's x, so the dependency wait must hold.
    from decode_kernel import capi

    K = 1024
    layers = [make_problem(K, K, 1, seed=40 + i, std=0.03) for i in range(6)]
    dev = [to_device(p, s, x) for p, s, x in layers]
    x0 = dev[0][2]
    outs = {}
    for flags in (0, capi.DK_FLAG_PDL):
        h = x0
        for tp, ts, _ in dev:
            h = capi_gemv(tp, ts, h, cfg(flags=flags), poison=False)
        torch.cuda.synchronize()
        outs[flags] = h
    assert torch.equal(outs[0], outs[capi.DK_FLAG_PDL])
    assert capi.load().dk_device_error(-1, 1) == 0


@pytest.mark.slow
@pytest.mark.parametrize("shape", [(4096, 4096), (11008, 4096), (4096, 11008)])
@pytest.mark.parametrize("batch", [1, 8])
def test_baseline_shapes(shape, batch, cuda_device):
    M, K = shape
    packed, scales, x = make_problem(M, K, batch, seed=2024)
    ref = oracle_y(x, packed, scales)
    tp, ts, tx = to_device(packed, scales, x)
    for c in (cfg(), cfg(reuse_weights=1), cfg(version=2), cfg(version=4, split_k=4)):
        assert max_err(capi_gemv(tp, ts, tx, c), ref) < MAX_ABS


# x rows above 68 KB staged in shared memory by the 16-warp streaming kernel:
# the ring shrinks to 2-3 stages and, for the largest x (K = 8192, B = 8;
# K = 11008, B = 6), the tile sums run on 2 buffers instead of 4.  Ragged M
# (partial last tiles), bitwise against the register-tiled v3 kernel (same
# canonical order) and within the tolerance of the oracle.
LARGE_X = [(300, 8192, 5), (1000, 8192, 8), (4109, 8192, 6), (257, 11008, 4), (999, 11008, 6),
           (64, 28672, 2)]


@pytest.mark.parametrize("M,K,B", LARGE_X)
def test_large_staged_x_bitwise_v3_and_oracle(M, K, B, cuda_device):
    packed, scales, x = make_problem(M, K, B, seed=4000 + M + B, std=0.05)
    tp, ts, tx = to_device(packed, scales, x)
    y5 = capi_gemv(tp, ts, tx, cfg())
    assert stamp() == 5
    assert torch.equal(y5, capi_gemv(tp, ts, tx, cfg(version=3)))
    assert max_err(y5, oracle_y(x, packed, scales)) < MAX_ABS
    from decode_kernel import capi

    assert capi.load().dk_device_error(-1, 0) == 0


@pytest.mark.parametrize("M,K,B", [(1000, 8192, 8), (2050, 8192, 6)])
def test_large_staged_x_pair_and_multi(M, K, B, cuda_device):
    # The gate/up pair (its gate tile is held until the up tile's sum, so on
    # 2 tile-sum buffers both are in use) and a two-matrix launch, against
    # single-matrix v3 GEMVs.
    import torch.nn.functional as F

    from decode_kernel import capi, gemv_multi, gemv_silu_mul

    pg, sg, x = make_problem(M, K, B, seed=4100 + M + B, std=0.05)
    pu, su, _ = make_problem(M + 37, K, 1, seed=4200 + M + B, std=0.05)
    tg, tsg, tx = to_device(pg, sg, x)
    tu, tsu, _ = to_device(pu, su, x)
    g3, u3 = capi_gemv(tg, tsg, tx, cfg(version=3)), capi_gemv(tu, tsu, tx, cfg(version=3))
    ys = gemv_multi([(tg, tsg), (tu, tsu)], tx)
    assert torch.equal(ys[0], g3) and torch.equal(ys[1], u3)
    h = gemv_silu_mul((tg, tsg), (tu[:M], tsu[:M]), tx)
    assert torch.equal(h, F.silu(g3) * u3[:, :M])
    assert capi.load().dk_device_error(-1, 0) == 0


@pytest.mark.slow
@pytest.mark.parametrize("shape", [(28672, 8192), (8192, 28672), (8192, 8192)])
@pytest.mark.parametrize("batch", [1, 8])
def test_llama70b_shapes_whole_output(shape, batch, cuda_device):
    # Every output row against the oracle's fp32 restatement (numpy, the host's
    # threads), and two windows against its double-precision C form.
    from oracle import oracle as O

    M, K = shape
    packed, scales, x = make_problem(M, K, batch, seed=70)
    tp, ts, tx = to_device(packed, scales, x)
    y = capi_gemv(tp, ts, tx, cfg())
    assert max_err(y, O.linear_fp32_np(x, packed, scales)) < MAX_ABS
    rng = np.random.default_rng(1)
    for a in rng.integers(0, M - 64, size=2):
        rows = (int(a), int(a) + 64)
        assert max_err(y, O.linear_fp32(x, packed, scales, rows=rows), rows=rows) < MAX_ABS
    yr = capi_gemv(tp, ts, tx, cfg(reuse_weights=1))
    assert torch.equal(yr, y)


@pytest.mark.parametrize("B", [9, 12, 16, 17, 24, 31, 32])
@pytest.mark.parametrize("shape", [(16, 128), (100, 1024), (333, 2304), (4096, 4096),
                                   (16384, 384), (20001, 1024), (40000, 256)])
def test_batch_rows_9_to_32(B, shape, cuda_device):
    # 9..32 rows: the mma.sync streaming kernel, or -- for B > 16 on matrices
    # of 16384+ rows -- the tcgen05 batch kernel (row tiles N = 112 .. 256,
    # one and several waves of CTAs, ragged M, K from one group up).
    from decode_kernel import capi

    M, K = shape
    packed, scales, x = make_problem(M, K, B, seed=7 * B + M, std=0.05)
    tp, ts, tx = to_device(packed, scales, x)
    y = capi_gemv(tp, ts, tx, cfg())
    assert capi.load().dk_last_kernel_stamp(-1) == 5
    rows = None if M * K * B <= 64 * 1024 * 1024 else (0, min(M, 2048))
    ref = oracle_y(x, packed, scales, rows=rows)
    assert max_err(y, ref, rows=rows) < MAX_ABS
    yr = capi_gemv(tp, ts, tx, cfg(reuse_weights=1))
    assert capi.load().dk_last_kernel_stamp(-1) == 15
    assert torch.equal(yr, y)
    assert capi.load().dk_device_error(-1, 0) == 0


@pytest.mark.parametrize("B", [1, 3, 9, 33])
@pytest.mark.parametrize("rows", [(4096, 4096, 4096), (11008, 11008), (17, 300, 1, 64), (1000,)])
def test_multi_gemv_is_bitwise_the_separate_gemvs(rows, B, cuda_device):
    # q/k/v- and gate/up-style launches: matrices sharing x, ragged row
    # counts (partial last tiles inside the concatenation), several passes.
    from decode_kernel import capi, gemv_multi

    K = 2048
    mats = [make_problem(m, K, 1, seed=900 + i + m, std=0.05)[:2] for i, m in enumerate(rows)]
    x = np.random.default_rng(B).standard_normal((B, K)).astype(np.float16)
    dev = [to_device(p, s, x) for p, s in mats]
    tx = dev[0][2]
    ys = gemv_multi([(tp, ts) for tp, ts, _ in dev], tx)
    for (tp, ts, _), y, (p, s) in zip(dev, ys, mats):
        assert torch.equal(y, capi_gemv(tp, ts, tx, cfg()))
        if p.shape[0] * B <= 4096 * 3:
            assert max_err(y, oracle_y(x, p, s)) < MAX_ABS
    assert capi.load().dk_device_error(-1, 0) == 0


def test_multi_gemv_rejects(cuda_device):
    from decode_kernel import capi

    c = cfg()
    assert capi.gemv_multi([], [], [], [], 16, 256, 1, c) == capi.DK_ERR_INVALID_ARG
    assert capi.gemv_multi([16] * 5, [16] * 5, [16] * 5, [16] * 5, 16, 256, 1, c) == \
        capi.DK_ERR_INVALID_ARG
    assert capi.gemv_multi([16], [16], [0], [16], 16, 256, 1, c) == capi.DK_ERR_INVALID_ARG
    assert capi.gemv_multi([16], [16], [64], [16], 16, 256, 1, cfg(version=3)) == \
        capi.DK_ERR_UNSUPPORTED


@pytest.mark.parametrize("reuse", [False, True])
@pytest.mark.parametrize("shape", [(11008, 4096, 1), (9500, 2048, 3), (4096, 4096, 4), (1000, 256, 3),
                                   (17, 128, 1), (4096, 1024, 16), (2000, 2048, 32), (300, 1024, 40)])
def test_silu_mul_is_the_unfused_fp16_sequence(shape, reuse, cuda_device):
    # Gate/up with the SiLU-mul epilogue: bitwise the unfused sequence (two
    # GEMVs, torch's silu, fp16 product), and within the propagated oracle
    # bound.  Ragged M (partial last pair), several batch passes (B=40); the
    # first two shapes run as two CTAs per SM (>= 8 tiles per SM).
    import torch.nn.functional as F

    from decode_kernel import gemv_silu_mul

    M, K, B = shape
    pg, sg, x = make_problem(M, K, B, seed=1300 + M + B, std=0.05)
    pu, su, _ = make_problem(M, K, 1, seed=1400 + M + B, std=0.05)
    tg, tsg, tx = to_device(pg, sg, x)
    tu, tsu, _ = to_device(pu, su, x)
    h = gemv_silu_mul((tg, tsg), (tu, tsu), tx, reuse_weights=reuse)
    c = cfg(reuse_weights=int(reuse))
    g16, u16 = capi_gemv(tg, tsg, tx, c), capi_gemv(tu, tsu, tx, c)
    assert torch.equal(h, F.silu(g16) * u16)
    if M * B <= 4096 * 4:
        g, u = oracle_y(x, pg, sg).astype(np.float64), oracle_y(x, pu, su).astype(np.float64)
        s = g / (1.0 + np.exp(-g))
        ref = s * u
        hh = h.float().cpu().numpy()
        assert np.isfinite(hh).all()
        bound = 1.2e-2 * (np.abs(u) + np.abs(s)) + 1e-3 * np.abs(ref) + 1e-3
        assert (np.abs(hh - ref) <= bound).all()
    from decode_kernel import capi

    assert capi.load().dk_device_error(-1, 0) == 0


def test_silu_mul_rejects(cuda_device):
    from decode_kernel import capi, gemv_silu_mul

    c = cfg()
    f = capi.gemv_silu_mul
    assert f(16, 16, 16, 16, 16, 16, 0, 256, 1, c) == capi.DK_ERR_INVALID_ARG       # M < 1
    assert f(16, 16, 16, 16, 16, 16, 64, 200, 1, c) == capi.DK_ERR_INVALID_ARG      # K % 128
    assert f(16, 16, 16, 16, 16, 16, 64, 256, 1, cfg(version=3)) == capi.DK_ERR_UNSUPPORTED
    assert f(16, 16, 16, 16, 16, 16, 64, 256, 1, cfg(flags=capi.DK_FLAG_F32_OUT)) == \
        capi.DK_ERR_UNSUPPORTED
    assert f(16, 16, 16, 16, 16, 16, 64, 256, 0, c) == capi.DK_OK                  # B = 0
    pg, sg, x = make_problem(64, 256, 2, seed=5)
    tg, tsg, tx = to_device(pg, sg, x)
    pu, su, _ = make_problem(32, 256, 1, seed=6)
    tu, tsu, _ = to_device(pu, su, x)
    with pytest.raises(RuntimeError):
        gemv_silu_mul((tg, tsg), (tu, tsu), tx)  # different M

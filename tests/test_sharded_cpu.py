"""Host side of the sharded path (decode_kernel.sharded), on CPU.

The partitioning arithmetic -- which rows / which whole 128-wide groups of K
each rank owns -- and the exchange it implies are checked with gloo process
groups (world 2, 3 and 4, spawned ranks on 127.0.0.1): every rank computes its
shard with the CPU oracle, the ranks all-gather (row-parallel) or all-reduce
(K-parallel) through torch.distributed, and the result must equal the oracle
on the whole matrix.  The CUDA kernels are exercised by test_sharded_gpu.py.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from dkhelpers import make_problem


def test_row_range_covers_every_row_once():
    from decode_kernel.sharded import row_range

    for M in (1, 7, 64, 4096, 11008, 28672):
        for world in range(1, 9):
            seen = []
            for r in range(world):
                row0, rows = row_range(M, world, r)
                assert rows >= M // world and rows <= M // world + 1
                seen.extend(range(row0, row0 + rows))
            assert seen == list(range(M))


def test_k_range_is_group_aligned_and_covers_k():
    from decode_kernel.sharded import k_range

    for K in (128, 4096, 11008, 28672):
        for world in range(1, 9):
            cols = []
            for r in range(world):
                k0, kn = k_range(K, world, r)
                assert k0 % 128 == 0 and kn % 128 == 0
                cols.extend(range(k0, k0 + kn))
            assert cols == list(range(K))
    with pytest.raises(ValueError):
        k_range(200, 2, 0)
    with pytest.raises(ValueError):
        k_range(256, 2, 2)


def test_slices_are_the_owned_parts():
    import torch

    from decode_kernel.sharded import slice_k, slice_rows

    packed, scales, _ = make_problem(40, 1024, 1, seed=3)
    tp = torch.from_numpy(packed)
    ts = torch.from_numpy(scales.view(np.int16)).view(torch.float16)
    rows = [slice_rows(tp, ts, 3, r) for r in range(3)]
    assert torch.equal(torch.cat([p for p, _, _ in rows]), tp)
    assert [r0 for _, _, r0 in rows] == [0, 13, 26]
    ks = [slice_k(tp, ts, 3, r) for r in range(3)]
    assert torch.equal(torch.cat([p for p, _, _ in ks], dim=1), tp)
    assert torch.equal(torch.cat([s for _, s, _ in ks], dim=1), ts)
    assert all(p.is_contiguous() and s.is_contiguous() for p, s, _ in ks)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, layout: str, M: int, K: int, B: int,
               out_path: str) -> None:
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from decode_kernel.sharded import k_range, row_range

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        packed, scales, x = make_problem(M, K, B, seed=91)
        if layout == "row":
            row0, rows = row_range(M, world, rank)
            part = O.linear_fp32(x, packed[row0:row0 + rows], scales[row0:row0 + rows])
            pieces = [None] * world
            dist.all_gather_object(pieces, part)
            y = np.concatenate(pieces, axis=1)
        else:
            k0, kn = k_range(K, world, rank)
            p = np.ascontiguousarray(packed[:, k0 // 8:(k0 + kn) // 8])
            s = np.ascontiguousarray(scales[:, k0 // 128:(k0 + kn) // 128])
            part = torch.from_numpy(O.linear_fp32(np.ascontiguousarray(x[:, k0:k0 + kn]), p, s))
            dist.all_reduce(part)
            y = part.numpy()
        np.save(f"{out_path}.{rank}.npy", y)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("layout", ["row", "k"])
@pytest.mark.parametrize("world", [2, 3, 4])
def test_gloo_exchange_matches_whole_matrix(layout, world, tmp_path):
    import torch.multiprocessing as mp

    from oracle import oracle as O

    M, K, B = 96, 1408, 2  # 11 groups: K slices of unequal size at world 2, 3 and 4
    out = str(tmp_path / "y")
    mp.start_processes(_rank_main, args=(world, _free_port(), layout, M, K, B, out),
                       nprocs=world, start_method="spawn", join=True)
    packed, scales, x = make_problem(M, K, B, seed=91)
    ref = O.linear_fp32(x, packed, scales)
    for r in range(world):
        y = np.load(f"{out}.{r}.npy")
        assert y.shape == ref.shape
        if layout == "row":
            assert np.array_equal(y, ref)  # row slices are independent
        else:
            assert np.abs(y - ref).max() < 1e-4


def _group(world=2, rank=0, **kw):
    from decode_kernel import capi

    g = capi.ShardGroup()
    g.rank, g.world = rank, world
    for r in range(min(world, capi.DK_MAX_SHARDS)):
        g.bufs[r] = 4096 * (r + 1)
        g.slots[r] = 8192 * (r + 1)
    g.seq = 64
    for k, v in kw.items():
        setattr(g, k, v)
    return g


def test_shard_entries_reject_bad_arguments_without_a_device():
    import ctypes

    from decode_kernel import capi

    lib = capi.load()
    cfg = capi.default_config()

    def row(g, M_shard=64, row0=0, M_total=128, K=256, B=1, c=cfg):
        return lib.dk_w4a16_gemv_rowshard(16, 16, 16, M_shard, row0, M_total, K, B,
                                          ctypes.byref(g), ctypes.byref(c), None)

    assert row(_group(world=0)) == capi.DK_ERR_INVALID_ARG
    assert row(_group(world=9)) == capi.DK_ERR_INVALID_ARG
    assert row(_group(world=2, rank=2)) == capi.DK_ERR_INVALID_ARG
    assert row(_group(seq=None)) == capi.DK_ERR_INVALID_ARG
    bad = _group()
    bad.bufs[1] = None
    assert row(bad) == capi.DK_ERR_INVALID_ARG
    assert row(_group(), row0=100) == capi.DK_ERR_INVALID_ARG  # rows past M_total
    assert row(_group(), K=200) == capi.DK_ERR_INVALID_ARG
    assert row(_group(), B=33) == capi.DK_ERR_UNSUPPORTED
    assert row(_group(), c=capi.default_config(version=3)) == capi.DK_ERR_UNSUPPORTED
    assert row(_group(), c=capi.default_config(flags=capi.DK_FLAG_F32_OUT)) == \
        capi.DK_ERR_UNSUPPORTED
    # K-parallel: x rows must be at least K_shard apart and 16-byte aligned.
    assert lib.dk_w4a16_gemv_kshard(16, 16, 16, 128, 64, 256, 1, ctypes.byref(_group()),
                                    ctypes.byref(cfg), None) == capi.DK_ERR_INVALID_ARG
    assert lib.dk_w4a16_gemv_kshard(16, 16, 16, 260, 64, 256, 1, ctypes.byref(_group()),
                                    ctypes.byref(cfg), None) == capi.DK_ERR_INVALID_ARG
    assert lib.dk_shard_wait(None, None) == capi.DK_ERR_INVALID_ARG
    assert lib.dk_shard_wait(ctypes.byref(_group(seq=None)), None) == capi.DK_ERR_INVALID_ARG
    assert lib.dk_shard_wait(ctypes.byref(_group(world=9)), None) == capi.DK_ERR_INVALID_ARG
    assert lib.dk_shard_reduce(ctypes.byref(_group(world=0)), 8, 1, 16, 0, None) == \
        capi.DK_ERR_INVALID_ARG
    assert lib.dk_shard_reduce(ctypes.byref(_group()), 8, 1, None, 0, None) == \
        capi.DK_ERR_INVALID_ARG
    # the in-kernel wait is for sharded calls only
    assert capi.gemv(16, 16, 16, 16, 64, 256, 1,
                     capi.default_config(flags=capi.DK_FLAG_SHARD_WAIT)) == capi.DK_ERR_INVALID_ARG


def test_f32_flag_only_on_the_streaming_kernel():
    from decode_kernel import capi

    for v in range(5):
        c = capi.default_config(version=v, flags=capi.DK_FLAG_F32_OUT)
        assert capi.gemv(16, 16, 16, 16, 64, 256, 1, c) == capi.DK_ERR_UNSUPPORTED
    assert capi.gemv(16, 16, 16, 16, 64, 256, 1,
                     capi.default_config(flags=0x8)) == capi.DK_ERR_INVALID_ARG


def _tp_rank_main(rank: int, world: int, port: int, out_path: str) -> None:
    import torch
    import torch.distributed as dist

    from oracle import oracle as O
    from decode_kernel.sharded import split_dim

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        (pg, sg, x), (pu, su, _), (pd, sd, _) = _tp_problem()
        # gate/up: this rank's output rows; down: the same range of its K
        i0, n = split_dim(pg.shape[0], world, rank)
        g = O.linear_fp32(x, pg[i0:i0 + n], sg[i0:i0 + n]).astype(np.float64)
        u = O.linear_fp32(x, pu[i0:i0 + n], su[i0:i0 + n]).astype(np.float64)
        h = (g / (1 + np.exp(-g)) * u).astype(np.float16)
        p = np.ascontiguousarray(pd[:, i0 // 8:(i0 + n) // 8])
        s = np.ascontiguousarray(sd[:, i0 // 128:(i0 + n) // 128])
        part = torch.from_numpy(O.linear_fp32(h, p, s))
        dist.all_reduce(part)  # the block's one exchange
        np.save(f"{out_path}.{rank}.npy", part.numpy())
    finally:
        dist.destroy_process_group()


def _tp_problem():
    I, K, M, B = 640, 256, 64, 2  # 5 blocks of 128: unequal splits at 2, 3 and 4 ranks
    return (make_problem(I, K, B, seed=95), make_problem(I, K, 1, seed=96),
            make_problem(M, I, 1, seed=97))


@pytest.mark.parametrize("world", [2, 3, 4])
def test_gloo_tensor_parallel_mlp_matches_whole_layer(world, tmp_path):
    # The row split of gate/up is the K split of down, so the ranks' partials
    # of down over their own h slices add up to the whole layer.
    import torch.multiprocessing as mp

    from oracle import oracle as O

    out = str(tmp_path / "y")
    mp.start_processes(_tp_rank_main, args=(world, _free_port(), out), nprocs=world,
                       start_method="spawn", join=True)
    (pg, sg, x), (pu, su, _), (pd, sd, _) = _tp_problem()
    g = O.linear_fp32(x, pg, sg).astype(np.float64)
    u = O.linear_fp32(x, pu, su).astype(np.float64)
    h = (g / (1 + np.exp(-g)) * u).astype(np.float16)
    ref = O.linear_fp32(h, pd, sd)
    for r in range(world):
        y = np.load(f"{out}.{r}.npy")
        assert y.shape == ref.shape
        assert np.abs(y - ref).max() < 1e-4 * max(1.0, np.abs(ref).max())


def test_split_dim_is_head_aligned():
    from decode_kernel.sharded import k_range, split_dim

    for n, world in [(8192, 8), (1024, 8), (11008, 4), (28672, 8)]:
        parts = [split_dim(n, world, r) for r in range(world)]
        assert parts == [k_range(n, world, r) for r in range(world)]
        assert all(k0 % 128 == 0 and kn % 128 == 0 and kn > 0 for k0, kn in parts)
        assert sum(kn for _, kn in parts) == n


def test_layer_inputs_are_checked_before_any_launch():
    # Every sharded layer passes x through this check before it hands a
    # pointer to the kernels; a tensor on another device is refused.
    import torch

    from decode_kernel.sharded import _as_batch

    cpu, gpu = torch.device("cpu"), torch.device("cuda", 0)
    x = torch.zeros(2, 256, dtype=torch.float16)
    assert _as_batch(x, 256, 2, cpu) is x
    assert _as_batch(x[0], 256, 1, cpu).shape == (1, 256)
    with pytest.raises(RuntimeError, match="is on cpu"):
        _as_batch(x, 256, 2, gpu)
    with pytest.raises(RuntimeError, match="max_batch"):
        _as_batch(x, 256, 1, cpu)
    for bad in (x.float(), x[:, :128], x.t(), x.reshape(2, 2, 128)):
        with pytest.raises(RuntimeError, match="contiguous fp16"):
            _as_batch(bad, 256, 2, cpu)


# --- failure detection on the host: a rank that leaves or never joins ------
#
# Ranks are gloo processes on the CPU and the failures are made on the host;
# nothing here touches a GPU.  The process group is created as the sharded
# benches create theirs, with a short timeout, so the surviving ranks end
# their next collective (or the rendezvous) with an error instead of waiting.

_FAIL_TIMEOUT_S = 5


def _fail_rank_main(rank: int, world: int, port: int, mode: str, out_path: str) -> None:
    import datetime
    import time

    import torch
    import torch.distributed as dist

    t0 = time.monotonic()

    def record(what: str) -> None:
        with open(f"{out_path}.{rank}", "w") as f:
            f.write(f"{what} {time.monotonic() - t0:.1f}")

    if mode == "never_joins" and rank == world - 1:
        return
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world,
                                timeout=datetime.timedelta(seconds=_FAIL_TIMEOUT_S))
    except Exception:  # the rendezvous gave up on the missing rank
        record("init_error")
        return
    x = torch.ones(64)
    try:
        dist.all_reduce(x)  # step 1: every rank takes part
        if mode == "exits" and rank == world - 1:
            record("left")
            return  # this rank leaves between steps, with no collective in flight
        dist.all_reduce(x)  # step 2: the survivors must get an error, not hang
        record("no_error")
    except Exception:
        record("step_error")


@pytest.mark.parametrize("mode", ["exits", "never_joins"])
def test_lost_rank_ends_the_survivors_collective_with_an_error(mode, tmp_path):
    import time

    import torch.multiprocessing as mp

    world = 3
    out = str(tmp_path / "r")
    ctx = mp.start_processes(_fail_rank_main, args=(world, _free_port(), mode, out),
                             nprocs=world, start_method="spawn", join=False)
    deadline = time.monotonic() + 120
    while not ctx.join(timeout=5):
        if time.monotonic() > deadline:
            for p in ctx.processes:
                p.kill()
            pytest.fail("ranks still running after 120 s")
    results = {}
    for r in range(world):
        path = f"{out}.{r}"
        if os.path.exists(path):
            what, secs = open(path).read().split()
            results[r] = (what, float(secs))
    want = "step_error" if mode == "exits" else "init_error"
    for r in range(world - 1):
        assert results[r][0] == want, results
        assert results[r][1] < 4 * _FAIL_TIMEOUT_S + 10, results
    if mode == "exits":
        assert results[world - 1][0] == "left"
    else:
        assert world - 1 not in results

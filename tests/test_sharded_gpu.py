"""The sharded GEMV on the GPU: fused exchange over peer memory.

Single GPU: ``PeerBuffers(emulate=G)`` keeps all G ranks' buffers and
counters on one GPU and launches every rank's kernel in turn on one stream,
so the fused path -- each rank's epilogue storing into every rank's buffer,
the arrival counters, the bounded waits, the rank-ordered K reduction -- runs
for G up to 8 without G GPUs.  Row-parallel results must equal the unsharded
GEMV bit for bit (row slices are independent); K-parallel results must equal,
bit for bit, fp16 of the rank-ordered sum of the fp32 slice GEMVs, and be
within 1e-2 of the oracle.  With two or more GPUs the same layers run as real
ranks (spawned processes, NCCL for the handle exchange).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from dkhelpers import MAX_ABS, capi_gemv, make_problem, max_err, oracle_y, to_device

pytestmark = pytest.mark.gpu


def f32_gemv(tp, ts, tx):
    from decode_kernel import capi

    M, K, B = tp.shape[0], tp.shape[1] * 8, tx.shape[0]
    y = torch.full((B, M), float("nan"), dtype=torch.float32, device=tp.device)
    capi.check(capi.gemv(tp.data_ptr(), ts.data_ptr(), tx.data_ptr(), y.data_ptr(), M, K, B,
                         capi.default_config(flags=capi.DK_FLAG_F32_OUT), 0, 0,
                         torch.cuda.current_stream().cuda_stream), "f32 gemv")
    return y


@pytest.mark.parametrize("B", [1, 5, 9, 33])
@pytest.mark.parametrize("reuse", [0, 1])
def test_f32_output_rounds_to_the_fp16_output(B, reuse, cuda_device):
    from decode_kernel import capi

    packed, scales, x = make_problem(300, 2048, B, seed=60 + B)
    tp, ts, tx = to_device(packed, scales, x)
    y16 = capi_gemv(tp, ts, tx, capi.default_config(reuse_weights=reuse))
    M, K = 300, 2048
    y32 = torch.full((B, M), float("nan"), dtype=torch.float32, device=cuda_device)
    cfg = capi.default_config(reuse_weights=reuse, flags=capi.DK_FLAG_F32_OUT)
    capi.check(capi.gemv(tp.data_ptr(), ts.data_ptr(), tx.data_ptr(), y32.data_ptr(), M, K, B,
                         cfg, 0, 0, 0), "f32")
    torch.cuda.synchronize()
    assert torch.equal(y32.half(), y16)
    assert max_err(y32, oracle_y(x, packed, scales)) < MAX_ABS


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("B", [1, 3])
def test_row_parallel_emulated_is_the_unsharded_gemv(world, B, cuda_device):
    from decode_kernel.sharded import PeerBuffers, RowParallelW4A16

    M, K = 1376, 4096
    packed, scales, x = make_problem(M, K, B, seed=200 + world)
    tp, ts, tx = to_device(packed, scales, x)
    peers = PeerBuffers(8 * B * M, emulate=world)
    layer = RowParallelW4A16(tp, ts, peers, max_batch=B)
    try:
        for call in range(3):  # both buffer sets, counters accumulating
            xc = (tx * (1 + call)).contiguous()
            full = capi_gemv(tp, ts, xc)
            layer(xc, pdl=(call == 1))
            torch.cuda.synchronize()
            which = call & 1
            for r in range(world):
                assert torch.equal(peers.view(r, which, (B, M), torch.float16), full), (call, r)
        from decode_kernel import capi

        assert capi.load().dk_device_error(-1, 1) == 0
    finally:
        peers.close()


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("B", [1, 4])
def test_k_parallel_emulated_sums_the_slices_in_rank_order(world, B, cuda_device):
    from decode_kernel.sharded import KParallelW4A16, PeerBuffers, slice_k

    M, K = 512, 11008  # 86 groups: unequal slices for 4 and 8 ranks
    packed, scales, x = make_problem(M, K, B, seed=300 + world, std=0.05)
    tp, ts, tx = to_device(packed, scales, x)
    peers = PeerBuffers(8 * world * B * M, emulate=world)
    layer = KParallelW4A16(tp, ts, peers, max_batch=B)
    try:
        for call in range(2):
            y = layer(tx).clone()
            outs = [layer.out[r][:B].clone() for r in range(world)]
            torch.cuda.synchronize()
            for o in outs[1:]:
                assert torch.equal(o, outs[0])
            # fp16(sum in rank order of the fp32 slice GEMVs), bit for bit.
            acc = torch.zeros((B, M), dtype=torch.float32, device=cuda_device)
            for r in range(world):
                p, s, k0 = slice_k(tp, ts, world, r)
                acc += f32_gemv(p, s, tx[:, k0:k0 + p.shape[1] * 8].contiguous())
            assert torch.equal(y, acc.half())
            assert max_err(y, oracle_y(x, packed, scales)) < MAX_ABS
    finally:
        peers.close()


def test_shard_wait_on_a_counter_nobody_bumps_times_out(cuda_device):
    # The bounded wait gives up after ~2 s, records the timeout in the
    # device error word and lets the stream continue; the context stays usable.
    # (A slot array that nothing marks.)
    import ctypes

    from decode_kernel import capi

    lib = capi.load()
    lib.dk_device_error(-1, 1)
    slots = torch.zeros(capi.DK_MAX_SHARDS * capi.DK_SHARD_SLOTS, dtype=torch.int32,
                        device=cuda_device)
    seq = torch.tensor([0, 3, 0, 0], dtype=torch.int32, device=cuda_device)  # 3 CTAs per rank
    g = capi.ShardGroup()
    g.rank, g.world = 0, 2
    g.bufs[0] = g.bufs[1] = slots.data_ptr()
    g.slots[0] = g.slots[1] = slots.data_ptr()
    g.seq = seq.data_ptr()
    st = torch.cuda.current_stream().cuda_stream
    capi.check(lib.dk_shard_wait(ctypes.byref(g), st), "dk_shard_wait")
    torch.cuda.synchronize()
    assert lib.dk_device_error(-1, 1) == 1
    assert lib.dk_device_error(-1, 0) == 0
    assert int(seq[0]) == 1  # the sequence moved on by one call
    # All 2 x 3 slots marked with call 2: the wait returns at once.
    for r in range(2):
        slots[r * capi.DK_SHARD_SLOTS:r * capi.DK_SHARD_SLOTS + 3] = 2
    capi.check(lib.dk_shard_wait(ctypes.byref(g), st), "dk_shard_wait")
    torch.cuda.synchronize()
    assert lib.dk_device_error(-1, 0) == 0
    assert int(seq[0]) == 2
    # One slot short of call 3: times out again.
    slots[0:3] = 3
    slots[capi.DK_SHARD_SLOTS:capi.DK_SHARD_SLOTS + 2] = 3
    capi.check(lib.dk_shard_wait(ctypes.byref(g), st), "dk_shard_wait")
    torch.cuda.synchronize()
    assert lib.dk_device_error(-1, 1) == 1


def test_row_parallel_step_replays_from_a_cuda_graph(cuda_device):
    # The waits keep their place in the arrival count on the device, so a
    # captured step replays: every replay waits for that replay's arrivals.
    from decode_kernel import capi
    from decode_kernel.sharded import PeerBuffers, RowParallelW4A16

    M, K, B, world = 1024, 2048, 1, 4
    packed, scales, x = make_problem(M, K, B, seed=5)
    tp, ts, tx = to_device(packed, scales, x)
    peers = PeerBuffers(8 * B * M, emulate=world)
    layer = RowParallelW4A16(tp, ts, peers, max_batch=B)
    try:
        xin = tx.clone()
        layer(xin)
        layer(xin)  # warm-up outside capture, both buffer sets
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            layer(xin)
            layer(xin)
        for step in range(3):
            xin.copy_(tx * (step + 2))
            full = capi_gemv(tp, ts, xin)
            g.replay()
            torch.cuda.synchronize()
            for which in (0, 1):
                for r in range(world):
                    assert torch.equal(peers.view(r, which, (B, M), torch.float16), full)
        assert capi.load().dk_device_error(-1, 1) == 0
        del g
    finally:
        peers.close()


def _k_parallel_expected(pd, sd, h, world):
    """fp16 of the rank-ordered sum of the fp32 GEMVs of down's K slices."""
    from decode_kernel.sharded import slice_k

    acc = torch.zeros((h.shape[0], pd.shape[0]), dtype=torch.float32, device=h.device)
    for r in range(world):
        p, s, k0 = slice_k(pd, sd, world, r)
        acc += f32_gemv(p, s, h[:, k0:k0 + p.shape[1] * 8].contiguous())
    return acc.half()


@pytest.mark.parametrize("world", [1, 2, 3, 4])
@pytest.mark.parametrize("B", [1, 3])
def test_tensor_parallel_mlp_emulated(world, B, cuda_device):
    # gate/up row-parallel through the SiLU-mul pair, down K-parallel over the
    # same split (9 blocks of 128: unequal for 2 and 4 ranks).
    from decode_kernel import gemv_silu_mul
    from decode_kernel.sharded import PeerBuffers, TensorParallelMLP

    I, K, M = 1152, 512, 384
    pg, sg, x = make_problem(I, K, B, seed=500 + world, std=0.05)
    pu, su, _ = make_problem(I, K, 1, seed=600 + world, std=0.05)
    pd, sd, _ = make_problem(M, I, 1, seed=700 + world, std=0.05)
    (tg, tsg, tx), (tu, tsu, _), (td, tsd, _) = (to_device(pg, sg, x), to_device(pu, su, x),
                                                  to_device(pd, sd, x[:, :0]))
    peers = PeerBuffers(8 * world * B * M, emulate=world)
    mlp = TensorParallelMLP((tg, tsg), (tu, tsu), (td, tsd), peers, max_batch=B)
    try:
        for call in range(2):
            xc = (tx * (1 + call)).contiguous()
            y = mlp(xc, pdl=(call == 1)).clone()
            h = gemv_silu_mul((tg, tsg), (tu, tsu), xc)
            assert torch.equal(y, _k_parallel_expected(td, tsd, h, world)), call
        from decode_kernel import capi

        assert capi.load().dk_device_error(-1, 1) == 0
    finally:
        peers.close()


@pytest.mark.parametrize("world", [1, 2, 4])
def test_tensor_parallel_attention_proj_emulated(world, cuda_device):
    # q/k/v by heads in one multi-GEMV per rank, o K-parallel over the head
    # split; the rank's q slice stands in for its attention output.
    from decode_kernel.sharded import PeerBuffers, TensorParallelAttentionProj

    B, K, Q, KV = 2, 1024, 1024, 512
    mats = [make_problem(m, K, B, seed=800 + i, std=0.05) for i, m in enumerate((Q, KV, KV))]
    po, so, _ = make_problem(K, Q, 1, seed=900, std=0.05)
    x = mats[0][2]
    dq, dk_, dv = (to_device(p, s, x) for p, s, _ in mats)
    tx = dq[2]
    to, tso, _ = to_device(po, so, x[:, :0])
    peers = PeerBuffers(8 * world * B * K, emulate=world)
    proj = TensorParallelAttentionProj(dq[:2], dk_[:2], dv[:2], (to, tso), peers, max_batch=B)
    try:
        y = proj(tx).clone()
        q = capi_gemv(*dq[:2], tx)
        assert torch.equal(y, _k_parallel_expected(to, tso, q, world))
        seen = []
        proj(tx, attn=lambda r, q_, k_, v_: seen.append((r, q_.shape, k_.shape, v_.shape)) or q_)
        assert [r for r, *_ in seen] == list(range(world))
        assert sum(sh[1][1] for sh in seen) == Q and sum(sh[2][1] for sh in seen) == KV
    finally:
        peers.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out_path: str) -> None:
    import datetime

    import torch.distributed as dist

    from decode_kernel.sharded import KParallelW4A16, PeerBuffers, RowParallelW4A16

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        M, K, B = 2048, 4096, 2
        packed, scales, x = make_problem(M, K, B, seed=77)
        dev = torch.device("cuda", rank)
        tp = torch.from_numpy(packed).to(dev)
        ts = torch.from_numpy(scales.view(np.int16)).to(dev).view(torch.float16)
        tx = torch.from_numpy(x.view(np.int16)).to(dev).view(torch.float16)
        peers = PeerBuffers(8 * world * 12 * max(M, K))
        rowl = RowParallelW4A16(tp, ts, peers, max_batch=B)
        kl = KParallelW4A16(tp, ts, peers, max_batch=B)
        for _ in range(3):  # both buffer sets, the call number advancing
            y_row = rowl(tx).clone()
            y_k = kl(tx).clone()
        y_row_nccl = RowParallelW4A16(tp, ts, peers, max_batch=B, exchange="nccl")(tx)
        y_k_nccl = KParallelW4A16(tp, ts, peers, max_batch=B, exchange="nccl")(tx)
        # 12 batch rows: above the 8 that the GEMV sums in-kernel, so the
        # K-parallel call stores partials and a separate kernel sums them.
        x12 = torch.from_numpy(make_problem(M, K, 12, seed=79)[2].view(np.int16)).to(dev)
        x12 = x12.view(torch.float16)
        y_k12 = KParallelW4A16(tp, ts, peers, max_batch=12)(x12).clone()
        y_k12_nccl = KParallelW4A16(tp, ts, peers, max_batch=12, exchange="nccl")(x12)
        # ... and the gathered row-parallel call with 12 rows takes the
        # fp16 stores with arrival slots instead of the in-kernel gather.
        y_row12 = RowParallelW4A16(tp, ts, peers, max_batch=12)(x12).clone()
        y_row12_nccl = RowParallelW4A16(tp, ts, peers, max_batch=12, exchange="nccl")(x12)
        # Tensor-parallel MLP (gate/up = W, down = W's first K rows as [K, M]
        # shapes): real ranks, NCCL, and both ranks emulated on this GPU.
        from decode_kernel.sharded import TensorParallelMLP

        pd, sd, _ = make_problem(K, M, 1, seed=78)
        td = torch.from_numpy(pd).to(dev)
        tsd = torch.from_numpy(sd.view(np.int16)).to(dev).view(torch.float16)
        args = ((tp, ts), (tp, ts), (td, tsd))
        y_tp = TensorParallelMLP(*args, peers, max_batch=B)(tx).clone()
        y_tp_nccl = TensorParallelMLP(*args, peers, max_batch=B, exchange="nccl")(tx).clone()
        emu = PeerBuffers(8 * world * B * K, emulate=world)
        y_tp_emu = TensorParallelMLP(*args, emu, max_batch=B)(tx).clone()
        torch.cuda.synchronize()
        emu.close()
        from decode_kernel import capi

        err = capi.load().dk_device_error(-1, 0)
        np.savez(f"{out_path}.{rank}.npz", row=y_row.float().cpu().numpy(),
                 k=y_k.float().cpu().numpy(), row_nccl=y_row_nccl.float().cpu().numpy(),
                 k_nccl=y_k_nccl.float().cpu().numpy(), tp=y_tp.float().cpu().numpy(),
                 k12=y_k12.float().cpu().numpy(), k12_nccl=y_k12_nccl.float().cpu().numpy(),
                 row12=y_row12.float().cpu().numpy(),
                 row12_nccl=y_row12_nccl.float().cpu().numpy(),
                 tp_nccl=y_tp_nccl.float().cpu().numpy(), tp_emu=y_tp_emu.float().cpu().numpy(),
                 err=err)
        dist.barrier()
        peers.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")
def test_two_real_ranks_fused_and_nccl(tmp_path):
    import torch.multiprocessing as mp

    world = 2
    out = str(tmp_path / "y")
    env = dict(os.environ)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.start_processes(_rank_main, args=(world, _free_port(), out), nprocs=world,
                           start_method="spawn", join=True)
    finally:
        os.environ.clear()
        os.environ.update(env)
    packed, scales, x = make_problem(2048, 4096, 2, seed=77)
    ref = oracle_y(x, packed, scales)
    got = [np.load(f"{out}.{r}.npz") for r in range(world)]
    for g in got:
        assert int(g["err"]) == 0
        assert np.array_equal(g["row"], got[0]["row"]) and np.array_equal(g["k"], got[0]["k"])
        assert np.array_equal(g["row"], g["row_nccl"])  # same kernel rows, gathered
        # the fused exchange sums the two partials as NCCL does (a + b), and the
        # real ranks equal the emulated ones bit for bit
        assert np.array_equal(g["tp"], g["tp_emu"]) and np.array_equal(g["tp"], g["tp_nccl"])
        assert np.array_equal(g["tp"], got[0]["tp"])
        assert np.array_equal(g["k12"], g["k12_nccl"]) and np.array_equal(g["k12"], got[0]["k12"])
        assert np.array_equal(g["row12"], g["row12_nccl"])
        for key in ("row", "k", "row_nccl", "k_nccl"):
            assert np.abs(g[key] - ref).max() < MAX_ABS, key

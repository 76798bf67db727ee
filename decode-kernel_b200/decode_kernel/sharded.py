"""W4A16 layers sharded across the GPUs of one node, one process per GPU.

Two layouts (the reference is single-GPU; these serve its 7B-stack and
70B-layer configurations across 1/2/4/8 B200s):

* ``RowParallelW4A16`` -- rank r owns the output rows
  ``[r*M//G, (r+1)*M//G)`` (a contiguous slice of ``packed`` and ``scales``,
  no repacking); ``x`` is replicated; every rank ends with the full ``y``.
* ``KParallelW4A16`` -- rank r owns a group-aligned slice of K (copied once
  into its own contiguous ``packed``/``scales``); every rank computes an fp32
  partial ``[B, M]`` and every rank ends with the sum in rank order.  The
  partials travel as 64-bit {value, call number} words (8 bytes per value
  in the peer buffers), which the sum polls directly.
* ``TensorParallelAttentionProj`` / ``TensorParallelMLP`` -- a decoder
  layer's projections in the tensor-parallel layout: q/k/v and gate/up split
  by output rows (heads, intermediate size) with no exchange, o and down
  K-parallel over the same split; one exchange per block instead of one per
  projection.

``exchange="fused"`` (default) runs the exchange inside the GEMV: the kernel's
epilogue stores its results straight into every rank's buffer over NVLink peer
memory and marks its arrival slot in every rank's slot array
(``dk_w4a16_gemv_rowshard`` / ``dk_w4a16_gemv_kshard``).  Ranks on their own
GPUs run with ``DK_FLAG_SHARD_WAIT``: the kernel's last CTA waits (bounded)
for every rank's part, so the call completes with the gather complete while a
PDL-launched successor already streams its weights; emulated ranks wait with a
separate ``dk_shard_wait`` after all of them have run.  One rank alone skips
the exchange and runs the plain GEMV.
``exchange="nccl"`` runs the plain GEMV followed by torch.distributed
collectives -- the baseline the fused path is measured against.

Peer buffers are plain device allocations shared by CUDA IPC handles that the
ranks swap over the process group.  ``PeerBuffers(..., emulate=G)`` instead
keeps all G ranks' buffers in one process on one GPU, so the whole code path
(every rank's kernel writing every rank's buffer, the counters, the waits) can
be exercised without G GPUs: the ranks' kernels then run one after another on
one stream, and no kernel ever waits for one that has not already finished.
"""

from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import torch

from . import capi
from .quantize import GROUP_SIZE

__all__ = [
    "PeerBuffers",
    "RowParallelW4A16",
    "KParallelW4A16",
    "row_range",
    "k_range",
    "slice_rows",
    "slice_k",
    "split_dim",
    "TensorParallelMLP",
    "TensorParallelAttentionProj",
]


# --------------------------------------------------------------------------
# Partitioning (host arithmetic; also what the CPU tests check)
# --------------------------------------------------------------------------

def row_range(M: int, world: int, rank: int) -> tuple[int, int]:
    """Output rows [row0, row0 + rows) of ``rank``: balanced and contiguous."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    row0 = rank * M // world
    return row0, (rank + 1) * M // world - row0


def k_range(K: int, world: int, rank: int) -> tuple[int, int]:
    """Reduction columns [k0, k0 + kn) of ``rank``: whole 128-wide groups,
    balanced over the ranks (K // 128 need not divide by the world)."""
    if K % GROUP_SIZE:
        raise ValueError(f"K={K} is not a multiple of {GROUP_SIZE}")
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    groups = K // GROUP_SIZE
    g0, g1 = rank * groups // world, (rank + 1) * groups // world
    return g0 * GROUP_SIZE, (g1 - g0) * GROUP_SIZE


def slice_rows(packed: torch.Tensor, scales: torch.Tensor, world: int, rank: int):
    """(packed rows, scales rows, row0) of ``rank`` (views, contiguous)."""
    row0, rows = row_range(packed.shape[0], world, rank)
    return packed[row0:row0 + rows], scales[row0:row0 + rows], row0


def slice_k(packed: torch.Tensor, scales: torch.Tensor, world: int, rank: int):
    """(packed, scales, k0) of ``rank``'s K slice as new contiguous tensors."""
    K = packed.shape[1] * 8
    k0, kn = k_range(K, world, rank)
    p = packed[:, k0 // 8:(k0 + kn) // 8].contiguous()
    s = scales[:, k0 // GROUP_SIZE:(k0 + kn) // GROUP_SIZE].contiguous()
    return p, s, k0


# --------------------------------------------------------------------------
# Peer memory
# --------------------------------------------------------------------------

class _DeviceArray:
    """A raw device allocation described by __cuda_array_interface__."""

    def __init__(self, ptr: int, shape: Sequence[int], typestr: str):
        self.__cuda_array_interface__ = {
            "data": (int(ptr), False), "shape": tuple(shape), "typestr": typestr,
            "strides": None, "version": 3,
        }


def _check(status: int, what: str) -> None:
    capi.check(status, what)


_SLOT_BYTES = 4 * capi.DK_MAX_SHARDS * capi.DK_SHARD_SLOTS


class PeerBuffers:
    """Result buffers (two sets, used in turn) and arrival slots of every
    rank, mapped in this process.

    ``nbytes`` is the size of one result buffer.  With a process group each
    process owns its own rank's memory and maps the others'; with
    ``emulate=G`` one process owns all G ranks' memory on its one GPU.
    """

    def __init__(self, nbytes: int, group=None, emulate: Optional[int] = None):
        self.lib = capi.load()
        self.nbytes = int(nbytes)
        self._owned: list[int] = []
        self._mapped: list[int] = []
        self.calls = 0
        if emulate is not None:
            self.world, self.rank, self.emulated = int(emulate), 0, True
            if not 1 <= self.world <= capi.DK_MAX_SHARDS:
                raise ValueError(f"world {self.world} outside 1..{capi.DK_MAX_SHARDS}")
            self.bufs = [[self._alloc(self.nbytes) for _ in range(self.world)] for _ in range(2)]
            self.slots = [self._alloc(_SLOT_BYTES) for _ in range(self.world)]
            self.seqs = [self._alloc(16) for _ in range(self.world)]
            return
        import torch.distributed as dist

        self.emulated = False
        self.world = dist.get_world_size(group) if group is not None or dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if self.world > 1 else 0
        if not 1 <= self.world <= capi.DK_MAX_SHARDS:
            raise ValueError(f"world {self.world} outside 1..{capi.DK_MAX_SHARDS}")
        mine = [self._alloc(self.nbytes), self._alloc(self.nbytes), self._alloc(_SLOT_BYTES)]
        self.seqs = [self._alloc(16)]
        if self.world == 1:
            self.bufs = [[mine[0]], [mine[1]]]
            self.slots = [mine[2]]
            return
        handles = []
        for ptr in mine:
            h = ctypes.create_string_buffer(capi.DK_PEER_HANDLE_BYTES)
            _check(self.lib.dk_peer_export(ptr, h), "dk_peer_export")
            handles.append(bytes(h.raw))
        everyone: list = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        table = []
        for r, hs in enumerate(everyone):
            if r == self.rank:
                table.append(mine)
                continue
            row = []
            for h in hs:
                p = ctypes.c_void_p()
                _check(self.lib.dk_peer_import(h, ctypes.byref(p)), "dk_peer_import")
                self._mapped.append(p.value)
                row.append(p.value)
            table.append(row)
        self.bufs = [[table[r][0] for r in range(self.world)],
                     [table[r][1] for r in range(self.world)]]
        self.slots = [table[r][2] for r in range(self.world)]

    def _alloc(self, n: int) -> int:
        p = ctypes.c_void_p()
        _check(self.lib.dk_peer_alloc(n, ctypes.byref(p)), "dk_peer_alloc")
        self._owned.append(p.value)
        return p.value

    # Ranks this process acts for: all of them when emulating, else its own.
    def local_ranks(self) -> list[int]:
        return list(range(self.world)) if self.emulated else [self.rank]

    def group(self, rank: int, which: int) -> capi.ShardGroup:
        g = capi.ShardGroup()
        g.rank, g.world = rank, self.world
        for r in range(self.world):
            g.bufs[r] = self.bufs[which][r]
            g.slots[r] = self.slots[r]
        g.seq = self.seqs[rank if self.emulated else 0]
        return g

    def view(self, rank: int, which: int, shape: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        """``rank``'s buffer of set ``which`` as a tensor (no copy)."""
        typestr = {torch.float16: "<f2", torch.float32: "<f4"}[dtype]
        n = 1
        for d in shape:
            n *= int(d)
        if n * torch.finfo(dtype).bits // 8 > self.nbytes:
            raise ValueError("view larger than the peer buffer")
        return torch.as_tensor(_DeviceArray(self.bufs[which][rank], shape, typestr),
                               device=torch.device("cuda", torch.cuda.current_device()))

    def begin(self) -> int:
        """Buffer set the next call writes (the sets alternate)."""
        which = self.calls & 1
        self.calls += 1
        return which

    def close(self) -> None:
        torch.cuda.synchronize()
        for p in self._mapped:
            self.lib.dk_peer_close(p)
        for p in self._owned:
            self.lib.dk_peer_free(p)
        self._mapped, self._owned = [], []

    def __del__(self):
        try:
            if self._owned or self._mapped:
                self.close()
        except Exception:
            pass


def _as_batch(x: torch.Tensor, K: int, max_batch: int, dev: torch.device) -> torch.Tensor:
    """x as [B, K] after the checks every layer makes before a launch: a
    contiguous fp16 [B, K] tensor on the layer's GPU with B <= max_batch.
    A tensor on another device would hand the kernels a pointer they cannot
    read, so it is refused here."""
    if x.dim() == 1:
        x = x.unsqueeze(0)
    if x.dim() != 2 or x.dtype != torch.float16 or not x.is_contiguous() or x.shape[1] != K:
        raise RuntimeError(f"x must be contiguous fp16 [B, {K}]")
    if x.device != dev:
        raise RuntimeError(f"x is on {x.device}, the layer's weights on {dev}")
    if x.shape[0] > max_batch:
        raise RuntimeError(f"batch {x.shape[0]} > max_batch {max_batch}")
    return x


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cfg(pdl: bool, await_all: bool = False) -> capi.GemvConfig:
    flags = (capi.DK_FLAG_PDL if pdl else 0) | (capi.DK_FLAG_SHARD_WAIT if await_all else 0)
    return capi.default_config(version=5, flags=flags)


# --------------------------------------------------------------------------
# Layers
# --------------------------------------------------------------------------

class RowParallelW4A16:
    """y[B, M] = x[B, K] . W^T with W's output rows split over the ranks.

    ``packed``/``scales`` are the FULL tensors; each local rank keeps its rows
    on the current GPU.  Call with the replicated x; returns the gathered
    fp16 y on every rank.  Ranks on their own GPUs with up to 8 batch rows
    exchange {value, call number} words and the GEMV gathers them into this
    layer's own output (valid until its next call); otherwise the rows are
    stored as fp16 into the peer buffers, marked by arrival slots, and y is a
    view of a buffer the call after next reuses.
    """

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, peers: PeerBuffers,
                 max_batch: int = 1, exchange: str = "fused", group=None):
        if exchange not in ("fused", "nccl"):
            raise ValueError(exchange)
        self.M, self.K = packed.shape[0], packed.shape[1] * 8
        self.peers, self.exchange, self.group = peers, exchange, group
        self.max_batch = int(max_batch)
        if 8 * self.max_batch * self.M > peers.nbytes:
            raise ValueError("peer buffers too small for [max_batch, M] 64-bit words")
        dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        self.shards = {}
        for r in peers.local_ranks():
            p, s, row0 = slice_rows(packed, scales, peers.world, r)
            # own copies, so the caller's full tensors can be freed
            self.shards[r] = (p.to(dev).clone(), s.to(dev).clone(), row0)
        self.out = torch.empty((self.max_batch, self.M), dtype=torch.float16, device=dev)

    def __call__(self, x: torch.Tensor, pdl: bool = False) -> torch.Tensor:
        x = _as_batch(x, self.K, self.max_batch, self.dev)
        B = x.shape[0]
        if self.exchange == "nccl":
            return self._nccl(x)
        lib, st = self.peers.lib, _stream()
        which = self.peers.begin()
        r0 = next(iter(self.shards))
        y = self.peers.view(r0, which, (B, self.M), torch.float16)
        if self.peers.world == 1 and not self.peers.emulated:  # nothing to exchange
            p, s, _ = self.shards[r0]
            _check(capi.gemv(p.data_ptr(), s.data_ptr(), x.data_ptr(), y.data_ptr(), self.M,
                             self.K, B, _cfg(pdl), 0, 0, st), "dk_w4a16_gemv")
            return y
        # Ranks on their own GPUs wait inside the kernel; emulated ranks
        # sharing this GPU's stream wait after all of them have run.
        inline = not self.peers.emulated
        if inline and B <= 8:
            group = self.peers.group(r0, which)
            p, s, row0 = self.shards[r0]
            _check(lib.dk_w4a16_gemv_rowshard_gather(p.data_ptr(), s.data_ptr(), x.data_ptr(),
                                                     p.shape[0], row0, self.M, self.K, B,
                                                     ctypes.byref(group),
                                                     self.out[:B].data_ptr(),
                                                     ctypes.byref(_cfg(pdl)), st),
                   "dk_w4a16_gemv_rowshard_gather")
            return self.out[:B]
        cfg = _cfg(pdl, await_all=inline)
        groups = {r: self.peers.group(r, which) for r in self.shards}
        for r, (p, s, row0) in self.shards.items():
            _check(lib.dk_w4a16_gemv_rowshard(p.data_ptr(), s.data_ptr(), x.data_ptr(),
                                              p.shape[0], row0, self.M, self.K, B,
                                              ctypes.byref(groups[r]), ctypes.byref(cfg), st),
                   "dk_w4a16_gemv_rowshard")
        if not inline:
            for r in self.shards:
                _check(lib.dk_shard_wait(ctypes.byref(groups[r]), st), "dk_shard_wait")
        return y

    def _nccl(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        from . import gemv

        if self.peers.emulated:
            raise RuntimeError("the NCCL exchange needs one process per rank")
        p, s, _ = self.shards[self.peers.rank]
        y_r = gemv(p, s, x)
        world = self.peers.world
        if world == 1:
            return y_r
        if self.M % world:
            raise RuntimeError("the NCCL exchange needs M divisible by the world size")
        out = torch.empty((world,) + tuple(y_r.shape), dtype=y_r.dtype, device=y_r.device)
        dist.all_gather_into_tensor(out, y_r.contiguous(), group=self.group)
        return out.permute(1, 0, 2).reshape(x.shape[0], self.M)


class KParallelW4A16:
    """y[B, M] = x[B, K] . W^T with W's reduction split over the ranks.

    Each local rank keeps its group-aligned K slice as contiguous tensors on
    the current GPU; every rank returns the same fp16 y = fp16(sum over ranks,
    in rank order, of the fp32 partials).
    """

    def __init__(self, packed: torch.Tensor, scales: torch.Tensor, peers: PeerBuffers,
                 max_batch: int = 1, exchange: str = "fused", group=None):
        if exchange not in ("fused", "nccl"):
            raise ValueError(exchange)
        self.M, self.K = packed.shape[0], packed.shape[1] * 8
        self.peers, self.exchange, self.group = peers, exchange, group
        self.max_batch = int(max_batch)
        if 8 * peers.world * self.max_batch * self.M > peers.nbytes:
            raise ValueError("peer buffers too small for [world, max_batch, M] 64-bit words")
        dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        self.shards = {}
        for r in peers.local_ranks():
            p, s, k0 = slice_k(packed, scales, peers.world, r)
            self.shards[r] = (p.to(dev), s.to(dev), k0)
        self.out = {r: torch.empty((self.max_batch, self.M), dtype=torch.float16, device=dev)
                    for r in self.shards}

    def __call__(self, x: torch.Tensor, pdl: bool = False) -> torch.Tensor:
        x = _as_batch(x, self.K, self.max_batch, self.dev)
        B = x.shape[0]
        if self.exchange == "nccl":
            return self._nccl(x)
        lib, st = self.peers.lib, _stream()
        r0 = next(iter(self.shards))
        if self.peers.world == 1 and not self.peers.emulated:  # nothing to exchange
            p, s, _ = self.shards[r0]
            _check(capi.gemv(p.data_ptr(), s.data_ptr(), x.data_ptr(), self.out[r0].data_ptr(),
                             self.M, self.K, B, _cfg(pdl), 0, 0, st), "dk_w4a16_gemv")
            return self.out[r0][:B]
        inline = not self.peers.emulated
        cfg = _cfg(pdl, await_all=inline)
        which = self.peers.begin()
        groups = {r: self.peers.group(r, which) for r in self.shards}
        for r, (p, s, k0) in self.shards.items():
            self._kshard(lib, p, s, x.data_ptr() + 2 * k0, self.K, B, groups[r], cfg, st, r,
                         inline)
        if not inline:
            self._reduce(lib, groups, B, st)
        return self.out[r0][:B]

    def _kshard(self, lib, p, s, x_ptr, ldx, B, group, cfg, st, r, inline):
        """Ranks on their own GPUs: the GEMV sums the world's partials itself
        (dk_w4a16_gemv_kshard_sum); emulated ranks sharing one GPU store their
        partials and are summed afterwards (dk_shard_reduce)."""
        if inline:
            _check(lib.dk_w4a16_gemv_kshard_sum(p.data_ptr(), s.data_ptr(), x_ptr, ldx, self.M,
                                                p.shape[1] * 8, B, ctypes.byref(group),
                                                self.out[r][:B].data_ptr(), ctypes.byref(cfg),
                                                st), "dk_w4a16_gemv_kshard_sum")
        else:
            _check(lib.dk_w4a16_gemv_kshard(p.data_ptr(), s.data_ptr(), x_ptr, ldx, self.M,
                                            p.shape[1] * 8, B, ctypes.byref(group),
                                            ctypes.byref(cfg), st), "dk_w4a16_gemv_kshard")

    def _reduce(self, lib, groups, B, st):
        for r in self.shards:
            _check(lib.dk_shard_reduce(ctypes.byref(groups[r]), self.M, B,
                                       self.out[r][:B].data_ptr(), 0, st), "dk_shard_reduce")

    def forward_local(self, xs: dict, pdl: bool = False) -> torch.Tensor:
        """Like ``__call__``, but each local rank r brings only its own K
        slice of x: ``xs[r]`` contiguous fp16 [B, kn_r] (a tensor-parallel
        layer's local activations).  Same result as ``__call__`` on the full
        x, bit for bit."""
        if sorted(xs) != sorted(self.shards):
            raise RuntimeError(f"expected inputs for ranks {sorted(self.shards)}")
        B = None
        for r, x in xs.items():
            kn = self.shards[r][0].shape[1] * 8
            if x.dtype != torch.float16 or not x.is_contiguous() or x.dim() != 2 or x.shape[1] != kn:
                raise RuntimeError(f"rank {r}: x must be contiguous fp16 [B, {kn}]")
            if x.device != self.dev:
                raise RuntimeError(f"rank {r}: x is on {x.device}, the layer's weights on {self.dev}")
            if B is not None and x.shape[0] != B:
                raise RuntimeError("every rank's x must have the same batch")
            B = x.shape[0]
        if B > self.max_batch:
            raise RuntimeError(f"batch {B} > max_batch {self.max_batch}")
        if self.exchange == "nccl":
            return self._nccl_local(xs[self.peers.rank])
        lib, st = self.peers.lib, _stream()
        r0 = next(iter(self.shards))
        if self.peers.world == 1 and not self.peers.emulated:
            p, s, _ = self.shards[r0]
            _check(capi.gemv(p.data_ptr(), s.data_ptr(), xs[r0].data_ptr(),
                             self.out[r0].data_ptr(), self.M, self.K, B, _cfg(pdl), 0, 0, st),
                   "dk_w4a16_gemv")
            return self.out[r0][:B]
        inline = not self.peers.emulated
        cfg = _cfg(pdl, await_all=inline)
        which = self.peers.begin()
        groups = {r: self.peers.group(r, which) for r in self.shards}
        for r, (p, s, _) in self.shards.items():
            kn = p.shape[1] * 8
            self._kshard(lib, p, s, xs[r].data_ptr(), kn, B, groups[r], cfg, st, r, inline)
        if not inline:
            self._reduce(lib, groups, B, st)
        return self.out[r0][:B]

    def _nccl_local(self, xs: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        if self.peers.emulated:
            raise RuntimeError("the NCCL exchange needs one process per rank")
        p, s, _ = self.shards[self.peers.rank]
        B, kn = xs.shape[0], p.shape[1] * 8
        y32 = torch.empty((B, self.M), dtype=torch.float32, device=xs.device)
        cfg = capi.default_config(version=5, flags=capi.DK_FLAG_F32_OUT)
        _check(capi.gemv(p.data_ptr(), s.data_ptr(), xs.data_ptr(), y32.data_ptr(), self.M, kn,
                         B, cfg, 0, 0, _stream()), "dk_w4a16_gemv")
        if self.peers.world > 1:
            dist.all_reduce(y32, group=self.group)
        return y32.half()

    def _nccl(self, x: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        if self.peers.emulated:
            raise RuntimeError("the NCCL exchange needs one process per rank")
        p, s, k0 = self.shards[self.peers.rank]
        B = x.shape[0]
        kn = p.shape[1] * 8
        xs = x[:, k0:k0 + kn].contiguous()
        y32 = torch.empty((B, self.M), dtype=torch.float32, device=x.device)
        cfg = capi.default_config(version=5, flags=capi.DK_FLAG_F32_OUT)
        _check(capi.gemv(p.data_ptr(), s.data_ptr(), xs.data_ptr(), y32.data_ptr(), self.M, kn,
                         B, cfg, 0, 0, _stream()), "dk_w4a16_gemv")
        if self.peers.world > 1:
            dist.all_reduce(y32, group=self.group)
        return y32.half()


# --------------------------------------------------------------------------
# Tensor-parallel decoder-layer projections (one exchange per block)
# --------------------------------------------------------------------------

def split_dim(n: int, world: int, rank: int) -> tuple[int, int]:
    """Tensor-parallel split of an inner dimension -- attention heads of 128
    (the quantization group) or a gated MLP's intermediate size: whole
    128-wide blocks, balanced.  It is ``k_range``, so rank r's row-parallel
    output slice is exactly the K slice of the next projection it owns."""
    return k_range(n, world, rank)


def _rows(packed: torch.Tensor, scales: torch.Tensor, r0: int, n: int, dev) -> tuple:
    return packed[r0:r0 + n].to(dev).clone(), scales[r0:r0 + n].to(dev).clone()


class TensorParallelMLP:
    """Gated MLP ``down(silu(gate(x)) * up(x))`` across the ranks in the
    tensor-parallel layout: gate and up are split by output rows and run as
    one SiLU-mul GEMV pair per rank with no exchange (rank r's slice of h is
    exactly the K slice of ``down`` it owns); ``down`` is K-parallel with the
    fused reduction.  One exchange per call.  Every rank returns the same y:
    fp16 of the rank-ordered sum of the fp32 partials of ``down`` over h's
    slices, where h = ``gemv_silu_mul(gate, up, x)`` (row slices are
    independent, so each rank's h slice has the unsharded bits).

    ``gate``, ``up``, ``down``: ``(packed, scales)``; gate/up [I, K], down
    [M, I], I a multiple of 128.
    """

    def __init__(self, gate, up, down, peers: PeerBuffers, max_batch: int = 1,
                 exchange: str = "fused", group=None):
        (pg, sg), (pu, su), (pd, sd) = gate, up, down
        if pu.shape != pg.shape or su.shape != sg.shape:
            raise ValueError("gate and up must have the same shape")
        self.I, self.K = pg.shape[0], pg.shape[1] * 8
        if pd.shape[1] * 8 != self.I:
            raise ValueError("down's K must equal gate/up's rows")
        self.M, self.peers, self.max_batch = pd.shape[0], peers, int(max_batch)
        if self.I // GROUP_SIZE < peers.world:
            raise ValueError("fewer 128-wide blocks of the intermediate size than ranks")
        dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        self.gu, self.h = {}, {}
        for r in peers.local_ranks():
            i0, n = split_dim(self.I, peers.world, r)
            self.gu[r] = _rows(pg, sg, i0, n, dev) + _rows(pu, su, i0, n, dev)
            self.h[r] = torch.empty((self.max_batch, n), dtype=torch.float16, device=dev)
        self.down = KParallelW4A16(pd, sd, peers, max_batch=max_batch, exchange=exchange,
                                   group=group)

    def __call__(self, x: torch.Tensor, pdl: bool = False) -> torch.Tensor:
        x = _as_batch(x, self.K, self.max_batch, self.dev)
        B = x.shape[0]
        cfg, st = _cfg(pdl), _stream()
        for r, (pg, sg, pu, su) in self.gu.items():
            _check(capi.gemv_silu_mul(pg.data_ptr(), sg.data_ptr(), pu.data_ptr(), su.data_ptr(),
                                      x.data_ptr(), self.h[r].data_ptr(), pg.shape[0], self.K, B,
                                      cfg, st), "dk_w4a16_gemv_silu_mul")
        return self.down.forward_local({r: self.h[r][:B] for r in self.gu}, pdl=pdl)


class TensorParallelAttentionProj:
    """An attention block's projections across the ranks, split by heads
    (128 wide, the quantization group): q/k/v row-parallel as one
    multi-matrix GEMV per rank with no exchange, o K-parallel over the same
    head split with the fused reduction.  One exchange per call.

    Attention itself is outside this library: ``__call__(x, attn=None)``
    takes a callable ``attn(rank, q, k, v) -> out`` returning the rank's
    attention output slice (fp16 [B, q rows of the rank]); without one, the
    rank's q slice -- the same shape -- stands in for it.
    """

    def __init__(self, q, k, v, o, peers: PeerBuffers, max_batch: int = 1,
                 exchange: str = "fused", group=None):
        (pq, sq), (pk, sk), (pv, sv), (po, so) = q, k, v, o
        self.K = pq.shape[1] * 8
        if pk.shape[1] * 8 != self.K or pv.shape[1] * 8 != self.K:
            raise ValueError("q, k, v must share K")
        if pk.shape != pv.shape:
            raise ValueError("k and v must have the same shape")
        self.Q, self.KV = pq.shape[0], pk.shape[0]
        if po.shape[1] * 8 != self.Q:
            raise ValueError("o's K must equal q's rows")
        self.M, self.peers, self.max_batch = po.shape[0], peers, int(max_batch)
        if min(self.Q, self.KV) // GROUP_SIZE < peers.world:
            raise ValueError("fewer 128-wide heads than ranks")
        dev = self.dev = torch.device("cuda", torch.cuda.current_device())
        self.qkv, self.outs = {}, {}
        for r in peers.local_ranks():
            q0, nq = split_dim(self.Q, peers.world, r)
            k0, nk = split_dim(self.KV, peers.world, r)
            self.qkv[r] = (_rows(pq, sq, q0, nq, dev), _rows(pk, sk, k0, nk, dev),
                           _rows(pv, sv, k0, nk, dev))
            self.outs[r] = tuple(torch.empty((self.max_batch, n), dtype=torch.float16, device=dev)
                                 for n in (nq, nk, nk))
        self.o = KParallelW4A16(po, so, peers, max_batch=max_batch, exchange=exchange,
                                group=group)

    def __call__(self, x: torch.Tensor, attn=None, pdl: bool = False) -> torch.Tensor:
        x = _as_batch(x, self.K, self.max_batch, self.dev)
        B = x.shape[0]
        cfg, st = _cfg(pdl), _stream()
        att = {}
        for r, mats in self.qkv.items():
            ys = self.outs[r]
            _check(capi.gemv_multi([p.data_ptr() for p, _ in mats], [s.data_ptr() for _, s in mats],
                                   [p.shape[0] for p, _ in mats], [y.data_ptr() for y in ys],
                                   x.data_ptr(), self.K, B, cfg, st), "dk_w4a16_gemv_multi")
            q, k, v = (y[:B] for y in ys)
            att[r] = q if attn is None else attn(r, q, k, v)
        return self.o.forward_local(att, pdl=pdl)

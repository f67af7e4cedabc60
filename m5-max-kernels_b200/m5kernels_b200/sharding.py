"""Multi-GPU host logic: token sharding, column-parallel output gather, timing.

The projection path shards by token rows with no collective: per-token
scales and row statistics never leave a row, weights are replicated, so each
rank quantizes and multiplies its own contiguous block of rows.  The optional
column-parallel variant (FFN-up: each rank holds N/g output channels of W)
ends with one all-gather of the BF16 output shards: `gather_columns` is that
step with NCCL (the baseline), and `ColumnParallelGather` fuses it into the
GEMM -- the epilogue stores every output tile into all ranks' [M, N] buffers
over NVLink (CUDA-IPC peer mappings, plain 16-byte peer stores), ordered by
two one-element all-reduces on the stream (no device-side waits on peers).

All functions take an optional process group and work with any
torch.distributed backend (NCCL over NVLink on the GPU box, gloo in tests).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist


def shard_rows(m: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) rows of rank `rank`; sizes differ by at most one
    (the first m % world ranks hold one extra row), e.g. 9914 rows on 8 ranks
    -> 1240 x 2 then 1239 x 6."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    if m < 0:
        raise ValueError("m must be non-negative")
    base, extra = divmod(m, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_columns(n: int, world: int, rank: int) -> tuple[int, int]:
    """Equal [start, stop) output-channel shard for the column-parallel variant."""
    if n % world:
        raise ValueError("N must be divisible by the number of ranks for column sharding")
    step = n // world
    return rank * step, (rank + 1) * step


def gather_columns(local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """[M, N/g] shards of every rank -> [M, N] (rank r's shard at columns r*N/g).

    One all_gather_into_tensor into a [g, M, N/g] buffer, then a permute; the
    receive buffer is laid out so the collective writes each shard
    contiguously.
    """
    m, ns = local.shape
    recv = torch.empty((world * m, ns), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(recv, local.contiguous(), group=group)
    return recv.view(world, m, ns).permute(1, 0, 2).reshape(m, world * ns)


def max_over_ranks(value: float, device=None, group=None) -> float:
    """Maximum of a per-rank scalar (e.g. a timed region in ms) over the group."""
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


class ColumnParallelGather:
    """Column-parallel projection with the all-gather fused into the GEMM epilogue.

    Every rank holds `out` [M, N] bf16 (allocated by the caller, alive for the
    lifetime of this object) and a shard of W with N / world output channels.
    On construction the ranks exchange CUDA IPC handles of their outputs (one
    all_gather of 72-byte records) and map the others' buffers.  `step` runs
    barrier -> m5b_gemm_allgather -> barrier on the current stream: the first
    barrier keeps a rank from overwriting a peer's output that the peer may
    still read, the second makes all shards visible everywhere.  Requires a
    process group whose collectives run on the GPU (NCCL) and world <= 8.
    """

    def __init__(self, out: torch.Tensor, group=None):
        from . import _lib

        if out.dim() != 2 or out.dtype != torch.bfloat16 or not out.is_contiguous():
            raise ValueError("out must be a contiguous bf16 [M, N] CUDA tensor")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise NotImplementedError("the fused all-gather supports up to 8 ranks")
        m, n = out.shape
        self.m, self.n = m, n
        self.col0, self.col1 = shard_columns(n, self.world, self.rank)
        self.out = out
        lib = _lib.lib()
        handle = ctypes.create_string_buffer(64)
        off = ctypes.c_int64(0)
        _lib.check(lib.m5b_ipc_export(_lib.ptr(out), handle, ctypes.byref(off)))
        rec = bytes(handle.raw) + int(off.value).to_bytes(8, "little", signed=True)
        mine = torch.tensor(list(rec), dtype=torch.uint8, device=out.device)
        allrec = [torch.empty_like(mine) for _ in range(self.world)]
        dist.all_gather(allrec, mine, group=group)
        self._mapped = []
        for r in range(self.world):
            if r == self.rank:
                continue
            raw = bytes(allrec[r].cpu().tolist())
            offset = int.from_bytes(raw[64:], "little", signed=True)
            p = ctypes.c_void_p(0)
            _lib.check(lib.m5b_ipc_import(raw[:64], offset, ctypes.byref(p)))
            self._mapped.append((p.value, offset))
        self._peers = (ctypes.c_void_p * 7)(*[p for p, _ in self._mapped])
        self._flag = torch.zeros(1, dtype=torch.float32, device=out.device)

    def barrier(self):
        dist.all_reduce(self._flag, group=self.group)

    def gemm(self, a, b_shard, a_scales=None, b_scales=None, mode="int8"):
        """This rank's shard of the projection, stored into every rank's output."""
        from . import _lib

        if b_shard.shape[0] != self.col1 - self.col0 or a.shape[0] != self.m:
            raise ValueError("shard shapes do not match the output")
        dev = _lib.require_cuda(a, b_shard, a_scales, b_scales, self.out)
        _lib.check(_lib.lib().m5b_gemm_allgather(
            _lib.ptr(a), _lib.ptr(b_shard), a.shape[0], b_shard.shape[0], a.shape[1],
            _lib.MODE[mode], _lib.ptr(a_scales), _lib.ptr(b_scales), _lib.ptr(self.out), self.n,
            self.col0, self._peers, len(self._mapped), _lib.stream_handle(dev)))

    def step(self, a, b_shard, a_scales=None, b_scales=None, mode="int8"):
        self.barrier()
        self.gemm(a, b_shard, a_scales, b_scales, mode)
        self.barrier()
        return self.out

    def close(self):
        """Unmap the peers' outputs (after every rank's last step has completed)."""
        from . import _lib

        torch.cuda.synchronize(self.out.device)
        for p, off in self._mapped:
            _lib.check(_lib.lib().m5b_ipc_release(ctypes.c_void_p(p), off))
        self._mapped = []

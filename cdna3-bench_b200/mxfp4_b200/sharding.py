"""Column-parallel (N-sharded) MXFP4 GEMM across the GPUs of one node.

The GEMM shards along N with no exchange on the data path: rank r owns the weight columns
[n0, n1) of the layer (a multiple of the 128-row chunk), computes Y_r = A @ dequant(B_r) with
the single-GPU kernels, and -- only when the caller wants the full [M, N] output on every
rank -- one all-gather joins the slices.  A is replicated.

These helpers hold the host-side logic (slice bounds, weight slicing, output assembly) so that
it is testable on CPU with the gloo backend; the compute call is the library's own GEMM.
"""

from __future__ import annotations

import torch

CHUNK_ROWS = 128  # weight rows per prepacked chunk; slices are multiples of this


def column_slice(N: int, world: int, rank: int, tile: int = CHUNK_ROWS) -> tuple[int, int]:
    """[n0, n1) of rank `rank`: whole tiles dealt out as evenly as possible, low ranks first.

    Raises ValueError when N is not a multiple of the tile or there are fewer tiles than ranks.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if N % tile:
        raise ValueError(f"N={N} is not a multiple of the {tile}-column tile")
    tiles = N // tile
    if tiles < world:
        raise ValueError(f"N={N} has {tiles} tiles, fewer than {world} ranks")
    base, extra = divmod(tiles, world)
    t0 = rank * base + min(rank, extra)
    t1 = t0 + base + (1 if rank < extra else 0)
    return t0 * tile, t1 * tile


def shard_reference_weights(B_packed, B_scales, world: int, rank: int):
    """This rank's columns of reference-layout weights ([K/2, N] and [K/32, N])."""
    n0, n1 = column_slice(B_packed.shape[1], world, rank)
    return B_packed[:, n0:n1].contiguous(), B_scales[:, n0:n1].contiguous()


def assemble(slices: list[torch.Tensor], N: int) -> torch.Tensor:
    """Join per-rank outputs [M, n1 - n0] (rank order) into [M, N]."""
    out = torch.cat(slices, dim=1)
    if out.shape[1] != N:
        raise ValueError(f"slices cover {out.shape[1]} columns, expected {N}")
    return out


def all_gather_columns(Y_local: torch.Tensor, N: int, group=None) -> torch.Tensor:
    """All-gather every rank's [M, n_r] slice and return the full [M, N] on each rank.

    With equal slices (N / 128 divisible by the world size, the usual case) this is one
    all_gather_into_tensor into [world * M, n] plus a local permute; unequal slices fall back to
    all_gather of padded slices.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    M, n = Y_local.shape
    sizes = [column_slice(N, world, r)[1] - column_slice(N, world, r)[0] for r in range(world)]
    n_max = max(sizes)
    if all(s == n_max for s in sizes):
        buf = torch.empty((world * M, n), dtype=Y_local.dtype, device=Y_local.device)
        dist.all_gather_into_tensor(buf, Y_local.contiguous(), group=group)
        return buf.view(world, M, n).permute(1, 0, 2).reshape(M, N)
    pad = torch.zeros((M, n_max), dtype=Y_local.dtype, device=Y_local.device)
    pad[:, :n] = Y_local
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad, group=group)
    return assemble([p[:, :s] for p, s in zip(parts, sizes)], N)


class ColumnParallelMXFP4:
    """One rank's share of an N-sharded MXFP4 linear layer.

    `B_packed` / `B_scales` are the FULL reference-layout weights (each rank slices its own
    columns) or, with `pre_sliced=True`, this rank's slice already.
    """

    def __init__(self, B_packed, B_scales, N: int, world: int, rank: int, pre_sliced: bool = False):
        from . import kernels as kk

        self.N, self.world, self.rank = N, world, rank
        self.n0, self.n1 = column_slice(N, world, rank)
        if not pre_sliced:
            B_packed, B_scales = shard_reference_weights(B_packed, B_scales, world, rank)
        self.weight = kk.prepack_b200(B_packed, B_scales)

    def local(self, A: torch.Tensor, out_dtype=torch.bfloat16) -> torch.Tensor:
        """This rank's output columns [M, n1 - n0]."""
        from . import kernels as kk

        return kk.gemm(A, self.weight, out_dtype=out_dtype)

    def forward(self, A: torch.Tensor, gather: bool = True, group=None, out_dtype=torch.bfloat16):
        Y = self.local(A, out_dtype)
        return all_gather_columns(Y, self.N, group) if gather and self.world > 1 else Y


class PeerOutput:
    """A full [M, N] output buffer on every GPU of the group, each mapped into every other
    process (CUDA IPC), so that a fused GEMM + all-gather can store its tiles straight into
    all of them over NVLink.  Collective: every rank constructs it with the same arguments."""

    def __init__(self, M: int, N: int, dtype=torch.bfloat16, group=None, device=None):
        import torch.distributed as dist

        from . import kernels as kk

        self.M, self.N, self.dtype, self.group = M, N, dtype, group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-gather writes to at most 8 GPUs")
        self.buffer = torch.empty((M, N), dtype=dtype, device=device or torch.cuda.current_device())
        handle, off = kk.ipc_export(self.buffer)
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (handle, off), group=group)
        self._opened = []
        self.ptrs = []
        for r, (h, o) in enumerate(everyone):
            if r == self.rank:
                self.ptrs.append(self.buffer.data_ptr())
            else:
                p = kk.ipc_open(h, o)
                self._opened.append((p, o))
                self.ptrs.append(p)
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.buffer.device)

    def close(self):
        from . import kernels as kk

        for p, o in self._opened:
            kk.ipc_close(p, o)
        self._opened = []

    def push(self, n0: int, n1: int, streams=None):
        """Copy this GPU's columns [n0, n1) of `buffer` into every peer's buffer with the copy
        engines (one pitched copy per peer; `streams`: one CUDA stream per peer, else the current
        stream).  No SM takes part, so the copies overlap kernels on other streams; `sync` after
        them (ordered after the copies on every GPU) makes them visible to the peers."""
        from . import kernels as kk

        esz = self.buffer.element_size()
        pitch = self.N * esz
        src = self.ptrs[self.rank] + n0 * esz
        peers = [r for r in range(self.world) if r != self.rank]
        for i, r in enumerate(peers):
            kk.copy_columns(self.ptrs[r] + n0 * esz, pitch, src, pitch, (n1 - n0) * esz, self.M,
                            stream=streams[i] if streams else None)

    def sync(self):
        """Order this GPU's later work after every peer's stores into `buffer` (a stream-ordered
        all-reduce of one int: it completes only after every rank's preceding kernels)."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)


def forward_fused(layer: "ColumnParallelMXFP4", A: torch.Tensor, out: PeerOutput) -> torch.Tensor:
    """Column-parallel GEMM with the all-gather fused into the epilogue: every output tile is
    stored into all GPUs' `out.buffer` as it is produced, then one tiny collective orders the
    reads.  Returns this GPU's full [M, N] output."""
    from . import kernels as kk

    if out.dtype not in (torch.bfloat16, torch.float32) or out.N != layer.N or out.M != A.shape[0]:
        raise ValueError("PeerOutput shape/dtype does not match the layer and A")
    kk.gemm_allgather(A, layer.weight, out.ptrs, layer.n0, layer.N, out_dtype=out.dtype)
    out.sync()
    return out.buffer


def forward_copy_engine(layer: "ColumnParallelMXFP4", A: torch.Tensor, out: PeerOutput) -> torch.Tensor:
    """Column-parallel GEMM whose slice is written straight into this GPU's full output and then
    pushed to every peer by the copy engines (NVLink, no SMs), then one tiny collective orders
    the reads.  Returns this GPU's full [M, N] output."""
    from . import kernels as kk

    if out.dtype not in (torch.bfloat16, torch.float32) or out.N != layer.N or out.M != A.shape[0]:
        raise ValueError("PeerOutput shape/dtype does not match the layer and A")
    kk.gemm_allgather(A, layer.weight, [out.ptrs[out.rank]], layer.n0, layer.N, out_dtype=out.dtype)
    out.push(layer.n0, layer.n1)
    out.sync()
    return out.buffer

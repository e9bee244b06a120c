"""N-sharded quantized matmul over the ranks of one node.

Every output column n of ``cpu_quant_matmul`` (one weight row) is independent
of the others (src/kernels_quant.cpp:390-397), so the weight rows split
across G ranks: rank r holds rows [r*N/G, (r+1)*N/G) and computes
Y[:, shard] for all M activation rows, an all-gather collects the G blocks
[G][M][N/G], and one CUDA re-layout (``pxq.gather_shards``) produces the
caller's row-major Y[M][N] (``output[c*rows + r]``, src/kernels_quant.cpp:398).
Each rank quantizes the replicated activation itself; the quantized bytes
are identical on every rank, so the gathered Y is bit-identical to a 1-GPU
run.

Two ways to assemble Y: ``sharded_matmul`` (local matmul, NCCL all-gather,
re-layout) and ``sharded_matmul_p2p`` (one kernel per rank: the GEMM epilogue
stores each output tile straight into every rank's Y through CUDA IPC
mappings over NVLink, so the transfer overlaps the next tiles' math and no
all-gather or re-layout pass remains).  Rank synchronisation goes through
``torch.distributed`` (NCCL on GPUs).
"""
from __future__ import annotations


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of ``rank``'s contiguous shard of ``rows``.

    The split is even: all-gather needs equal blocks, so ``rows`` must be a
    multiple of ``world`` (BASELINE's sharded shapes are: 12288/8 = 1536).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if rows % world:
        raise ValueError(f"{rows} weight rows do not split evenly over {world} ranks")
    per = rows // world
    return rank * per, per


def gathered_layout(gathered, world: int, columns: int, shard: int):
    """The [G][M][N/G] all-gather result viewed as row-major [M][N], as a
    strided view (no copy); ``pxq.gather_shards`` writes the same layout
    densely on the GPU."""
    return gathered.view(world, columns, shard).permute(1, 0, 2).reshape(columns, world * shard)


class ShardedWeight:
    """This rank's shard of a GGUF weight [rows][weight_bytes(inner)], uploaded
    to the current device.  ``weights`` holds the full tensor's bytes (host
    numpy or device tensor); only the shard's rows are uploaded."""

    def __init__(self, weights, wtype: int, inner: int, rows: int, world: int, rank: int):
        from . import pxq

        self.world, self.rank, self.rows = world, rank, rows
        self.first, self.count = shard_rows(rows, world, rank)
        self.weight = pxq.Weight(weights[self.first:self.first + self.count], wtype, inner, self.count)

    def release(self) -> None:
        self.weight.release()


def sharded_matmul(sw: ShardedWeight, x, out=None, group=None, path: str = "auto", scratch=None):
    """Y[M][N] = X * W^T with W's rows split over the process group.

    ``x``: fp32 [M][K] on this rank's device (replicated on every rank).
    ``scratch``: optional (local block [M][N/G], gather buffer [G*M*N/G])
    reused across calls.  Every rank must call it with the same shapes.
    """
    import torch
    import torch.distributed as dist

    from . import pxq

    M = x.shape[0]
    G, Ns = sw.world, sw.count
    if scratch is None:
        scratch = (torch.empty((M, Ns), dtype=torch.float32, device=x.device),
                   torch.empty((G * M * Ns,), dtype=torch.float32, device=x.device))
    local, gathered = scratch
    pxq.matmul(sw.weight, x, out=local, path=path)
    if out is None:
        out = torch.empty((M, G * Ns), dtype=torch.float32, device=x.device)
    if G == 1:
        out.copy_(local)
        return out
    dist.all_gather_into_tensor(gathered, local.view(-1), group=group)
    pxq.gather_shards(gathered, G, M, Ns, out=out)
    return out


class PeerOutput:
    """Y [columns][rows] on every rank of the group, each rank's buffer mapped
    into every other rank (CUDA IPC): the destinations of
    ``pxq.matmul_scatter``.  Collective: every rank constructs and closes it
    together."""

    def __init__(self, columns: int, rows: int, group=None):
        import torch
        import torch.distributed as dist

        from . import pxq

        self.group = group
        self.buf = pxq.IpcBuffer(columns, rows)
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        handles = [None] * world
        dist.all_gather_object(handles, self.buf.handle, group=group)
        self.peers = []
        self.ptrs = [self.buf.ptr]  # this rank's buffer first, then the others' (the scatter's order)
        for r, h in enumerate(handles):
            if r != rank:
                peer = pxq.IpcPeer(h)
                self.peers.append(peer)
                self.ptrs.append(peer.ptr)
        self.tensor = self.buf.tensor
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.tensor.device)

    def sync(self) -> None:
        """Device-ordered barrier of the group (a one-element NCCL all-reduce)."""
        import torch.distributed as dist

        dist.all_reduce(self._flag, group=self.group)

    def close(self) -> None:
        import torch
        import torch.distributed as dist

        torch.cuda.synchronize()
        for peer in self.peers:
            peer.close()
        self.peers = []
        dist.barrier(group=self.group)  # every mapping of this buffer is closed before it is freed
        self.tensor = None
        self.buf.free()


def sharded_matmul_p2p(sw: ShardedWeight, x, out: PeerOutput, sync_before: bool = True):
    """Y[M][N] = X * W^T with W's rows split over the group, each rank's GEMM
    writing its columns into every rank's ``out`` (M > 8: the GEMM path).
    ``sync_before``: wait until every rank is done with the previous contents
    of its Y before anyone overwrites it.  Returns this rank's Y (a view of
    ``out``), complete once the call returns in stream order."""
    from . import pxq

    if sync_before:
        out.sync()
    pxq.matmul_scatter(sw.weight, x, out.ptrs, ldy=sw.rows, col_offset=sw.first)
    out.sync()  # every rank's stores into this Y have landed
    return out.tensor

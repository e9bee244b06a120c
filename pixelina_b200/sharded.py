"""N-sharded quantized matmul over the ranks of one node.

Every output column n of ``cpu_quant_matmul`` (one weight row) is independent
of the others (src/kernels_quant.cpp:390-397), so the weight rows split
across G ranks: rank r holds rows [r*N/G, (r+1)*N/G) and computes
Y[:, shard] for all M activation rows, an all-gather collects the G blocks
[G][M][N/G], and one CUDA re-layout (``pxq.gather_shards``) produces the
caller's row-major Y[M][N] (``output[c*rows + r]``, src/kernels_quant.cpp:398).
Each rank quantizes the replicated activation itself; the quantized bytes
are identical on every rank, so the gathered Y is bit-identical to a 1-GPU
run.  Collectives go through ``torch.distributed`` (NCCL on GPUs); this
module adds no compute path of its own.
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

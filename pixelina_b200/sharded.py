"""N-sharded quantized matmul over the ranks of one node (Python side of the
C ABI's pxq_comm_* / pxq_sharded_* entry points, include/pxq.h).

Every output column n of ``cpu_quant_matmul`` (one weight row) is independent
of the others (src/kernels_quant.cpp:390-397), so the weight rows split
across G ranks: rank r holds rows [r*N/G, (r+1)*N/G) and computes
Y[:, shard] for all M activation rows.  libpxq assembles the row-major
Y[M][N] (``output[c*rows + r]``, src/kernels_quant.cpp:398) on every rank,
either fused -- each rank's GEMM epilogue stores its columns into every
rank's output over NVLink (``ShardedOutput``) -- or through an NCCL
all-gather and one re-layout kernel.  Each rank quantizes the replicated
activation itself; the quantized bytes are identical on every rank, so Y is
bit-identical to a 1-GPU run.

The communicator (NCCL inside libpxq) needs its 128-byte id on every rank;
``Comm`` takes it from rank 0 through a ``torch.distributed`` broadcast, or
from the caller.  Every wait is bounded by the communicator's timeout.
"""
from __future__ import annotations

import ctypes as C

COMM_ID_BYTES = 128


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of ``rank``'s contiguous shard of ``rows``.

    The split is even (every rank's block has the same shape), so ``rows``
    must be a multiple of ``world`` (BASELINE's sharded shapes are: 12288/8 = 1536).
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if rows % world:
        raise ValueError(f"{rows} weight rows do not split evenly over {world} ranks")
    per = rows // world
    return rank * per, per


def gathered_layout(gathered, world: int, columns: int, shard: int):
    """The [G][M][N/G] all-gather result viewed as row-major [M][N], as a
    strided view (no copy); ``pxq_gather_shards`` writes the same layout
    densely on the GPU."""
    return gathered.view(world, columns, shard).permute(1, 0, 2).reshape(columns, world * shard)


class Comm:
    """pxq_comm: this rank's member of a node-wide communicator.

    ``comm_id``: the id bytes from ``unique_id()`` on one rank; ``None`` takes
    it from rank 0 of the default ``torch.distributed`` group (collective)."""

    def __init__(self, world: int, rank: int, comm_id: bytes | None = None, timeout_ms: int = 60000):
        from . import pxq

        if comm_id is None:
            import torch.distributed as dist

            box = [unique_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            comm_id = box[0]
        buf = (C.c_uint8 * COMM_ID_BYTES).from_buffer_copy(comm_id)
        h = C.c_void_p()
        pxq._check(pxq.load().pxq_comm_init(C.cast(buf, C.c_void_p), world, rank, timeout_ms, C.byref(h)))
        self.handle, self.world, self.rank = h.value, world, rank

    def barrier(self) -> None:
        from . import pxq

        pxq._check(pxq.load().pxq_comm_barrier(C.c_void_p(self.handle)))

    def synchronize(self, stream=None) -> None:
        from . import pxq

        pxq._check(pxq.load().pxq_comm_synchronize(C.c_void_p(self.handle), pxq._stream_ptr(stream)))

    def close(self) -> None:
        from . import pxq

        if self.handle:
            pxq._check(pxq.load().pxq_comm_destroy(C.c_void_p(self.handle)))
            self.handle = None


def unique_id() -> bytes:
    from . import pxq

    buf = (C.c_uint8 * COMM_ID_BYTES)()
    pxq._check(pxq.load().pxq_comm_unique_id(C.cast(buf, C.c_void_p)))
    return bytes(buf)


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


class ShardedOutput:
    """pxq_sharded_output: Y [columns][rows] on every rank, mapped into every
    other rank (the fused path's destinations).  Collective to create and to
    close; ``tensor`` views this rank's buffer."""

    def __init__(self, comm: Comm, columns: int, rows: int):
        from . import pxq

        torch = pxq._torch()
        h, local = C.c_void_p(), C.c_void_p()
        pxq._check(pxq.load().pxq_sharded_output_create(C.c_void_p(comm.handle), columns, rows, C.byref(h), C.byref(local)))
        self.handle, self.comm = h.value, comm
        self.tensor = torch.as_tensor(pxq._CudaArray(local.value, (columns, rows)), device="cuda")

    def close(self) -> None:
        from . import pxq

        if self.handle:
            self.tensor = None
            pxq._check(pxq.load().pxq_sharded_output_destroy(C.c_void_p(self.handle)))
            self.handle = None


def sharded_matmul(comm: Comm, sw: ShardedWeight, x, out=None, stream=None):
    """Y[M][N] = X * W^T with W's rows split over the communicator.

    ``x``: fp32 [M][K] on this rank's device (replicated on every rank).
    ``out``: a ``ShardedOutput`` (fused path; returns its tensor) or a device
    tensor [M][N] (NCCL all-gather path) or ``None`` (a new tensor, all-gather
    path).  Queued on ``stream``; every rank makes the same calls."""
    from . import pxq

    torch = pxq._torch()
    x = x.contiguous()
    M = x.shape[0]
    lib = pxq.load()
    if isinstance(out, ShardedOutput):
        pxq._check(lib.pxq_sharded_matmul(C.c_void_p(comm.handle), sw.weight.handle, sw.count, pxq._ptr(x), M,
                                          C.c_void_p(out.handle), C.c_void_p(0), 0, pxq._stream_ptr(stream)))
        return out.tensor
    if out is None:
        out = torch.empty((M, sw.rows), dtype=torch.float32, device=x.device)
    pxq._check(lib.pxq_sharded_matmul(C.c_void_p(comm.handle), sw.weight.handle, sw.count, pxq._ptr(x), M, C.c_void_p(0),
                                      pxq._ptr(out), out.stride(0), pxq._stream_ptr(stream)))
    return out


def sharded_matmul_host_ptr(comm: Comm, sw: ShardedWeight, x_ptr: int, columns: int, inner: int, y_ptr: int) -> int:
    """pxq_sharded_matmul_host on raw host pointers (pinned or pageable):
    returns the status code; the full Y [columns][rows] lands in y_ptr."""
    from . import pxq

    return pxq.load().pxq_sharded_matmul_host(C.c_void_p(comm.handle), sw.weight.handle, sw.count, C.c_void_p(x_ptr), columns,
                                              inner, C.c_void_p(y_ptr))

"""N-sharded matmul host logic on two gloo ranks (CPU, no GPU).

Each rank takes its shard of the weight rows (pixelina_b200.sharded.shard_rows),
computes its [M][N/G] block with the oracle (the CPU checker stands in for the
GPU kernel here), all-gathers the blocks exactly as the GPU path does
(all_gather_into_tensor), and views them with sharded.gathered_layout, the
layout pxq.gather_shards produces on the GPU (tests/test_gpu_parity.py checks
that kernel against the same permute).  The gathered result must equal the
unsharded oracle result bit for bit: the split, the gather order and the
re-layout lose or reorder nothing.
"""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT

Q8_0, Q5_K = 8, 13


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, wtype: int, rows: int, inner: int, columns: int, out_q) -> None:
    import sys

    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist

    from oracle.oracle import Oracle
    from pixelina_b200 import sharded, synth

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = synth.weights_for(wtype, rows, inner, seed=11)  # same seed on every rank
        x = synth.activations(columns, inner, seed=12)
        first, count = sharded.shard_rows(rows, world, rank)
        ok, block = Oracle().quant_matmul(w[first:first + count], wtype, x, count)
        assert ok
        gathered = torch.empty(world * columns * count, dtype=torch.float32)
        dist.all_gather_into_tensor(gathered, torch.from_numpy(np.ascontiguousarray(block)).view(-1))
        y = sharded.gathered_layout(gathered, world, columns, count).contiguous().numpy()
        if rank == 0:
            ok_full, ref = Oracle().quant_matmul(w, wtype, x, rows)
            out_q.put((bool(ok_full), bool(np.array_equal(y.view(np.uint32), ref.view(np.uint32)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("wtype,rows,inner,columns", [(Q8_0, 96, 256, 5), (Q5_K, 64, 512, 3)])
def test_two_rank_shard_gather_matches_unsharded(wtype, rows, inner, columns):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, wtype, rows, inner, columns, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], f"rank exit codes {codes}"
    ok_full, equal = q.get(timeout=5)
    assert ok_full and equal


def test_shard_rows_partition():
    from pixelina_b200 import sharded

    for rows, world in ((12288, 8), (3840, 8), (96, 2), (18944, 4), (7, 1)):
        spans = [sharded.shard_rows(rows, world, r) for r in range(world)]
        assert spans[0][0] == 0 and sum(c for _, c in spans) == rows
        assert all(spans[i][0] + spans[i][1] == spans[i + 1][0] for i in range(world - 1))
        assert len({c for _, c in spans}) == 1  # equal blocks for the all-gather
    with pytest.raises(ValueError):
        sharded.shard_rows(100, 8, 0)
    with pytest.raises(ValueError):
        sharded.shard_rows(96, 2, 2)

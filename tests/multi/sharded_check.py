"""Run under torchrun (one rank per GPU): the N-sharded matmul through the C
ABI (pxq_comm_* / pxq_sharded_*) -- NCCL all-gather, and for GEMM shapes
also the fused path whose GEMM epilogue stores into every rank's output --
must give Y bit-identical to the single-GPU matmul of the whole weight, and
so must the host-buffer entry point.  Exit status 0 on success; rank 0
prints one line per check."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main() -> int:
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from pixelina_b200 import pxq, sharded, synth

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    failures = 0
    comm = None
    try:
        pxq.init(local)
        comm = sharded.Comm(world, rank, timeout_ms=60000)  # id from rank 0 over the gloo group

        def report(name, got, ref):
            nonlocal failures
            same = torch.equal(got.view(torch.int32), ref.view(torch.int32))
            failures += 0 if same else 1
            if rank == 0:
                print(f"{name}: {'bit-identical' if same else 'DIFFERENT'}", flush=True)

        for wtype, rows, inner, columns in ((8, 512, 1024, 300), (13, 256, 1024, 260), (14, 512, 512, 140),
                                           (13, 512, 3584, 4), (8, 256, 512, 1)):
            w = synth.weights_for(wtype, rows, inner, seed=rows)  # same bytes on every rank
            xh = synth.activations(columns, inner, seed=columns)
            x = torch.from_numpy(xh).cuda()
            W = pxq.Weight(w, wtype, inner, rows)
            ref = pxq.matmul(W, x)
            torch.cuda.synchronize()
            W.release()
            sw = sharded.ShardedWeight(w, wtype, inner, rows, world, rank)
            tag = f"type {wtype} [{rows}x{inner}] M={columns}"
            y = sharded.sharded_matmul(comm, sw, x)
            comm.synchronize()
            report(f"{tag} all-gather", y, ref)
            if columns > 8:  # the fused path runs on the GEMM
                out = sharded.ShardedOutput(comm, columns, rows)
                for _ in range(2):  # twice: the second call overwrites the first one's output
                    y2 = sharded.sharded_matmul(comm, sw, x, out=out)
                    comm.synchronize()
                report(f"{tag} fused P2P stores", y2.clone(), ref)
                out.close()
                yh = np.empty((columns, rows), dtype=np.float32)
                rc = sharded.sharded_matmul_host_ptr(comm, sw, xh.ctypes.data, columns, inner, yh.ctypes.data)
                failures += 0 if rc == 0 else 1
                report(f"{tag} host buffers", torch.from_numpy(yh).cuda(), ref)
            sw.release()
        flag = torch.tensor([failures])
        dist.all_reduce(flag)
        failures = int(flag.item())
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())

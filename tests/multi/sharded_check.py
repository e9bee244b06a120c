"""Run under torchrun (one rank per GPU): the N-sharded matmul -- NCCL
all-gather, and for the GEMM cases also the one-kernel P2P-store path -- must
give Y bit-identical to the single-GPU matmul of the whole weight.  Exit
status 0 on success; rank 0 prints one line per check."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main() -> int:
    import datetime

    import torch
    import torch.distributed as dist

    from pixelina_b200 import pxq, sharded, synth

    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    failures = 0
    try:
        pxq.init(local)
        for wtype, rows, inner, columns, path in ((8, 512, 1024, 300, "gemm"), (13, 256, 1024, 260, "gemm"),
                                                 (13, 512, 3584, 4, "matvec"), (8, 256, 512, 1, "matvec")):
            w = synth.weights_for(wtype, rows, inner, seed=rows)  # same bytes on every rank
            x = torch.from_numpy(synth.activations(columns, inner, seed=columns)).cuda()
            sw = sharded.ShardedWeight(w, wtype, inner, rows, world, rank)
            y = sharded.sharded_matmul(sw, x, path=path)
            torch.cuda.synchronize()
            y2 = None
            if path == "gemm":  # the one-kernel path: GEMM epilogue stores into every rank's Y
                po = sharded.PeerOutput(columns, rows)
                y2 = sharded.sharded_matmul_p2p(sw, x, po).clone()
                torch.cuda.synchronize()
                po.close()
            sw.release()
            if rank == 0:
                W = pxq.Weight(w, wtype, inner, rows)
                ref = pxq.matmul(W, x, path=path)
                torch.cuda.synchronize()
                W.release()
                same = torch.equal(y.view(torch.int32), ref.view(torch.int32))
                failures += 0 if same else 1
                print(f"type {wtype} [{rows}x{inner}] M={columns} {path}: {'bit-identical' if same else 'DIFFERENT'}",
                      flush=True)
                if y2 is not None:
                    same = torch.equal(y2.view(torch.int32), ref.view(torch.int32))
                    failures += 0 if same else 1
                    print(f"type {wtype} [{rows}x{inner}] M={columns} gemm, P2P stores: "
                          f"{'bit-identical' if same else 'DIFFERENT'}", flush=True)
        flag = torch.tensor([failures], device="cuda")
        dist.broadcast(flag, 0)
        failures = int(flag.item())
    finally:
        dist.destroy_process_group()
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())

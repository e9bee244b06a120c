"""The multi-GPU C ABI (pxq_comm_* / pxq_sharded_*) on one GPU.

A one-rank communicator runs both assembly paths of pxq_sharded_matmul (the
fused GEMM that stores into every rank's output, and the NCCL all-gather +
re-layout) and the host-buffer entry point; with one rank both must equal
the plain matmul bit for bit.  Failure detection: a communicator whose
second rank never joins must give up after its timeout with
PXQ_ERR_TIMEOUT (the wait is on the host; nothing waits on the GPU), and
an aborted communicator must refuse later calls.  Both run in child
processes with NVLS off, as every multi-rank test does."""
import os
import subprocess
import sys
import textwrap

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _run(code: str, timeout: int = 180):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run([sys.executable, "-c", textwrap.dedent(code)], cwd=ROOT, env=env, capture_output=True, text=True,
                         timeout=timeout)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    return res.stdout


def test_one_rank_sharded_paths_equal_plain_matmul():
    out = _run("""
        import sys, numpy as np, torch
        sys.path.insert(0, ".")
        from pixelina_b200 import pxq, sharded, synth
        pxq.init(0)
        comm = sharded.Comm(1, 0, comm_id=sharded.unique_id(), timeout_ms=30000)
        for wtype, rows, inner, columns in ((8, 384, 1024, 300), (13, 256, 512, 140), (14, 256, 512, 9)):
            w = synth.weights_for(wtype, rows, inner, seed=rows)
            xh = synth.activations(columns, inner, seed=columns)
            x = torch.from_numpy(xh).cuda()
            W = pxq.Weight(w, wtype, inner, rows)
            ref = pxq.matmul(W, x)
            sw = sharded.ShardedWeight(w, wtype, inner, rows, 1, 0)
            y1 = sharded.sharded_matmul(comm, sw, x)
            out = sharded.ShardedOutput(comm, columns, rows)
            y2 = sharded.sharded_matmul(comm, sw, x, out=out)
            comm.synchronize()
            yh = np.empty((columns, rows), dtype=np.float32)
            assert sharded.sharded_matmul_host_ptr(comm, sw, xh.ctypes.data, columns, inner, yh.ctypes.data) == 0
            for name, y in (("all-gather", y1), ("fused", y2), ("host", torch.from_numpy(yh).cuda())):
                assert torch.equal(y.view(torch.int32), ref.view(torch.int32)), (wtype, name)
            out.close()
            sw.release()
            W.release()
        comm.close()
        print("one-rank ok")
    """)
    assert "one-rank ok" in out


def test_missing_rank_times_out_and_aborts():
    out = _run("""
        import sys, time, ctypes as C
        sys.path.insert(0, ".")
        from pixelina_b200 import pxq, sharded
        pxq.init(0)
        lib = pxq.load()
        cid = (C.c_uint8 * 128).from_buffer_copy(sharded.unique_id())
        h = C.c_void_p()
        t0 = time.time()
        rc = lib.pxq_comm_init(C.cast(cid, C.c_void_p), 2, 0, 2000, C.byref(h))  # rank 1 never joins
        dt = time.time() - t0
        assert rc == pxq.ERR_TIMEOUT, (rc, pxq.last_error())
        assert "ms" in pxq.last_error() and 1.9 < dt < 30, dt
        assert not h.value
        # the GPU is still usable afterwards
        import torch
        assert float(torch.ones(4, device="cuda").sum()) == 4.0
        print("timeout ok", round(dt, 2))
    """)
    assert "timeout ok" in out

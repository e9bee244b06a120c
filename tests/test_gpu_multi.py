"""Multi-GPU (one node): the N-sharded matmul of the C ABI -- NCCL all-gather,
the fused P2P-store GEMM and the host-buffer entry point -- checked bit for
bit against the single-GPU result.  Needs at least two visible GPUs; with one
it is skipped (tests/test_gpu_comm.py runs the same entry points on a
one-rank communicator, tests/test_sharded_gloo.py the host logic on CPU)."""
import os
import socket
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_matmul_two_gpus_bit_identical():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}", os.path.join(ROOT, "tests", "multi", "sharded_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert res.stdout.count("bit-identical") == 11

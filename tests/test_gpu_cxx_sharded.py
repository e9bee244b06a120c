"""GPU: a C++ program drives the N-sharded C ABI (pxq_comm_init,
pxq_sharded_matmul_host) with one process per GPU -- two GPUs when the box
has them, else a one-rank communicator -- and every rank's whole output must
equal the single-GPU pxq_quant_matmul bit for bit.  NVLS stays off, as in
every multi-rank test."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cxx_sharded_matmul_bit_identical(tmp_path):
    import torch

    exe = str(tmp_path / "sharded_check")
    lib_dir = os.path.join(ROOT, "pixelina_b200")
    obj = str(tmp_path / "pxq_oracle.o")
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-c", os.path.join(ROOT, "oracle", "pxq_oracle.c"),
                    "-o", obj], check=True)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cxx", "sharded_check.cpp"), obj, "-L", lib_dir, "-lpxq",
                    f"-Wl,-rpath,{lib_dir}", "-lm", "-lpthread", "-o", exe], check=True)
    world = 2 if torch.cuda.device_count() >= 2 else 1
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    idf = str(tmp_path / "comm.id")
    procs = [subprocess.Popen([exe, str(world), str(r), idf], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True,
                              env=env) for r in range(world)]
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=180)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append((p.returncode, out))
    for r, (rc, out) in enumerate(outs):
        assert rc == 0, f"rank {r}: {out}"
        assert f"OK rank {r} of {world}" in out

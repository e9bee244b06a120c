"""The Q8_0 GEMM has five operand kinds (gemm_q8.cu): exact fp16 copies of
the quants with kind::f16 block-dot MMAs and the scale products from a one-hot
tensor-core MMA ("f16s", the default), the same on the int8 quants with
kind::i8 block dots ("i8s"), fp16 copies with the block scales applied on the
CUDA cores ("f16"), the int8 quants likewise ("i8"), and "f16" on CTA pairs
("pair").  The library picks one per process (PXQ_Q8_0_MMA, read once), and
for "f16s" and "i8s" a drain of eight 64-column warps (the default) or sixteen
32-column ones (PXQ_Q8_0_DRAIN=16).  The rest of the GPU suite runs the
default; this test reruns the GEMM parity files in a child process with each
choice, so all stay bit-exact in their block dots and within max-abs-rel 1e-3
of the oracle."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind,drain", [("f16", "8"), ("i8", "8"), ("f16s", "8"), ("pair", "8"), ("i8s", "8"),
                                        ("f16s", "16"), ("i8s", "16")])
def test_q8_0_gemm_parity_in_each_mma_kind(kind, drain):
    env = dict(os.environ, PXQ_Q8_0_MMA=kind, PXQ_Q8_0_DRAIN=drain)
    files = [os.path.join(ROOT, "tests", f) for f in ("test_gpu_parity.py", "test_gpu_baseline_shapes.py")]
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-k", "gemm or matmul or q6_K_golden",
                          *files], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]

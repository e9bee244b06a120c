"""The Q8_0 GEMM has five operand kinds (gemm_q8.cu): the int8 quants with
kind::i8 block-dot MMAs and the scale products from a one-hot tensor-core MMA
("i8s", the default), the same on exact fp16 copies of the quants ("f16s"),
fp16 copies with the block scales applied on the CUDA cores ("f16"), the int8
quants likewise ("i8"), and "f16" on CTA pairs ("pair").  The library picks
one per process (PXQ_Q8_0_MMA, read once).  The rest of the GPU suite runs
the default kind; this test reruns the GEMM parity files in a child process
with each kind, so all stay bit-exact in their block dots and within
max-abs-rel 1e-3 of the oracle."""
import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["f16", "i8", "f16s", "pair", "i8s"])
def test_q8_0_gemm_parity_in_each_mma_kind(kind):
    env = dict(os.environ, PXQ_Q8_0_MMA=kind)
    files = [os.path.join(ROOT, "tests", f) for f in ("test_gpu_parity.py", "test_gpu_baseline_shapes.py")]
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-k", "gemm or matmul or q6_K_golden",
                          *files], cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-2000:]

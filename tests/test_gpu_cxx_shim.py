"""GPU: the C++ drop-in shim (include/pxq_pixelina.hpp) used from a C++
program, the way Pixelina's backend_cpu.cpp would call it."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cxx_shim_against_oracle(tmp_path):
    exe = str(tmp_path / "shim_check")
    lib_dir = os.path.join(ROOT, "pixelina_b200")
    obj = str(tmp_path / "pxq_oracle.o")
    subprocess.run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-c", os.path.join(ROOT, "oracle", "pxq_oracle.c"),
                    "-o", obj], check=True)
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cxx", "shim_check.cpp"), obj, "-L", lib_dir, "-lpxq",
                    f"-Wl,-rpath,{lib_dir}", "-lm", "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "OK" in out.stdout

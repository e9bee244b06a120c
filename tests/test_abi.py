"""CPU: the C-ABI library loads, exports exactly what include/pxq.h declares,
and its host-only logic (sizes, argument contract) matches the reference.
No kernel is launched here."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from pixelina_b200 import pxq

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "pxq.h")


def declared_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"PXQ_API\s+[\w\s\*]+?\b(pxq_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = pxq.load()
    names = declared_functions()
    assert len(names) >= 15
    for n in names:
        assert hasattr(lib, n), f"libpxq.so does not export {n}"


def test_python_mirror_covers_header():
    assert sorted(pxq.SIGNATURES) == declared_functions()


def test_library_is_sm100a_only():
    # the shared object carries no fallback: every kernel is built for sm_100a
    data = open(pxq.LIB_PATH, "rb").read()
    assert b"sm_100a" in data


@pytest.mark.parametrize("wtype", [0, 1, 8, 13, 14, 30, 2, 99])
def test_weight_bytes_matches_reference(oracle, wtype):
    for inner, rows in ((32, 1), (256, 3), (3840, 3840), (96, 7), (100, 2), (0, 5), (512, 0)):
        assert pxq.weight_bytes(inner, rows, wtype) == oracle.weight_bytes(inner, rows, wtype)


def test_quant_matmul_not_handled_contract():
    """pxq_quant_matmul returns UNSUPPORTED exactly where cpu_quant_matmul
    returns false (src/kernels_quant.cpp:373-377); validated before any
    device work."""
    lib = pxq.load()
    w = np.zeros(4096, dtype=np.uint8)
    x = np.zeros(4096, dtype=np.float32)
    y = np.zeros(4096, dtype=np.float32)
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    cases = [(0, 4, 2, 32), (1, 4, 2, 32), (8, 4, 2, 48), (13, 4, 2, 128), (14, 4, 2, 128), (8, 0, 2, 32), (8, 4, 0, 32),
             (8, 4, 2, 0)]
    for wtype, rows, columns, inner in cases:
        rc = lib.pxq_quant_matmul(p(w), wtype, p(x), p(y), rows, columns, inner)
        assert rc == pxq.ERR_UNSUPPORTED, (wtype, rows, columns, inner, rc)


def test_init_without_device_is_an_error_not_a_crash():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    rc = pxq.load().pxq_init(0)
    assert rc == pxq.ERR_NO_DEVICE
    assert "device" in pxq.last_error()


def test_library_loads_no_nccl_until_a_communicator_is_used():
    """libpxq binds NCCL at the first communicator call, so loading it never
    pulls an NCCL into a process (one loaded later, e.g. PyTorch's, would
    otherwise clash with it)."""
    import subprocess
    import sys

    code = ("import ctypes, sys; sys.path.insert(0, %r); from pixelina_b200 import pxq; pxq.load(); "
            "maps = open('/proc/self/maps').read(); print('nccl' in maps)") % ROOT
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    assert res.stdout.strip() == "False"


def test_comm_argument_contract():
    """The multi-GPU entry points reject bad arguments before any NCCL or
    device work."""
    lib = pxq.load()
    cid = (C.c_uint8 * 128)()
    h = C.c_void_p()
    assert lib.pxq_comm_init(None, 2, 0, 1000, C.byref(h)) == pxq.ERR_INVALID
    assert lib.pxq_comm_init(C.cast(cid, C.c_void_p), 0, 0, 1000, C.byref(h)) == pxq.ERR_INVALID
    assert lib.pxq_comm_init(C.cast(cid, C.c_void_p), 2, 2, 1000, C.byref(h)) == pxq.ERR_INVALID
    assert lib.pxq_comm_init(C.cast(cid, C.c_void_p), 9, 0, 1000, C.byref(h)) == pxq.ERR_INVALID
    assert lib.pxq_comm_init(C.cast(cid, C.c_void_p), 2, 0, 0, C.byref(h)) == pxq.ERR_INVALID
    assert lib.pxq_comm_unique_id(None) == pxq.ERR_INVALID
    assert lib.pxq_comm_destroy(None) == pxq.ERR_INVALID
    assert lib.pxq_comm_barrier(None) == pxq.ERR_INVALID
    assert lib.pxq_sharded_output_destroy(None) == pxq.ERR_INVALID
    assert lib.pxq_sharded_matmul(None, None, 1, None, 1, None, None, 0, None) == pxq.ERR_INVALID
    assert lib.pxq_sharded_matmul_host(None, None, 1, None, 1, 1, None) == pxq.ERR_INVALID
    assert "communicator" in pxq.last_error()

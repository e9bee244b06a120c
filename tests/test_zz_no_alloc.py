"""GPU: pxq_matvec_noalloc, the decode matvec that allocates no device memory.

It is meant for callers that cannot call cudaMalloc while they run (a decode
loop that must not stall on the allocator, a region where the application
forbids allocation, a fixed device-memory budget).  Its quantized activations
live in a static 4 MiB device array of the library instead of per-call
scratch, so its results must equal those of pxq_matvec, the entry point that
allocates.  This file sorts last so a `-x` run has already run every other
test if it fails; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from conftest import TOL, max_abs_rel
from pixelina_b200 import synth

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


@pytest.mark.parametrize("wtype", [8, 13, 14])
def test_noalloc_matches_allocating_matvec_twice(pxq, wtype):
    import torch

    lib = pxq.load()
    rows, inner = 300, 3584
    w = synth.weights_for(wtype, rows, inner, seed=21)
    W = pxq.Weight(w, wtype, inner, rows)
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    # calls in a row with different inputs and shapes, each reusing the static
    # scratch the one before filled: 8 activation rows (a separate quantize
    # kernel for the K-quants), then 3 and 1 (the matvec quantizes them itself)
    for call, (columns, first, count) in enumerate(((8, 0, 300), (3, 7, 250), (1, 0, 300))):
        x = torch.from_numpy(synth.activations(columns, inner, seed=30 + call)).cuda()
        bias = torch.linspace(-0.5, 0.5, count, device="cuda")
        want = torch.empty((columns, count), device="cuda")
        got = torch.full((columns, count), float("nan"), device="cuda")
        rc = lib.pxq_matvec(W.handle, first, count, _p(x), columns, _p(want), count, _p(bias), sp)
        assert rc == 0, pxq.last_error()
        rc = lib.pxq_matvec_noalloc(W.handle, first, count, _p(x), columns, _p(got), count, _p(bias), sp)
        assert rc == 0, pxq.last_error()
        torch.cuda.synchronize()
        assert max_abs_rel(got.cpu().numpy(), want.cpu().numpy()) <= TOL
    W.release()


def test_noalloc_makes_no_device_allocation(pxq):
    import torch

    lib = pxq.load()
    rows, inner = 512, 4096
    W = pxq.Weight(synth.q5_K_weights(rows, inner, seed=3), 13, inner, rows)
    x = torch.from_numpy(synth.activations(4, inner, seed=4)).cuda()
    y = torch.empty((4, rows), device="cuda")
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.pxq_matvec_noalloc(W.handle, 0, rows, _p(x), 4, _p(y), rows, None, sp) == 0  # first call: set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert lib.pxq_matvec_noalloc(W.handle, 0, rows, _p(x), 4, _p(y), rows, None, sp) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    W.release()


def test_noalloc_rejects_oversized_activation(pxq):
    import torch

    lib = pxq.load()
    rows, inner = 16, 524288  # activation alone: 8 rows x 2048 super-blocks x 288 B > 4 MiB
    W = pxq.Weight(synth.random_q5_K(rows, inner, np.random.default_rng(1)), 13, inner, rows)
    x = torch.zeros((8, inner), device="cuda")
    y = torch.zeros((8, rows), device="cuda")
    rc = lib.pxq_matvec_noalloc(W.handle, 0, rows, _p(x), 8, _p(y), rows, None, None)
    assert rc == pxq.ERR_UNSUPPORTED
    assert "PXQ_NOALLOC_SCRATCH_BYTES" in pxq.last_error()
    W.release()


def test_bounded_wait_timeout_then_both_scratches_recover(pxq, oracle):
    """Failure detection without a fault: a matvec whose CTA 0 loads nothing
    (pxq_debug_matvec_stall) gives up its bounded waits after their limit and
    records a status; pxq_synchronize reports PXQ_ERR_DEVICE_STATUS.  The
    interrupted call leaves split-K counts behind in the scratch it used --
    the static no-allocation array or the stream's buffer -- and the next
    fused calls (which have no quantize kernel to clear them) must still
    compute correctly, because pxq_synchronize zeroes them on that error."""
    import torch

    lib = pxq.load()
    rows, inner = 200, 18944  # split-K over the whole grid, one activation row: the fused path
    w = synth.random_q5_K(rows, inner, np.random.default_rng(5))
    W = pxq.Weight(w, 13, inner, rows)
    xh = synth.activations(1, inner, seed=6)
    ok, ref = oracle.quant_matmul(w, 13, xh, rows)
    assert ok
    x = torch.from_numpy(xh).cuda()
    sp = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for static in (1, 0):
        junk = torch.empty((1, rows), device="cuda")
        assert lib.pxq_debug_matvec_stall(W.handle, _p(x), 1, _p(junk), static, sp) == 0, pxq.last_error()
        assert lib.pxq_synchronize(sp) == pxq.ERR_DEVICE_STATUS
        assert "gave up" in pxq.last_error()
        for name in ("pxq_matvec_noalloc", "pxq_matvec"):
            for _ in range(2):
                y = torch.full((1, rows), float("nan"), device="cuda")
                rc = getattr(lib, name)(W.handle, 0, rows, _p(x), 1, _p(y), rows, None, sp)
                assert rc == 0, pxq.last_error()
                assert lib.pxq_synchronize(sp) == 0, pxq.last_error()
                assert max_abs_rel(y.cpu().numpy(), ref) <= TOL, (static, name)
    W.release()

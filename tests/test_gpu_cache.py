"""GPU: the weight cache's residency budget and the host-buffer drop-in's
cache identity.

The reference's GPU backend keeps device copies of weights in a cache with a
byte budget and evicts the least recently used entry when an upload would
exceed it (src/backend_vulkan.cpp:671-681, :742-758); a tensor larger than
the whole budget is not cached and the caller falls back.  Here the cached
bytes are the raw rows plus the GEMM operand copies.  Every result must
still match the oracle after entries were evicted and made again, and a host
buffer refilled at the same address must not return the old device copy.
"""
import numpy as np
import pytest

from conftest import TOL, max_abs_rel
from pixelina_b200 import synth

pytestmark = pytest.mark.gpu

Q8_0, Q5_K = 8, 13


@pytest.fixture
def fresh_cache(pxq):
    pxq.load().pxq_weight_cache_clear()
    yield pxq
    pxq.cache_limit(0)
    pxq.load().pxq_weight_cache_clear()


def test_budget_evicts_least_recently_used_and_results_stay_exact(fresh_cache, oracle):
    pxq = fresh_cache
    rows, inner, columns = 256, 1024, 300  # the GEMM path: raw rows + operand copy per weight
    ws = [synth.weights_for(Q8_0, rows, inner, seed=40 + i) for i in range(4)]
    x = synth.activations(columns, inner, seed=50)
    refs = [oracle.quant_matmul(w, Q8_0, x, rows)[1] for w in ws]
    handled, _ = pxq.quant_matmul(ws[0], Q8_0, x, rows)
    assert handled
    one, _, _ = pxq.cache_usage()
    assert one > rows * inner  # raw rows and the operand copy
    pxq.cache_limit(int(2.5 * one))  # room for two weights
    for i, w in enumerate(ws):
        handled, y = pxq.quant_matmul(w, Q8_0, x, rows)
        assert handled and max_abs_rel(y, refs[i]) <= TOL, i
        used, limit, entries = pxq.cache_usage()
        assert used <= limit and entries <= 2, (i, used, limit, entries)
    # the first weight was evicted: it is uploaded again and still exact
    handled, y = pxq.quant_matmul(ws[0], Q8_0, x, rows)
    assert handled and max_abs_rel(y, refs[0]) <= TOL


def test_keyed_weight_loses_only_its_operand_copy(fresh_cache, oracle):
    import torch

    pxq = fresh_cache
    rows, inner, columns = 256, 1024, 140
    w = synth.weights_for(Q5_K, rows, inner, seed=61)
    x = synth.activations(columns, inner, seed=62)
    ok, ref = oracle.quant_matmul(w, Q5_K, x, rows)
    W = pxq.Weight(w, Q5_K, inner, rows, key="test:keyed")
    xd = torch.from_numpy(x).cuda()
    assert max_abs_rel(pxq.matmul(W, xd, path="gemm").cpu().numpy(), ref) <= TOL
    with_copy, _, _ = pxq.cache_usage()
    pxq.cache_limit(with_copy - 1)  # the operand copy must go, the raw rows stay
    used, _, entries = pxq.cache_usage()
    assert entries == 1 and used < with_copy
    # the handle still works: the GEMM rebuilds the copy, the matvec needs none
    assert max_abs_rel(pxq.matmul(W, xd, path="gemm").cpu().numpy(), ref) <= TOL
    assert max_abs_rel(pxq.matmul(W, xd[:3], path="matvec").cpu().numpy(), ref[:3]) <= TOL
    W.release()
    assert pxq.cache_usage()[2] == 0


def test_tensor_larger_than_the_budget_is_not_handled(fresh_cache):
    pxq = fresh_cache
    w = synth.weights_for(Q8_0, 256, 1024, seed=71)
    x = synth.activations(16, 1024, seed=72)
    pxq.cache_limit(64 << 10)
    handled, _ = pxq.quant_matmul(w, Q8_0, x, 256)
    assert not handled  # the reference's nullptr: the caller falls back
    assert "budget" in pxq.last_error()


def test_refilled_host_buffer_is_not_served_stale(fresh_cache, oracle):
    pxq = fresh_cache
    rows, inner = 192, 512
    buf = synth.weights_for(Q8_0, rows, inner, seed=81)
    other = synth.weights_for(Q8_0, rows, inner, seed=82)
    for columns in (5, 200):  # matvec and GEMM
        x = synth.activations(columns, inner, seed=83 + columns)
        w = buf.copy()
        handled, y = pxq.quant_matmul(w, Q8_0, x, rows)
        assert handled and max_abs_rel(y, oracle.quant_matmul(w, Q8_0, x, rows)[1]) <= TOL
        w[:] = other  # same address, new contents
        handled, y = pxq.quant_matmul(w, Q8_0, x, rows)
        assert handled and max_abs_rel(y, oracle.quant_matmul(other, Q8_0, x, rows)[1]) <= TOL
        assert pxq.cache_usage()[2] == 1  # the stale entry was dropped
        pxq.load().pxq_weight_cache_clear()

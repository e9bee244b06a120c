"""GPU parity of the tensor-core GEMM at the benchmark configurations.

The small-shape parity tests give every CTA (pair) at most one output tile.
The timed configurations run far more tiles than the GPU holds CTAs, so each
persistent CTA (pair) walks several tiles and carries its accumulator slots,
operand ring and barrier phases from one tile to the next.  These tests run
those exact shapes and compare a sampled grid of the output against the
oracle (the restatement of cpu_quant_matmul, src/kernels_quant.cpp:369-412).

Output elements are independent (each depends on one weight row and one
activation row, src/kernels_quant.cpp:389-400), so the oracle only computes
the sampled rows: a few weight rows from every 256-row band (both CTAs of a
pair, all four TMEM lane quadrants) against a few activation rows from every
256-row band (both column halves of the accumulator).  Tolerance: max-abs-rel
1e-3 (conftest.TOL), as the full-size tests.
"""
import numpy as np
import pytest

from conftest import TOL, max_abs_rel
from pixelina_b200 import synth

pytestmark = pytest.mark.gpu

Q8_0, Q5_K, Q6_K = 8, 13, 14
# offsets inside every 256-row band: both 128-row CTA halves, every 32-row
# lane quadrant, both 64-column halves of a drain warp's accumulator
OFFSETS = np.array([0, 1, 37, 63, 64, 101, 127, 128, 159, 190, 223, 255])


def sample_rows(total: int) -> np.ndarray:
    idx = (np.arange(0, total, 256)[:, None] + OFFSETS[None, :]).reshape(-1)
    idx = idx[idx < total]
    return np.unique(np.concatenate([idx, [total - 1]]))


def weights(wtype: int, rows: int, inner: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if wtype == Q8_0:
        return synth.encode_q8_0(rng.normal(0.0, 0.02, size=(rows, inner)).astype(np.float32))
    if wtype == Q5_K:
        return synth.random_q5_K(rows, inner, rng)
    return synth.random_q6_K(rows, inner, rng)


def check_sampled(pxq, oracle, wtype, M, N, K, seed):
    import torch

    w = weights(wtype, N, K, seed)
    x = synth.activations(M, K, seed=seed + 1)
    W = pxq.Weight(w, wtype, K, N)
    y = pxq.matmul(W, torch.from_numpy(x).cuda(), path="gemm")
    st = pxq.synchronize()
    mi, ni = sample_rows(M), sample_rows(N)
    got = y[torch.from_numpy(mi).cuda()][:, torch.from_numpy(ni).cuda()].cpu().numpy()
    del y
    W.release()
    ok, ref = oracle.quant_matmul(w[ni], wtype, x[mi], len(ni))
    assert ok
    err = max_abs_rel(got, ref)
    assert err <= TOL, (wtype, M, N, K, err)
    return st


@pytest.mark.parametrize("wtype,M,N,K", [
    (Q5_K, 4096, 10240, 3840),   # configs[1]: 640 pair tiles on ~74 pairs
    (Q6_K, 4096, 10240, 3840),   # the same shape with Q6_K weights
    (Q8_0, 4096, 3840, 3840),    # configs[0]: 960 single-CTA tiles
    (Q8_0, 16384, 12288, 3072),  # configs[4]: 12288 tiles, K = 3072
    (Q5_K, 4352, 9216, 3072),    # DiT QKV shape: partial last M tile, K = 3072
    (Q8_0, 4352, 3072, 12288),   # DiT FFN down shape: K = 12288
])
def test_gemm_baseline_shapes(pxq, oracle, wtype, M, N, K):
    check_sampled(pxq, oracle, wtype, M, N, K, seed=M + N + K)


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K, Q6_K])
def test_gemm_block_dots_exact_many_tiles(pxq, oracle, wtype):
    """The exact block dots when every CTA (pair) walks several tiles: 256
    pair tiles (K-quants) or 1024 tiles (Q8_0), more than the GPU holds."""
    import torch

    M, N, K = 4096, 4096, 512
    w = weights(wtype, N, K, seed=77)
    x = synth.activations(M, K, seed=78)
    W = pxq.Weight(w, wtype, K, N)
    dump = pxq.gemm_block_dots(W, torch.from_numpy(x).cuda())  # [items, M, N]
    pxq.synchronize()
    mi, ni = sample_rows(M)[::3], sample_rows(N)[::3]
    got = dump[:, torch.from_numpy(mi).cuda()][:, :, torch.from_numpy(ni).cuda()].cpu().numpy()
    del dump
    W.release()
    xs = x[mi]
    if wtype == Q8_0:
        xq = oracle.quantize_q8_0(xs)
        for a, c in enumerate(mi):
            for b, r in enumerate(ni):
                want = oracle.block_dots_q8_0(K, w[r], xq[a])
                assert np.array_equal(got[:, a, b], want.astype(np.float32)), (c, r)
        return
    xq = oracle.quantize_q8_K(xs)
    nsb = K // 256
    for a, c in enumerate(mi):
        for b, r in enumerate(ni):
            if wtype == Q6_K:
                s, chunks = oracle.block_dots_q6_K(K, w[r], xq[a])
                items = got[:, a, b].reshape(-1, 4)
                assert np.array_equal(items, chunks.astype(np.float32)), (c, r)
            else:
                s, m = oracle.block_dots_q5_K(K, w[r], xq[a])
                items = got[:, a, b].reshape(nsb, 5)
                assert np.all(items == np.round(items)), (c, r)
                assert np.array_equal(items[:, :4].astype(np.int64).sum(axis=1), s.astype(np.int64)), (c, r)
                assert np.array_equal(items[:, 4].astype(np.int64), m.astype(np.int64)), (c, r)

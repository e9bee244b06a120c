"""pxq_attention against Pixelina's own tensor_attention (src/tensor.cpp:347-427,
built into oracle/_ref) on the same fp32 inputs: multi-head with grouped
key/value heads, non-causal, causal, query ranges with a key-cache offset,
head sizes 64 / 80 / 128, the tiled prefill kernel and the key-split decode
kernel.  Both sides compute in fp32; the kernel takes the softmax online over
key tiles, so the sums are reordered: outputs agree to ATT_TOL max-abs-rel."""
import numpy as np
import pytest

from conftest import max_abs_rel
from oracle.oracle import TYPE_Q5_K, Reference, reference_available

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not reference_available(), reason="oracle/_ref is missing")]
ATT_TOL = 2e-5

CASES = [
    # q_rows, k_rows, heads, kv_heads, d, ranges, query_offset
    (96, 96, 4, 4, 128, [(0, 96, 96, False)], 0),                      # DiT-like, non-causal
    (70, 70, 4, 2, 64, [(0, 70, 70, True)], 0),                        # causal, grouped kv heads
    (130, 150, 2, 1, 80, [(0, 50, 150, False), (50, 130, 120, True)], 20),  # ranges with an offset
    (300, 300, 8, 8, 128, [(0, 300, 300, False)], 0),                   # several 64-row query tiles
    (1, 777, 7, 1, 128, [(0, 1, 777, True)], 776),                      # decode, one row
    (5, 1000, 8, 2, 64, [(0, 5, 1000, True)], 995),                     # decode, five rows
    (8, 4096, 28, 4, 128, [(0, 8, 4096, True)], 4088),                  # VL decode shape, eight rows
    (3, 50, 2, 2, 80, [(0, 2, 50, False), (2, 3, 30, True)], 10),      # decode with two ranges
    (12, 40, 3, 1, 64, [(0, 12, 40, True)], 28),                        # 16-row query tiles
    (20, 200, 4, 2, 80, [(0, 20, 200, False)], 0),                      # 32-row query tiles
    (8, 300, 28, 2, 128, [(0, 8, 300, True)], 292),                     # 14 heads per kv head: two CTAs per group
]


@pytest.mark.parametrize("case", range(len(CASES)))
def test_attention_matches_reference(pxq, case):
    import torch

    rows, keys, heads, kvh, d, ranges, off = CASES[case]
    rng = np.random.default_rng(100 + case)
    q = rng.standard_normal((rows, heads * d)).astype(np.float32)
    k = rng.standard_normal((keys, kvh * d)).astype(np.float32)
    v = rng.standard_normal((keys, kvh * d)).astype(np.float32)
    want = Reference().attention(q, k, v, heads, kvh, ranges, off)
    assert want is not None
    got = pxq.attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), heads, kvh,
                        ranges=ranges, query_offset=off).cpu().numpy()
    pxq.synchronize()
    assert max_abs_rel(got, want) <= ATT_TOL


def test_attention_first_overload_and_argument_checks(pxq):
    """ranges=None is the first overload (non-causal or causal from row 0); the
    reference's argument checks are errors here."""
    import torch

    rng = np.random.default_rng(7)
    q = rng.standard_normal((40, 2 * 64)).astype(np.float32)
    k = rng.standard_normal((40, 64)).astype(np.float32)
    v = rng.standard_normal((40, 64)).astype(np.float32)
    qd, kd, vd = (torch.from_numpy(a).cuda() for a in (q, k, v))
    for causal in (False, True):
        want = Reference().attention(q, k, v, 2, 1, [(0, 40, 40, causal)], 0)
        got = pxq.attention(qd, kd, vd, 2, 1, causal=causal).cpu().numpy()
        assert max_abs_rel(got, want) <= ATT_TOL
    for bad in ([(0, 20, 40, False)], [(0, 20, 40, False), (21, 40, 40, False)], [(0, 40, 41, False)], [(0, 40, 0, False)]):
        assert Reference().attention(q, k, v, 2, 1, bad, 0) is None  # the reference rejects these too
        with pytest.raises(pxq.PxqError) as err:
            pxq.attention(qd, kd, vd, 2, 1, ranges=bad)
        assert err.value.code == pxq.ERR_INVALID
    with pytest.raises(pxq.PxqError) as err:  # 3 heads over 2 kv heads
        pxq.attention(torch.zeros((4, 3 * 64), device="cuda"), torch.zeros((4, 2 * 64), device="cuda"),
                      torch.zeros((4, 2 * 64), device="cuda"), 3, 2)
    assert err.value.code == pxq.ERR_INVALID


def test_attention_unaligned_rows(pxq):
    """Tensors that start one float past a 16-byte boundary take the kernel's
    word-by-word loads and stores; results are the same."""
    import torch

    rows, keys, heads, kvh, d = 70, 90, 2, 1, 64
    rng = np.random.default_rng(11)
    q = rng.standard_normal((rows, heads * d)).astype(np.float32)
    k = rng.standard_normal((keys, kvh * d)).astype(np.float32)
    v = rng.standard_normal((keys, kvh * d)).astype(np.float32)

    def shifted(x):
        buf = torch.zeros(x.size + 1, device="cuda")
        buf[1:] = torch.from_numpy(x.reshape(-1)).cuda()
        return buf[1:].view(x.shape)

    for r, ranges in ((rows, [(0, rows, keys, True)]), (3, [(0, 3, keys, True)])):
        want = Reference().attention(q[:r], k, v, heads, kvh, ranges, keys - r)
        out = shifted(np.zeros((r, heads * d), np.float32))
        assert out.data_ptr() % 16 == 4
        pxq.attention(shifted(q[:r]), shifted(k), shifted(v), heads, kvh, ranges=ranges, query_offset=keys - r, out=out)
        pxq.synchronize()
        assert max_abs_rel(out.cpu().numpy(), want) <= ATT_TOL


def test_attention_leaves_matvec_counters_alone(pxq, oracle):
    """The decode kernels' partial sums share the stream's scratch with the
    matvec's stream-K counters, which every call must leave zero: a stream-K
    matvec right after a decode attention on the same stream is still exact."""
    import torch

    from pixelina_b200 import synth

    rng = np.random.default_rng(3)
    q = torch.from_numpy(rng.standard_normal((8, 28 * 128)).astype(np.float32)).cuda()
    kv = torch.from_numpy(rng.standard_normal((4096, 4 * 128)).astype(np.float32)).cuda()
    pxq.attention(q, kv, kv, 28, 4, ranges=[(0, 8, 4096, True)], query_offset=4088)
    rows, inner = 100, 1024  # a few stream-K CTAs sharing tiles
    w = synth.weights_for(TYPE_Q5_K, rows, inner, seed=1)
    x = synth.activations(1, inner, seed=51)
    W = pxq.Weight(w, TYPE_Q5_K, inner, rows)
    y = pxq.matmul(W, torch.from_numpy(x).cuda(), path="matvec").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, TYPE_Q5_K, x, rows)
    assert ok and max_abs_rel(y, ref) <= 1e-3

"""CPU: pin the oracle restatement to the reference.

1. Against the committed golden vectors (outputs of Pixelina's own CPU kernels,
   tests/golden/make_golden.py): bit-exact quantize, decode and matmul.
2. Against the live reference build, when oracle/_ref was built here: random
   shapes and crafted rounding ties.
3. Internal consistency: exact block dots reproduce the float dots.
"""
import numpy as np
import pytest

from oracle.oracle import TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0
from pixelina_b200 import synth


def test_quantize_q8_0_golden(oracle, golden):
    assert np.array_equal(oracle.quantize_q8_0(golden["q8_0_x"]), golden["q8_0_blocks"])


def test_quantize_q8_K_golden(oracle, golden):
    assert np.array_equal(oracle.quantize_q8_K(golden["q8_K_x"]), golden["q8_K_blocks"])


@pytest.mark.parametrize("name,wtype", [("q8_0", TYPE_Q8_0), ("q5_K", TYPE_Q5_K), ("q6_K", TYPE_Q6_K)])
def test_decode_golden(oracle, golden, name, wtype):
    w = golden[f"w_{name}"]
    got = oracle.decode(w.reshape(-1), wtype, golden[f"decode_{name}"].size)
    assert np.array_equal(got.view(np.uint32), golden[f"decode_{name}"].view(np.uint32))


@pytest.mark.parametrize("name,wtype", [("q8_0", TYPE_Q8_0), ("q5_K", TYPE_Q5_K), ("q6_K", TYPE_Q6_K)])
def test_matmul_golden_bitexact(oracle, golden, name, wtype):
    w = golden[f"w_{name}"]
    ok, y = oracle.quant_matmul(w, wtype, golden["mm_x"], w.shape[0])
    assert ok
    assert np.array_equal(y.view(np.uint32), golden[f"mm_{name}"].view(np.uint32))


def test_unhandled_contract(oracle, golden):
    # inner % 32 != 0 -> not handled, as the reference reported
    ok, _ = oracle.quant_matmul(golden["w_q8_0"][:, :34], TYPE_Q8_0, golden["mm_x"][:, :48], 48)
    assert int(ok) == int(golden["mm_unhandled"][0]) == 0
    ok, _ = oracle.quant_matmul(golden["w_q8_0"], 0, golden["mm_x"], 48)
    assert not ok


def test_half_conversions(oracle):
    h = np.arange(0, 65536, 97, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.half_to_float(int(v)) for v in h], dtype=np.float32)
    fin = np.isfinite(ref)
    assert np.array_equal(got[fin].view(np.uint32), ref[fin].view(np.uint32))
    rng = np.random.default_rng(0)
    f = np.concatenate([rng.standard_normal(3000) * s for s in (1e-7, 1e-5, 1e-3, 1, 1e3, 6e4)]).astype(np.float32)
    f = np.concatenate([f, np.float32([0.0, -0.0, 65504, 65520, 65519.99, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26])])
    with np.errstate(over="ignore"):
        want = f.astype(np.float16).view(np.uint16)
    got = np.array([oracle.float_to_half(float(v)) for v in f], dtype=np.uint16)
    assert np.array_equal(got, want)


def test_block_dots_match_float_dots(oracle):
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, 512)).astype(np.float32)
    w8 = synth.q8_0_weights(4, 512, seed=6)
    xq = oracle.quantize_q8_0(x)
    for r in range(4):
        for c in range(3):
            I = oracle.block_dots_q8_0(512, w8[r], xq[c]).astype(np.float64)
            dw = w8[r].reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float64)[:, 0]
            dx = xq[c].reshape(-1, 34)[:, :2].copy().view(np.float16).astype(np.float64)[:, 0]
            exact = float((I * dw * dx).sum())
            assert abs(exact - oracle.dot(TYPE_Q8_0, 512, w8[r], xq[c])) <= 1e-5 * max(1.0, abs(exact))
    w5 = synth.q5_K_weights(2, 512, seed=7)
    xk = oracle.quantize_q8_K(x)
    for r in range(2):
        s, m = oracle.block_dots_q5_K(512, w5[r], xk[0])
        blk = w5[r].reshape(-1, 176)
        d = blk[:, 0:2].copy().view(np.float16).astype(np.float64)[:, 0]
        dm = blk[:, 2:4].copy().view(np.float16).astype(np.float64)[:, 0]
        yd = xk[0].reshape(-1, 292)[:, 0:4].copy().view(np.float32).astype(np.float64)[:, 0]
        exact = float((yd * d * s).sum() - (yd * dm * m).sum())
        assert abs(exact - oracle.dot(TYPE_Q5_K, 512, w5[r], xk[0])) <= 1e-5 * max(1.0, abs(exact))
    w6 = synth.random_q6_K(3, 512, np.random.default_rng(8))
    for r in range(3):
        for c in range(3):
            s, ch = oracle.block_dots_q6_K(512, w6[r], xk[c])
            assert np.array_equal(ch.astype(np.int64).sum(axis=1), s.astype(np.int64))
            d = w6[r].reshape(-1, 210)[:, 208:210].copy().view(np.float16).astype(np.float64)[:, 0]
            yd = xk[c].reshape(-1, 292)[:, 0:4].copy().view(np.float32).astype(np.float64)[:, 0]
            exact = float((yd * d * s).sum())
            assert abs(exact - oracle.dot(TYPE_Q6_K, 512, w6[r], xk[c])) <= 1e-5 * max(1.0, abs(exact))


def test_synth_q8_0_matches_reference_quantizer(oracle):
    # the weight encoder uses the same arithmetic as quantize_row_q8_0_ref
    w = np.random.default_rng(8).normal(0, 0.02, size=(16, 1024)).astype(np.float32)
    assert np.array_equal(synth.encode_q8_0(w), oracle.quantize_q8_0(w))


def test_synth_q5_K_roundtrip(oracle):
    w = np.random.default_rng(9).normal(0, 0.02, size=(8, 1024)).astype(np.float32)
    b = synth.encode_q5_K(w)
    dec = oracle.decode(b.reshape(-1), TYPE_Q5_K, w.size).reshape(w.shape)
    # 5-bit quantization of each 32-value sub-block: error below one step
    assert np.abs(dec - w).max() < 0.25 * np.abs(w).max()
    assert np.corrcoef(dec.ravel(), w.ravel())[0, 1] > 0.99


# ---- against the live reference build (only where it was built) ------------

@pytest.mark.parametrize("seed", [1, 2, 3])
def test_oracle_vs_reference_random(oracle, reference, seed):
    rng = np.random.default_rng(100 + seed)
    inner = 256 * int(rng.integers(1, 9))
    x = (rng.standard_normal((5, inner)) * rng.uniform(0.01, 100)).astype(np.float32)
    assert np.array_equal(oracle.quantize_q8_0(x), reference.quantize_q8_0(x))
    assert np.array_equal(oracle.quantize_q8_K(x), reference.quantize_q8_K(x))
    for wtype, w in ((TYPE_Q8_0, synth.q8_0_weights(33, inner, seed)), (TYPE_Q5_K, synth.q5_K_weights(17, inner, seed))):
        ok1, y1 = oracle.quant_matmul(w, wtype, x, w.shape[0])
        ok2, y2 = reference.quant_matmul(w, wtype, x, w.shape[0])
        assert ok1 and ok2
        assert np.array_equal(y1.view(np.uint32), y2.view(np.uint32))


def test_q8_K_fused_rounding_ties(oracle, reference):
    """The reference build fuses iscale*x + 1.5*2^23 into one FMA; crafted
    near-ties tell the fused and unfused forms apart."""
    base = np.array([(k + 0.5) / 127 for k in range(126)], dtype=np.float32)
    vals = np.concatenate([base, np.nextafter(base, np.float32(2)), np.nextafter(base, np.float32(-2))])
    blk = np.concatenate([[np.float32(1.0)], vals[:255]]).astype(np.float32)[None, :]
    assert blk.shape == (1, 256)
    r = reference.quantize_q8_K(blk)
    assert np.array_equal(oracle.quantize_q8_K(blk), r)
    q = r[0, 4:260].view(np.int8).astype(np.int64)
    exact = np.float64(np.float32(-127.0)) * blk[0].astype(np.float64)
    fused = np.minimum(np.round(exact), 127)            # one rounding: round-half-even of the exact product
    unfused = np.minimum(np.round(exact.astype(np.float32).astype(np.float64)), 127)
    assert np.array_equal(q, fused) and not np.array_equal(q, unfused)

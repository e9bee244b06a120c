"""Generate tests/golden/golden.npz from Pixelina's own CPU kernels.

Run where the reference tree is available and oracle/_ref/libpixref.so has
been built (``make -C oracle REF=<Pixelina tree>``):

    python tests/golden/make_golden.py

Every array in the fixture is an input we generated (seeded, plus crafted
edge cases) or an output of the reference build (quantized bytes, decoded
floats, matmul outputs).  The tests compare the oracle restatement and the
CUDA kernels against these outputs, so they keep working where the reference
tree is absent (e.g. on the GPU box).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import TYPE_Q5_K, TYPE_Q6_K, TYPE_Q8_0, Reference  # noqa: E402
from pixelina_b200 import synth  # noqa: E402


def edge_rows_q8_0(rng: np.random.Generator, inner: int) -> np.ndarray:
    """Rows exercising the Q8_0 rounding contract block by block."""
    rows = []
    # all-zero blocks (d = 0 -> id = 0 branch, src/kernels_quant.cpp:134)
    r = rng.standard_normal(inner).astype(np.float32)
    r[:32] = 0
    rows.append(r)
    # ties on |max| with opposite signs, and x*id exactly at k + 0.5
    r = rng.standard_normal(inner).astype(np.float32)
    r[32:64] = np.linspace(-1, 1, 32, dtype=np.float32)
    r[32] = 127.0
    r[33] = -127.0
    for j in range(34, 64):  # amax = 127 -> d = 1, id = 1: x = k + 0.5 exactly
        r[j] = np.float32((j - 34) - 15 + 0.5)
    rows.append(r)
    # tiny values -> fp16 subnormal scale; huge values -> large scale
    r = (rng.standard_normal(inner) * 1e-6).astype(np.float32)
    r[64:96] *= 1e-3
    r[96:128] = (rng.standard_normal(32) * 3e4).astype(np.float32)
    rows.append(r)
    # single spike per block
    r = np.zeros(inner, dtype=np.float32)
    r[::32] = 1.0
    r[5::32] = -2.5
    rows.append(r)
    return np.stack(rows)


def edge_rows_q8_K(rng: np.random.Generator, inner: int) -> np.ndarray:
    rows = []
    r = rng.standard_normal(inner).astype(np.float32)
    r[:256] = 0  # all-zero super-block (src/kernels_quant.cpp:96-102)
    rows.append(r)
    # the largest |x| appears twice with opposite signs: the first one wins
    r = rng.standard_normal(inner).astype(np.float32)
    r[256 + 3] = -4.0
    r[256 + 200] = 4.0
    rows.append(r)
    # iscale = -127 with values at (k + 0.5)/127 +- 1 ulp: the fused
    # multiply-add of the reference build decides these ties
    r = np.zeros(inner, dtype=np.float32)
    base = np.array([(k + 0.5) / 127 for k in range(0, 126)], dtype=np.float32)
    vals = np.concatenate([base, np.nextafter(base, np.float32(2)), np.nextafter(base, np.float32(-2))])
    r[0] = 1.0
    r[1:256] = vals[:255]
    r[256] = -1.0
    r[257:512] = -vals[255 - 255:255][:255]
    rows.append(r)
    # positive max (d < 0 in the reference) and negative max
    r = np.abs(rng.standard_normal(inner)).astype(np.float32)
    rows.append(r)
    rows.append(-r)
    return np.stack(rows)


def main() -> None:
    ref = Reference()
    ref.set_threads(1)
    rng = np.random.default_rng(20261201)
    out = {}

    inner = 512
    xq0 = np.concatenate([rng.standard_normal((6, inner)).astype(np.float32), edge_rows_q8_0(rng, inner)])
    out["q8_0_x"] = xq0
    out["q8_0_blocks"] = ref.quantize_q8_0(xq0)

    xqk = np.concatenate([rng.standard_normal((4, inner)).astype(np.float32), edge_rows_q8_K(rng, inner)])
    out["q8_K_x"] = xqk
    out["q8_K_blocks"] = ref.quantize_q8_K(xqk)

    # weights: Q8_0 and Q5_K from N(0, 0.02); Q6_K random valid bytes
    w8 = synth.q8_0_weights(48, inner, seed=3)
    w5 = synth.q5_K_weights(40, inner, seed=4)
    S6 = 24 * inner // 256
    raw6 = rng.integers(0, 256, size=(S6, 210), dtype=np.uint8)
    raw6[:, 192:208] = rng.integers(-32, 32, size=(S6, 16)).astype(np.int8).view(np.uint8)
    raw6[:, 208:210] = (rng.uniform(0.5, 1.5, S6) * 1e-3).astype(np.float16).view(np.uint8).reshape(S6, 2)
    w6 = raw6.reshape(24, inner // 256 * 210)
    out["w_q8_0"], out["w_q5_K"], out["w_q6_K"] = w8, w5, w6
    out["decode_q8_0"] = ref.decode(w8.reshape(-1), TYPE_Q8_0, 48 * inner)
    out["decode_q5_K"] = ref.decode(w5.reshape(-1), TYPE_Q5_K, 40 * inner)
    out["decode_q6_K"] = ref.decode(w6.reshape(-1), TYPE_Q6_K, 24 * inner)

    xm = rng.standard_normal((7, inner)).astype(np.float32)
    xm[2, :256] = 0
    out["mm_x"] = xm
    for name, w, t, rows in (("q8_0", w8, TYPE_Q8_0, 48), ("q5_K", w5, TYPE_Q5_K, 40), ("q6_K", w6, TYPE_Q6_K, 24)):
        ok, y = ref.quant_matmul(w, t, xm, rows)
        assert ok
        out[f"mm_{name}"] = y
    # reference's "not handled" contract
    ok_bad_inner, _ = ref.quant_matmul(w8[:, :34], TYPE_Q8_0, xm[:, :48], 48)
    out["mm_unhandled"] = np.array([int(ok_bad_inner)])

    path = os.path.join(HERE, "golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()

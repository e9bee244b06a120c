"""Seeded synthetic GGUF weights and activations for tests and benchmarks.

The reference ships no model files and no tests, so every workload here is
built from seeded random data with the shapes and value distributions of
the benchmark configurations:

* ``encode_q8_0``: GGUF Q8_0 weight rows from fp32 values (per 32-block
  ``d = absmax/127`` stored as fp16, ``q = round(v/d)``), the block format
  of src/kernels_quant.cpp:14-17 and src/backend_cpu.cpp:92-95.
* ``encode_q5_K``: GGUF Q5_K super-blocks from fp32 values.  Pixelina has no
  Q5_K encoder (it only reads the format), so this is a small encoder of our
  own written from the bit layout that cpu_decode reads
  (src/backend_cpu.cpp:97-120): value = d*sc*q - dmin*m with 6-bit sub-block
  scales/mins and 5-bit quants.  It is not a quality-optimised k-quant
  search; it only has to produce valid, typical bytes.
* ``random_q5_K``: structurally valid Q5_K bytes drawn directly (for the
  multi-GB decode stack, where encoding floats would take minutes).

Everything is numpy and deterministic for a given seed.
"""
from __future__ import annotations

import numpy as np

TYPE_Q8_0 = 8
TYPE_Q5_K = 13
TYPE_Q6_K = 14


def _round_half_away(v: np.ndarray) -> np.ndarray:
    return np.sign(v) * np.floor(np.abs(v) + 0.5)


def encode_q8_0(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, inner] -> uint8 [rows, inner/32*34] (GGUF Q8_0)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, inner = w.shape
    assert inner % 32 == 0
    b = w.reshape(rows, inner // 32, 32)
    amax = np.abs(b).max(axis=2)
    d = (amax / np.float32(127)).astype(np.float32)
    inv = np.where(d != 0, np.float32(1) / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = _round_half_away(b * inv[:, :, None]).clip(-127, 127).astype(np.int8)
    out = np.empty((rows, inner // 32, 34), dtype=np.uint8)
    out[:, :, 0:2] = d.astype(np.float16).view(np.uint8).reshape(rows, inner // 32, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, inner // 32 * 34)


def _pack_q5_K(d16, dmin16, sc, mn, q) -> np.ndarray:
    """Pack fields into 176-byte super-blocks.

    d16, dmin16: float16 [S]; sc, mn: uint8 [S, 8] (6-bit); q: uint8 [S, 256] (5-bit).
    """
    S = d16.shape[0]
    out = np.zeros((S, 176), dtype=np.uint8)
    out[:, 0:2] = d16.astype(np.float16).view(np.uint8).reshape(S, 2)
    out[:, 2:4] = dmin16.astype(np.float16).view(np.uint8).reshape(S, 2)
    sc = sc.astype(np.uint8)
    mn = mn.astype(np.uint8)
    scales = np.zeros((S, 12), dtype=np.uint8)
    for j in range(4):
        scales[:, j] = (sc[:, j] & 63) | ((sc[:, j + 4] >> 4) << 6)
        scales[:, j + 4] = (mn[:, j] & 63) | ((mn[:, j + 4] >> 4) << 6)
        scales[:, j + 8] = (sc[:, j + 4] & 15) | ((mn[:, j + 4] & 15) << 4)
    out[:, 4:16] = scales
    q = q.reshape(S, 8, 32).astype(np.uint8)
    qh = np.zeros((S, 32), dtype=np.uint8)
    for g in range(8):
        qh |= ((q[:, g, :] >> 4) & 1) << g
    out[:, 16:48] = qh
    qs = np.zeros((S, 128), dtype=np.uint8)
    for p in range(4):
        qs[:, 32 * p:32 * p + 32] = (q[:, 2 * p, :] & 15) | ((q[:, 2 * p + 1, :] & 15) << 4)
    out[:, 48:176] = qs
    return out


def encode_q5_K(w: np.ndarray) -> np.ndarray:
    """fp32 [rows, inner] -> uint8 [rows, inner/256*176] (GGUF Q5_K)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, inner = w.shape
    assert inner % 256 == 0
    S = rows * inner // 256
    x = w.reshape(S, 8, 32)
    lo = np.minimum(x.min(axis=2), 0).astype(np.float32)          # <= 0
    hi = x.max(axis=2).astype(np.float32)
    scale = ((hi - lo) / np.float32(31)).astype(np.float32)        # per sub-block
    d = (scale.max(axis=1) / np.float32(63)).astype(np.float32)
    dmin = ((-lo).max(axis=1) / np.float32(63)).astype(np.float32)
    d16 = d.astype(np.float16)
    dmin16 = dmin.astype(np.float16)
    df = d16.astype(np.float32)
    mf = dmin16.astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        sc = np.where(df[:, None] > 0, _round_half_away(scale / df[:, None]), 0).clip(0, 63)
        mn = np.where(mf[:, None] > 0, _round_half_away(-lo / mf[:, None]), 0).clip(0, 63)
        step = (df[:, None] * sc).astype(np.float32)               # [S, 8]
        off = (mf[:, None] * mn).astype(np.float32)
        q = np.where(step[:, :, None] > 0, _round_half_away((x + off[:, :, None]) / step[:, :, None]), 0).clip(0, 31)
    return _pack_q5_K(d16, dmin16, sc.astype(np.uint8), mn.astype(np.uint8), q.astype(np.uint8)).reshape(rows, inner // 256 * 176)


def random_q5_K(rows: int, inner: int, rng: np.random.Generator, d_scale: float = 0.02 / 63 / 4) -> np.ndarray:
    """Structurally valid random Q5_K rows (fields drawn independently)."""
    assert inner % 256 == 0
    S = rows * inner // 256
    d16 = (rng.uniform(0.5, 1.5, S) * d_scale).astype(np.float16)
    dmin16 = (rng.uniform(0.5, 1.5, S) * d_scale * 8).astype(np.float16)
    sc = rng.integers(0, 64, size=(S, 8), dtype=np.uint8)
    mn = rng.integers(0, 64, size=(S, 8), dtype=np.uint8)
    q = rng.integers(0, 32, size=(S, 256), dtype=np.uint8)
    return _pack_q5_K(d16, dmin16, sc, mn, q).reshape(rows, inner // 256 * 176)


def random_q6_K(rows: int, inner: int, rng: np.random.Generator, d_scale: float = 0.02 / 32 / 64) -> np.ndarray:
    """Structurally valid random Q6_K rows: {u8 ql[128]; u8 qh[64]; i8 scales[16]; fp16 d}
    per 256 values (src/kernels_quant.cpp:25-29), fields drawn independently."""
    assert inner % 256 == 0
    S = rows * inner // 256
    ql = rng.integers(0, 256, size=(S, 128), dtype=np.uint8)
    qh = rng.integers(0, 256, size=(S, 64), dtype=np.uint8)
    sc = rng.integers(-128, 128, size=(S, 16)).astype(np.int8).view(np.uint8)
    d16 = (rng.uniform(0.5, 1.5, S) * d_scale).astype(np.float16).view(np.uint8).reshape(S, 2)
    return np.concatenate([ql, qh, sc, d16], axis=1).reshape(rows, inner // 256 * 210)


def q8_0_weights(rows: int, inner: int, seed: int, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return encode_q8_0(rng.normal(0.0, std, size=(rows, inner)).astype(np.float32))


def q5_K_weights(rows: int, inner: int, seed: int, std: float = 0.02) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return encode_q5_K(rng.normal(0.0, std, size=(rows, inner)).astype(np.float32))


def activations(columns: int, inner: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.standard_normal(size=(columns, inner), dtype=np.float32)


def weights_for(wtype: int, rows: int, inner: int, seed: int) -> np.ndarray:
    if wtype == TYPE_Q8_0:
        return q8_0_weights(rows, inner, seed)
    if wtype == TYPE_Q5_K:
        return q5_K_weights(rows, inner, seed)
    if wtype == TYPE_Q6_K:
        return random_q6_K(rows, inner, np.random.default_rng(seed))
    raise ValueError(f"no synthetic encoder for type {wtype}")

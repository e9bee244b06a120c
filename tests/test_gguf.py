"""GGUF loader (pxq_gguf_*) against Pixelina's own loader (PixModelFile::open,
src/model.cpp:138-251, built into oracle/_ref): the same files are accepted
and rejected, and accepted files give the same tensor directory (names,
types, shapes, absolute offsets, byte sizes) and metadata key count.  CPU only:
opening and parsing touch no device."""
import os

import numpy as np
import pytest

from conftest import ROOT
from gguf_writer import ARRAY, BOOL, F32, F64, I8, I32, STRING, U8, U16, U32, U64, write_gguf
from oracle.oracle import Reference, reference_available
from pixelina_b200 import pxq, synth

pytestmark = pytest.mark.skipif(not reference_available(), reason="oracle/_ref (the reference build) is missing")

Q8_0, Q5_K, Q6_K, F32T, F16T, BF16T = 8, 13, 14, 0, 1, 30


def _tensors():
    rng = np.random.default_rng(3)
    return [
        ("blk.0.ffn_up.weight", Q8_0, [512, 96], synth.q8_0_weights(96, 512, seed=1).tobytes()),
        ("blk.0.ffn_gate.weight", Q5_K, [512, 64], synth.q5_K_weights(64, 512, seed=2).tobytes()),
        ("output.weight", Q6_K, [256, 3, 2], synth.random_q6_K(6, 256, rng).tobytes()),
        ("norm.weight", F32T, [512], rng.standard_normal(512).astype(np.float32).tobytes()),
        ("tok.half", F16T, [64, 2], rng.standard_normal(128).astype(np.float16).tobytes()),
        ("tok.bf16", BF16T, [16], b"\x01\x02" * 16),
    ]


META = [("general.architecture", STRING, "qwen2vl"), ("general.alignment", U32, 64), ("a.u8", U8, 7), ("a.i8", I8, -3),
        ("a.u16", U16, 65535), ("a.f32", F32, 1.5), ("a.f64", F64, -2.25), ("a.bool", BOOL, 1), ("a.u64", U64, 2 ** 40),
        ("tokenizer.ggml.tokens", ARRAY, (STRING, ["a", "bb", "ccc"])), ("a.ints", ARRAY, (I32, [1, -2, 3])),
        ("a.empty", ARRAY, (99, []))]


def _ours(path):
    try:
        with pxq.GGUF(path) as f:
            return 0, f.tensors(), f.metadata_count
    except pxq.PxqError as e:
        return e.code, [], 0


def _check_same(path):
    ref_rc, ref_t, ref_k = Reference().gguf_list(path)
    rc, t, k = _ours(path)
    expect = {0: 0, 1: pxq.ERR_IO, 2: pxq.ERR_FORMAT}[ref_rc]
    assert rc == expect, (path, ref_rc, rc, pxq.last_error())
    if ref_rc == 0:
        assert t == ref_t and k == ref_k
    return ref_rc


def test_valid_file_matches_reference(tmp_path):
    p = str(tmp_path / "model.gguf")
    write_gguf(p, _tensors(), META, alignment=64)
    assert _check_same(p) == 0
    with pxq.GGUF(p) as f:
        t = f.find("blk.0.ffn_gate.weight")
        assert t["type"] == Q5_K and t["shape"] == [512, 64] and t["offset"] % 64 == 0
        raw = np.fromfile(p, dtype=np.uint8)
        want = synth.q5_K_weights(64, 512, seed=2).reshape(-1)
        assert np.array_equal(raw[t["offset"]:t["offset"] + t["bytes"]], want)


@pytest.mark.parametrize("case", ["magic", "version", "no_tensors", "misaligned", "overlap", "bad_type", "truncated",
                                  "bool2", "nested_array", "dup_key", "dup_name", "align_3", "align_float", "align_negative",
                                  "bad_value_type", "rank0", "rank6", "ragged_q8", "missing_file", "default_alignment",
                                  "align_u8", "long_string"])
def test_malformed_and_edge_files_match_reference(tmp_path, case):
    p = str(tmp_path / f"{case}.gguf")
    ts, meta = _tensors(), list(META)
    kw = {"alignment": 64}
    if case == "magic":
        kw["magic"] = b"GGUG"
    elif case == "version":
        kw["version"] = 2
    elif case == "no_tensors":
        ts = []
    elif case == "misaligned":
        kw["offsets"] = [0, 64, 130, 4096, 8192, 12288]
    elif case == "overlap":
        kw["offsets"] = [0, 64, 1024, 4096, 8192, 12288]
    elif case == "bad_type":
        ts[0] = (ts[0][0], 2, ts[0][2], ts[0][3])  # Q4_0: not a type the loader sizes
    elif case == "truncated":
        kw["truncate"] = 100
    elif case == "bool2":
        meta.append(("a.bad_bool", BOOL, 2))
    elif case == "nested_array":
        meta.append(("a.nested", ARRAY, (ARRAY, [])))
    elif case == "dup_key":
        meta.append(("a.u8", U8, 9))
    elif case == "dup_name":
        ts.append((ts[0][0], ts[1][1], ts[1][2], ts[1][3]))
    elif case == "align_3":
        meta[1] = ("general.alignment", U32, 3)
        kw["alignment"] = 64
    elif case == "align_float":
        meta[1] = ("general.alignment", F32, 64.0)
    elif case == "align_negative":
        meta[1] = ("general.alignment", I32, -64)
    elif case == "bad_value_type":
        meta.append(("a.weird", 13, 0))
    elif case == "rank0":
        ts[3] = (ts[3][0], ts[3][1], [], ts[3][3])
    elif case == "rank6":
        ts[3] = (ts[3][0], ts[3][1], [512, 1, 1, 1, 1, 1], ts[3][3])
    elif case == "ragged_q8":
        ts[0] = (ts[0][0], Q8_0, [500, 96], ts[0][3])
    elif case == "missing_file":
        assert _check_same(str(tmp_path / "nope.gguf")) == 1
        return
    elif case == "default_alignment":
        meta.pop(1)
        kw["alignment"] = 32
    elif case == "align_u8":
        meta[1] = ("general.alignment", U8, 128)
        kw["alignment"] = 128
    elif case == "long_string":
        meta.append(("a.long", STRING, "x" * 100000))
    write_gguf(p, ts, meta, **kw)
    _check_same(p)


@pytest.mark.gpu
def test_upload_from_file_row_views_and_gated(tmp_path, oracle):
    """Tensors uploaded from a mapped file compute what the oracle computes on
    the same bytes: whole tensors, row views (tensor_linear_rows) and a gated
    pair made of two row slices of one fused tensor (src/qwen_image.cpp:271)."""
    import torch

    from conftest import TOL, max_abs_rel

    fused = synth.q5_K_weights(128, 512, seed=4)  # rows 0..63 gate, 64..127 up
    p = str(tmp_path / "model.gguf")
    write_gguf(p, _tensors() + [("blk.0.ffn_fused.weight", Q5_K, [512, 128], fused.tobytes())], META, alignment=64)
    x = synth.activations(5, 512, seed=9)
    xd = torch.from_numpy(x).cuda()
    with pxq.GGUF(p) as f:
        for name, wtype, rows in (("blk.0.ffn_up.weight", Q8_0, 96), ("blk.0.ffn_gate.weight", Q5_K, 64)):
            wbytes = dict((t[0], t[3]) for t in _tensors())[name]
            w = np.frombuffer(wbytes, dtype=np.uint8).reshape(rows, -1)
            ok, ref = oracle.quant_matmul(w, wtype, x, rows)
            W = f.upload(name)
            V = f.upload(name, row_first=16, row_count=32)
            y = pxq.matmul(W, xd).cpu().numpy()
            yv = pxq.matmul(V, xd).cpu().numpy()
            pxq.synchronize()
            assert ok and max_abs_rel(y, ref) <= TOL and max_abs_rel(yv, ref[:, 16:48]) <= TOL
            W.release()
            V.release()
        G = f.upload_gated("blk.0.ffn_fused.weight", 0, "blk.0.ffn_fused.weight", 64, 64)
        for cols in (3, 20):
            xs = synth.activations(cols, 512, seed=10 + cols)
            okg, g = oracle.quant_matmul(fused[:64], Q5_K, xs, 64)
            oku, u = oracle.quant_matmul(fused[64:], Q5_K, xs, 64)
            h = pxq.matmul_gated(G, torch.from_numpy(xs).cuda()).cpu().numpy()
            pxq.synchronize()
            want = (g / (np.float32(1) + np.exp(-g))).astype(np.float32) * u
            assert okg and oku and max_abs_rel(h, want) <= TOL
        G.release()

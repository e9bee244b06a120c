"""GPU parity: every CUDA kernel against the oracle and the golden vectors.

Bit-exact: quantized bytes (Q8_0, Q8_K), decoded floats, and the int32 block
dots the tensor-core GEMM computes.  Tolerance: fp32 matmul outputs within
max-abs-rel 1e-3 (tests/conftest.py: TOL) of the reference's CPU result.
"""
import numpy as np
import pytest

from conftest import TOL, max_abs_rel
from pixelina_b200 import synth

pytestmark = pytest.mark.gpu

Q8_0, Q5_K, Q6_K = 8, 13, 14


def cuda(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


# ---------------------------------------------------------------- quantize --

def test_quantize_q8_0_golden(pxq, golden):
    got = pxq.quantize_q8_0(cuda(golden["q8_0_x"])).cpu().numpy()
    assert np.array_equal(got, golden["q8_0_blocks"])


def test_quantize_q8_K_golden(pxq, golden):
    got = pxq.quantize_q8_K(cuda(golden["q8_K_x"])).cpu().numpy()
    assert np.array_equal(got, golden["q8_K_blocks"])


@pytest.mark.parametrize("rows,inner,scale", [(1, 256, 1.0), (37, 4096, 1e-3), (64, 3840, 50.0), (3, 18944, 1.0)])
def test_quantize_random_bitexact(pxq, oracle, rows, inner, scale):
    rng = np.random.default_rng(rows * 7 + inner)
    x = (rng.standard_normal((rows, inner)) * scale).astype(np.float32)
    x[0, :32] = 0.0
    xd = cuda(x)
    assert np.array_equal(pxq.quantize_q8_0(xd).cpu().numpy(), oracle.quantize_q8_0(x))
    if inner % 256 == 0:
        assert np.array_equal(pxq.quantize_q8_K(xd).cpu().numpy(), oracle.quantize_q8_K(x))


def _records_to_q8_K_blocks(rec: np.ndarray) -> np.ndarray:
    """Undo the matvec record permutation: [rows, nsb*288] -> [rows, nsb*292]
    GGUF Q8_K blocks (d, qs[256], bsums[16] rebuilt from the quants), and
    return the records' 32-element sums for a separate check."""
    rows = rec.shape[0]
    r = rec.reshape(rows, -1, 288)
    nsb = r.shape[1]
    qs = np.empty((rows, nsb, 256), np.int8)
    for j in range(8):
        for t in range(4):
            off = 64 * (j // 2) + 16 * t + 8 * (j % 2)
            qs[:, :, 32 * j + 8 * t:32 * j + 8 * t + 8] = r[:, :, off:off + 8].view(np.int8)
    d = r[:, :, 272:276].copy().view(np.float32)
    sums = r[:, :, 256:272].copy().view(np.int16)
    bsums = qs.reshape(rows, nsb, 16, 16).astype(np.int32).sum(axis=3).astype(np.int16)
    blocks = np.concatenate([d.view(np.uint8), qs.view(np.uint8), bsums.view(np.uint8)], axis=2)
    return blocks.reshape(rows, nsb * 292), sums


@pytest.mark.parametrize("src", ["golden", "random"])
def test_quantize_q8_K_matvec_records_bitexact(pxq, oracle, golden, src):
    """The matvec's Q8_K records carry exactly the reference's quants, scale
    and 32-element sums (permuted), for every row count 1..8."""
    if src == "golden":
        x = golden["q8_K_x"]
    else:
        rng = np.random.default_rng(5)
        x = (rng.standard_normal((8, 3584)) * 3).astype(np.float32)
        x[1, :256] = 0.0
    for rows in sorted({1, min(8, x.shape[0]), x.shape[0] if x.shape[0] <= 8 else 8}):
        xs = np.ascontiguousarray(x[:rows])
        rec = pxq.quantize_q8_K_matvec(cuda(xs)).cpu().numpy()
        blocks, sums = _records_to_q8_K_blocks(rec)
        want = oracle.quantize_q8_K(xs)
        assert np.array_equal(blocks, want)
        wb = want.reshape(rows, -1, 292)[:, :, 260:292].copy().view(np.int16).astype(np.int32)
        assert np.array_equal(sums.astype(np.int32), wb[:, :, 0::2] + wb[:, :, 1::2])


@pytest.mark.parametrize("name,wtype", [("q8_0", Q8_0), ("q5_K", Q5_K), ("q6_K", Q6_K)])
def test_decode_golden(pxq, golden, name, wtype):
    w = golden[f"w_{name}"]
    want = golden[f"decode_{name}"]
    got = pxq.decode(cuda(w.reshape(-1)), wtype, want.size).cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


# ------------------------------------------------------------------ matmul --

@pytest.mark.parametrize("name,wtype", [("q8_0", Q8_0), ("q5_K", Q5_K), ("q6_K", Q6_K)])
@pytest.mark.parametrize("path", ["matvec", "gemm", "auto"])
def test_matmul_golden(pxq, golden, name, wtype, path):
    w = golden[f"w_{name}"]
    rows, inner = w.shape[0], golden["mm_x"].shape[1]
    W = pxq.Weight(w, wtype, inner, rows)
    y = pxq.matmul(W, cuda(golden["mm_x"]), path=path).cpu().numpy()
    pxq.synchronize()
    W.release()
    assert max_abs_rel(y, golden[f"mm_{name}"]) <= TOL


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K, Q6_K])
@pytest.mark.parametrize("columns", [1, 2, 3, 4, 5, 8])
def test_matvec_vs_oracle(pxq, oracle, wtype, columns):
    rows, inner = 100, 1024
    w = synth.weights_for(wtype, rows, inner, seed=columns)
    x = synth.activations(columns, inner, seed=50 + columns)
    W = pxq.Weight(w, wtype, inner, rows)
    y = pxq.matmul(W, cuda(x), path="matvec").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, wtype, x, rows)
    assert ok and max_abs_rel(y, ref) <= TOL


@pytest.mark.parametrize("wtype", [Q5_K, Q6_K])
@pytest.mark.parametrize("rows", [18944, 9472, 4608, 3584, 200])
@pytest.mark.parametrize("inner,columns", [(256, 1), (768, 3), (3584, 8)])
def test_matvec_kquant_tile_shapes(pxq, oracle, wtype, rows, inner, columns):
    """Every K-quant matvec schedule: on a 148-SM B200 these row counts select
    whole 64-, 32- and 16-row tiles per CTA and the stream-K split; odd
    super-block counts leave the last stage partly empty."""
    rng = np.random.default_rng(rows + inner)
    w = synth.random_q5_K(rows, inner, rng) if wtype == Q5_K else synth.random_q6_K(rows, inner, rng)
    x = synth.activations(columns, inner, seed=columns)
    W = pxq.Weight(w, wtype, inner, rows)
    y = pxq.matmul(W, cuda(x), path="matvec").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, wtype, x, rows)
    assert ok and max_abs_rel(y, ref) <= TOL


@pytest.mark.parametrize("rows", [18944, 9472, 4608, 3584, 200])
@pytest.mark.parametrize("inner,columns", [(256, 1), (768, 3), (3584, 8), (3584, 2)])
def test_matvec_q8_0_streamed_tile_shapes(pxq, oracle, rows, inner, columns):
    """Q8_0 with K a multiple of 256 streams groups of eight raw blocks
    through the TMA-fed kernel: every schedule (whole 64/32-row tiles,
    16-row tiles with the fused quantize, stream-K) against the oracle."""
    w = synth.q8_0_weights(rows, inner, seed=rows + columns)
    x = synth.activations(columns, inner, seed=columns)
    W = pxq.Weight(w, Q8_0, inner, rows)
    y = pxq.matmul(W, cuda(x), path="matvec").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, Q8_0, x, rows)
    assert ok and max_abs_rel(y, ref) <= TOL


@pytest.mark.parametrize("rows,inner", [(300, 96), (4608, 800), (200, 18976)])
@pytest.mark.parametrize("columns", [1, 3, 8])
def test_matvec_q8_0_unaligned_k(pxq, oracle, rows, inner, columns):
    """Q8_0 with K not a multiple of 256 (rows that are no 16-byte multiple):
    the block-walking kernel, with and without the K split."""
    w = synth.q8_0_weights(rows, inner, seed=inner + columns)
    x = synth.activations(columns, inner, seed=columns + 7)
    W = pxq.Weight(w, Q8_0, inner, rows)
    y = pxq.matmul(W, cuda(x), path="matvec").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, Q8_0, x, rows)
    assert ok and max_abs_rel(y, ref) <= TOL


def test_q6_K_golden_past_the_matvec(pxq, golden):
    """Q6_K weights with more activation rows than the matvec takes go to the
    tensor-core GEMM; each output row depends on its own activation row only,
    so the reference build's outputs for the golden rows, repeated, are the
    expected result."""
    w = golden["w_q6_K"]
    rows, inner = w.shape[0], golden["mm_x"].shape[1]
    W = pxq.Weight(w, Q6_K, inner, rows)
    x9 = np.concatenate([golden["mm_x"], golden["mm_x"][:2]])
    want = np.concatenate([golden["mm_q6_K"], golden["mm_q6_K"][:2]])
    for path in ("gemm", "auto"):
        y = pxq.matmul(W, cuda(x9), path=path).cpu().numpy()
        pxq.synchronize()
        assert max_abs_rel(y, want) <= TOL
    W.release()


def test_matvec_scratch_reuse_across_schedules(pxq, oracle):
    """Consecutive calls on one stream share the matvec scratch: activation
    sizes, fused vs separate quantize and whole-tile vs stream-K alternate
    (down-shape 3584x18944: whole 16-row tiles with a separate quantize; a
    200x18944 slice: stream-K, the quantize fused into the matvec at M=1 and
    separate at M=8; QKV-shape whole tiles, fused), and every result must still
    match the oracle."""
    down = synth.random_q5_K(3584, 18944, np.random.default_rng(21))
    qkv = synth.random_q5_K(4608, 3584, np.random.default_rng(22))
    xd = synth.activations(8, 18944, seed=23)
    xq = synth.activations(8, 3584, seed=24)
    Wd = pxq.Weight(down, Q5_K, 18944, 3584)
    Ws = pxq.Weight(down[:200], Q5_K, 18944, 200)
    Wq = pxq.Weight(qkv, Q5_K, 3584, 4608)
    refs = {}
    for W, w, x, m in ((Wd, down, xd, 8), (Ws, down[:200], xd, 1), (Wd, down, xd, 1), (Wq, qkv, xq, 1), (Ws, down[:200], xd, 8),
                       (Wd, down, xd, 2), (Ws, down[:200], xd, 1), (Wd, down, xd, 8), (Wq, qkv, xq, 8), (Wd, down, xd, 1)):
        rows = W.rows
        y = pxq.matmul(W, cuda(x[:m]), path="matvec").cpu().numpy()
        pxq.synchronize()
        key = (rows, m)
        if key not in refs:
            ok, refs[key] = oracle.quant_matmul(w, Q5_K, x[:m], rows)
            assert ok
        assert max_abs_rel(y, refs[key]) <= TOL, key
    Wd.release()
    Ws.release()
    Wq.release()


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K, Q6_K])
@pytest.mark.parametrize("columns,rows,inner", [(9, 48, 512), (130, 260, 512), (259, 520, 768), (128, 256, 2048),
                                                (200, 300, 256)])
def test_gemm_vs_oracle(pxq, oracle, wtype, columns, rows, inner):
    w = synth.weights_for(wtype, rows, inner, seed=rows)
    x = synth.activations(columns, inner, seed=columns)
    W = pxq.Weight(w, wtype, inner, rows)
    y = pxq.matmul(W, cuda(x), path="gemm").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, wtype, x, rows)
    assert ok and max_abs_rel(y, ref) <= TOL


@pytest.mark.parametrize("rows,columns", [(70, 140), (2560, 2048)])
def test_gemm_q8_0_odd_block_count(pxq, oracle, rows, columns):
    # inner = 96: three 32-blocks, the last 64-wide stage is half empty; with
    # 320 output tiles every CTA walks several, so the per-block accumulator
    # slots start a new tile mid-cycle
    inner = 96
    w = synth.q8_0_weights(rows, inner, seed=1)
    x = synth.activations(columns, inner, seed=2)
    W = pxq.Weight(w, Q8_0, inner, rows)
    y = pxq.matmul(W, cuda(x), path="gemm").cpu().numpy()
    pxq.synchronize()
    W.release()
    ok, ref = oracle.quant_matmul(w, Q8_0, x, rows)
    assert ok and max_abs_rel(y, ref) <= TOL


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K, Q6_K])
def test_gemm_block_dots_exact(pxq, oracle, wtype):
    """The tensor-core path's per-block integer dots equal the reference's."""
    rows, inner, columns = 40, 512, 20
    w = synth.weights_for(wtype, rows, inner, seed=3)
    x = synth.activations(columns, inner, seed=4)
    W = pxq.Weight(w, wtype, inner, rows)
    dump = pxq.gemm_block_dots(W, cuda(x)).cpu().numpy()  # [items, columns, rows]
    pxq.synchronize()
    W.release()
    if wtype == Q8_0:
        xq = oracle.quantize_q8_0(x)
        for c in range(columns):
            for r in range(rows):
                want = oracle.block_dots_q8_0(inner, w[r], xq[c])
                assert np.array_equal(dump[:, c, r], want.astype(np.float32))
    elif wtype == Q6_K:
        xq = oracle.quantize_q8_K(x)
        for c in range(columns):
            for r in range(rows):
                s, chunks = oracle.block_dots_q6_K(inner, w[r], xq[c])
                items = dump[:, c, r].reshape(-1, 4)
                assert np.array_equal(items, chunks.astype(np.float32))  # every 64-value chunk, exactly
                assert np.array_equal(items.astype(np.int64).sum(axis=1), s.astype(np.int64))
    else:
        xq = oracle.quantize_q8_K(x)
        nsb = inner // 256
        for c in range(columns):
            for r in range(rows):
                s, m = oracle.block_dots_q5_K(inner, w[r], xq[c])
                items = dump[:, c, r].reshape(nsb, 5)
                assert np.array_equal(items[:, :4].astype(np.int64).sum(axis=1), s.astype(np.int64))
                assert np.all(items == np.round(items))  # every chunk sum is an exact integer
                assert np.array_equal(items[:, 4].astype(np.int64), m.astype(np.int64))


@pytest.mark.parametrize("path,wtype", [("matvec", Q8_0), ("matvec", Q5_K), ("matvec", Q6_K), ("gemm", Q8_0), ("gemm", Q5_K),
                                        ("gemm", Q6_K)])
def test_row_views_ldy_bias(pxq, oracle, path, wtype):
    """tensor_linear_rows-style row ranges, strided output, fused bias."""
    import torch

    rows, inner = 300, 512
    columns = 5 if path == "matvec" else 140
    w = synth.weights_for(wtype, rows, inner, seed=9)
    x = synth.activations(columns, inner, seed=10)
    W = pxq.Weight(w, wtype, inner, rows)
    ok, ref = oracle.quant_matmul(w, wtype, x, rows)
    # counts and strides exercise both epilogues (TMA store: count % 4 == 0 and
    # ldy % 4 == 0; direct stores otherwise)
    for first, count, pad in ((0, 300, 7), (4, 256, 4), (3, 97, 7), (3, 97, 3), (128, 172, 4), (8, 96, 0)):
        bias = torch.linspace(-1, 1, count, device="cuda", dtype=torch.float32)
        out = torch.full((columns, count + pad), float("nan"), device="cuda")
        pxq.matmul(W, cuda(x), row_first=first, row_count=count, bias=bias, out=out, ldy=count + pad, path=path)
        pxq.synchronize()
        got = out.cpu().numpy()
        want = ref[:, first:first + count] + bias.cpu().numpy()[None, :]
        assert max_abs_rel(got[:, :count], want) <= TOL
        assert np.isnan(got[:, count:]).all()  # padding columns untouched
    W.release()


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K])
@pytest.mark.parametrize("columns", [4, 150])
def test_qkv_split_into_separate_outputs(pxq, oracle, wtype, columns):
    """The QKV split of src/inference.cpp:299-313 (tensor_linear, then copying
    the three row ranges of each output row into q, k, v) as one activation
    quantize and three row-view products writing q, k and v directly."""
    H, inner = 192, 512
    w = synth.weights_for(wtype, 3 * H, inner, seed=31)
    x = synth.activations(columns, inner, seed=32)
    W = pxq.Weight(w, wtype, inner, 3 * H)
    a = pxq.Activation(wtype, cuda(x))
    q, k, v = (pxq.matmul_quantized(W, a, row_first=i * H, row_count=H) for i in range(3))
    pxq.synchronize()
    a.release()
    W.release()
    ok, ref = oracle.quant_matmul(w, wtype, x, 3 * H)
    assert ok
    for i, t in enumerate((q, k, v)):
        assert max_abs_rel(t.cpu().numpy(), ref[:, i * H:(i + 1) * H]) <= TOL


def test_host_drop_in_matches_reference_contract(pxq, oracle, golden):
    for name, wtype in (("q8_0", Q8_0), ("q5_K", Q5_K)):
        w = golden[f"w_{name}"]
        handled, y = pxq.quant_matmul(w, wtype, golden["mm_x"], w.shape[0])
        assert handled and max_abs_rel(y, golden[f"mm_{name}"]) <= TOL
    handled, y = pxq.quant_matmul(golden["w_q6_K"], Q6_K, golden["mm_x"], 24)
    assert handled and max_abs_rel(y, golden["mm_q6_K"]) <= TOL  # Q6_K on the matvec
    x9 = np.concatenate([golden["mm_x"], golden["mm_x"][:2]])
    handled, y = pxq.quant_matmul(golden["w_q6_K"], Q6_K, x9, 24)  # and on the GEMM
    assert handled and max_abs_rel(y, np.concatenate([golden["mm_q6_K"], golden["mm_q6_K"][:2]])) <= TOL
    # large-M through the host entry point
    w = synth.q8_0_weights(256, 1024, seed=5)
    x = synth.activations(300, 1024, seed=6)
    handled, y = pxq.quant_matmul(w, Q8_0, x, 256)
    ok, ref = oracle.quant_matmul(w, Q8_0, x, 256)
    assert handled and max_abs_rel(y, ref) <= TOL


@pytest.mark.parametrize("off", [128, 129])  # 16-byte aligned (4-float peer stores, TMA-store local copy) or not
@pytest.mark.parametrize("wtype", [Q8_0, Q5_K, Q6_K])
def test_matmul_scatter_local_destinations(pxq, wtype, off):
    """pxq_matmul_scatter writes each element to every destination at the
    column offset (the N-sharded path's P2P-store GEMM, here with two buffers
    on one GPU): both hold exactly the plain GEMM's output there, and nothing
    outside the rank's columns is touched."""
    import torch

    rows, inner, M, total = 192, 1024, 40, 512
    w = synth.weights_for(wtype, rows, inner, seed=21)
    x = cuda(synth.activations(M, inner, seed=22))
    W = pxq.Weight(w, wtype, inner, rows)
    ref = pxq.matmul(W, x, path="gemm")
    dst = [torch.full((M, total), 7.0, device="cuda") for _ in range(2)]
    pxq.matmul_scatter(W, x, [d.data_ptr() for d in dst], ldy=total, col_offset=off)
    pxq.synchronize()
    W.release()
    for d in dst:
        assert torch.equal(d[:, off:off + rows].contiguous().view(torch.int32), ref.view(torch.int32))
        assert bool((d[:, :off] == 7.0).all()) and bool((d[:, off + rows:] == 7.0).all())
    with pytest.raises(pxq.PxqError):  # the scatter runs on the GEMM path only
        W2 = pxq.Weight(w, wtype, inner, rows)
        try:
            pxq.matmul_scatter(W2, x[:4], [dst[0].data_ptr()], ldy=total, col_offset=off)
        finally:
            W2.release()


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K])
def test_host_matmul_chunked_pipeline(pxq, oracle, wtype):
    """Host-buffer calls with many activation rows run as chunks whose
    uploads, GEMMs and downloads overlap: the result is the one-shot result
    (each output element depends on its own activation row only), and with
    ldy > rows the caller's elements between output rows are left as they were."""
    import ctypes as C

    rows, inner, M = 96, 512, 1300  # chunks of 128, 256, 512 and 404 rows
    w = synth.weights_for(wtype, rows, inner, seed=41)
    x = synth.activations(M, inner, seed=42)
    ok, ref = oracle.quant_matmul(w, wtype, x, rows)
    assert ok
    handled, y = pxq.quant_matmul(w, wtype, x, rows)
    assert handled and max_abs_rel(y, ref) <= TOL
    W = pxq.Weight(w, wtype, inner, rows)
    ldy = rows + 5
    out = np.full((M, ldy), -3.0, dtype=np.float32)
    rc = pxq.load().pxq_matmul_host(W.handle, 0, rows, x.ctypes.data_as(C.c_void_p), M, out.ctypes.data_as(C.c_void_p), ldy)
    W.release()
    assert rc == pxq.OK
    assert np.array_equal(out[:, :rows].view(np.uint32), y.view(np.uint32))
    assert bool((out[:, rows:] == -3.0).all())


def test_gather_shards(pxq):
    import torch

    shards, columns, shard_rows = 4, 33, 20
    src = torch.arange(shards * columns * shard_rows, dtype=torch.float32, device="cuda")
    out = pxq.gather_shards(src, shards, columns, shard_rows)
    want = src.view(shards, columns, shard_rows).permute(1, 0, 2).reshape(columns, shards * shard_rows)
    assert torch.equal(out, want)


# ------------------------------------------------------------ gated matmul --

def _silu_gate(g, u):
    # tensor_silu then tensor_gate (src/tensor.cpp:199-208, :334-345), in fp32
    g = g.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32) * u.astype(np.float32)


@pytest.mark.parametrize("wtype", [Q8_0, Q5_K, Q6_K])
@pytest.mark.parametrize("rows,columns", [(192, 1), (64, 5), (320, 8), (192, 9), (320, 140), (2048, 300)])
def test_matmul_gated_vs_oracle(pxq, oracle, wtype, rows, columns):
    """pxq_matmul_gated = the callers' gate/up linears, tensor_silu, tensor_gate:
    the matvec path (<= 8 rows) and the GEMM with the gate in its epilogue
    (the repack interleaves gate and up rows in 64-row groups)."""
    inner = 512
    g = synth.weights_for(wtype, rows, inner, seed=21)
    u = synth.weights_for(wtype, rows, inner, seed=22)
    x = synth.activations(columns, inner, seed=23)
    W = pxq.GatedWeight(g, u, wtype, inner, rows)
    y = pxq.matmul_gated(W, cuda(x)).cpu().numpy()
    pxq.synchronize()
    okg, G = oracle.quant_matmul(g, wtype, x, rows)
    oku, U = oracle.quant_matmul(u, wtype, x, rows)
    assert okg and oku
    assert max_abs_rel(y, _silu_gate(G, U)) <= TOL
    # a strided output leaves the padding untouched
    import torch

    out = torch.full((columns, rows + 5), float("nan"), device="cuda")
    pxq.matmul_gated(W, cuda(x), out=out, ldy=rows + 5)
    pxq.synchronize()
    got = out.cpu().numpy()
    assert max_abs_rel(got[:, :rows], _silu_gate(G, U)) <= TOL and np.isnan(got[:, rows:]).all()
    # the gated weight serves pxq_matmul_gated only
    with pytest.raises(pxq.PxqError) as err:
        pxq.matmul(W, cuda(x))
    assert err.value.code == pxq.ERR_INVALID
    W.release()


@pytest.mark.parametrize("columns", [1, 8])
def test_matmul_gated_q8_0_unaligned_k(pxq, oracle, columns):
    """Q8_0 gated pair with K not a multiple of 256: the block-walking matvec
    over both halves, then the silu(gate) * up epilogue kernel."""
    rows, inner = 192, 800
    g = synth.weights_for(Q8_0, rows, inner, seed=24)
    u = synth.weights_for(Q8_0, rows, inner, seed=25)
    x = synth.activations(columns, inner, seed=26)
    W = pxq.GatedWeight(g, u, Q8_0, inner, rows)
    y = pxq.matmul_gated(W, cuda(x)).cpu().numpy()
    pxq.synchronize()
    W.release()
    okg, G = oracle.quant_matmul(g, Q8_0, x, rows)
    oku, U = oracle.quant_matmul(u, Q8_0, x, rows)
    assert okg and oku and max_abs_rel(y, _silu_gate(G, U)) <= TOL

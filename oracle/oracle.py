"""ctypes loaders for the CPU checkers built by oracle/Makefile.

TEST INFRASTRUCTURE ONLY: imported by tests/, by the smoke check in
__graft_entry__.py and by the cpu_baseline / reference leg of bench.py.  The
product package never imports this module.

Two libraries, same calling convention (numpy in, numpy out):

* ``Oracle`` wraps ``_build/libpxq_oracle.so``, the scalar C restatement of
  Pixelina's quantize/dot/matmul (``pxq_oracle.c``, each function cites the
  reference line it restates).
* ``Reference`` wraps ``_ref/libpixref.so``, Pixelina's own CPU kernels
  compiled from the reference sources (``ref_shim.cpp``).  It exists only
  where the reference tree was present at build time (or where the built .so
  was carried along).
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libpxq_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libpixref.so")

TYPE_Q8_0 = 8
TYPE_Q5_K = 13
TYPE_Q6_K = 14
Q8_0_BYTES = 34
Q8_K_BYTES = 292
Q5_K_BYTES = 176
Q6_K_BYTES = 210
BLOCK_BYTES = {TYPE_Q8_0: Q8_0_BYTES, TYPE_Q5_K: Q5_K_BYTES, TYPE_Q6_K: Q6_K_BYTES}
BLOCK_ELEMS = {TYPE_Q8_0: 32, TYPE_Q5_K: 256, TYPE_Q6_K: 256}


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class _Lib:
    prefix = ""

    def __init__(self, path: str):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.path = path
        self.lib = C.CDLL(path)
        p = self.prefix
        L = self.lib
        for name in ("quantize_q8_0", "quantize_q8_K"):
            f = getattr(L, p + ("quantize_row_" if p == "pxo_" else "quantize_") + name.split("_", 1)[1])
            f.argtypes = [C.c_void_p, C.c_void_p, C.c_int64]
            f.restype = None
            setattr(self, "_" + name, f)
        for t in ("q8_0", "q5_K", "q6_K"):
            f = getattr(L, p + "dot_" + t)
            f.argtypes = [C.c_int, C.c_void_p, C.c_void_p]
            f.restype = C.c_float
            setattr(self, "_dot_" + t, f)
        self._qmm = getattr(L, p + "quant_matmul")
        self._qmm.argtypes = [C.c_void_p, C.c_uint32, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t]
        self._qmm.restype = C.c_int
        self._decode = getattr(L, p + "decode")
        self._decode.argtypes = [C.c_void_p, C.c_uint32, C.c_size_t, C.c_void_p]
        self._decode.restype = None
        self._wbytes = getattr(L, p + "weight_bytes")
        self._wbytes.argtypes = [C.c_uint64, C.c_uint64, C.c_uint32]
        self._wbytes.restype = C.c_uint64

    # -- quantize: fp32 [rows, inner] -> uint8 [rows, blocks*bytes]
    def quantize_q8_0(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
        rows, inner = x.shape
        out = np.zeros((rows, inner // 32 * Q8_0_BYTES), dtype=np.uint8)
        for r in range(rows):
            self._quantize_q8_0(_ptr(x[r]), _ptr(out[r]), inner)
        return out

    def quantize_q8_K(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, x.shape[-1])
        rows, inner = x.shape
        out = np.zeros((rows, inner // 256 * Q8_K_BYTES), dtype=np.uint8)
        for r in range(rows):
            self._quantize_q8_K(_ptr(x[r]), _ptr(out[r]), inner)
        return out

    def dot(self, wtype: int, inner: int, wrow: np.ndarray, arow: np.ndarray) -> float:
        f = {TYPE_Q8_0: self._dot_q8_0, TYPE_Q5_K: self._dot_q5_K, TYPE_Q6_K: self._dot_q6_K}[wtype]
        wrow = np.ascontiguousarray(wrow, dtype=np.uint8)
        arow = np.ascontiguousarray(arow, dtype=np.uint8)
        return float(f(inner, _ptr(wrow), _ptr(arow)))

    def quant_matmul(self, weights: np.ndarray, wtype: int, x: np.ndarray, rows: int):
        """cpu_quant_matmul: returns (handled, Y[columns, rows])."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        columns, inner = x.shape
        w = np.ascontiguousarray(weights, dtype=np.uint8)
        y = np.zeros((columns, rows), dtype=np.float32)
        ok = self._qmm(_ptr(w), wtype, _ptr(x), _ptr(y), rows, columns, inner)
        return bool(ok), y

    def decode(self, data: np.ndarray, wtype: int, count: int) -> np.ndarray:
        data = np.ascontiguousarray(data, dtype=np.uint8)
        out = np.zeros(count, dtype=np.float32)
        self._decode(_ptr(data), wtype, count, _ptr(out))
        return out

    def weight_bytes(self, inner: int, rows: int, wtype: int) -> int:
        return int(self._wbytes(inner, rows, wtype))


class Oracle(_Lib):
    """The C restatement (oracle/pxq_oracle.c)."""

    prefix = "pxo_"

    def __init__(self, path: str = ORACLE_SO):
        super().__init__(path)
        L = self.lib
        L.pxo_block_dots_q8_0.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]
        L.pxo_block_dots_q8_0.restype = None
        L.pxo_block_dots_q5_K.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.pxo_block_dots_q5_K.restype = None
        L.pxo_block_dots_q6_K.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]
        L.pxo_block_dots_q6_K.restype = None
        L.pxo_float_to_half.argtypes = [C.c_float]
        L.pxo_float_to_half.restype = C.c_uint16
        L.pxo_half_to_float.argtypes = [C.c_uint16]
        L.pxo_half_to_float.restype = C.c_float

    def block_dots_q8_0(self, inner: int, wrow: np.ndarray, arow: np.ndarray) -> np.ndarray:
        out = np.zeros(inner // 32, dtype=np.int32)
        self.lib.pxo_block_dots_q8_0(inner, _ptr(np.ascontiguousarray(wrow)), _ptr(np.ascontiguousarray(arow)), _ptr(out))
        return out

    def block_dots_q5_K(self, inner: int, wrow: np.ndarray, arow: np.ndarray):
        s = np.zeros(inner // 256, dtype=np.int32)
        m = np.zeros(inner // 256, dtype=np.int32)
        self.lib.pxo_block_dots_q5_K(inner, _ptr(np.ascontiguousarray(wrow)), _ptr(np.ascontiguousarray(arow)), _ptr(s), _ptr(m))
        return s, m

    def block_dots_q6_K(self, inner: int, wrow: np.ndarray, arow: np.ndarray):
        """(super-block dots [nsb], 64-value chunk dots [nsb, 4]), exact int32."""
        s = np.zeros(inner // 256, dtype=np.int32)
        ch = np.zeros(inner // 64, dtype=np.int32)
        self.lib.pxo_block_dots_q6_K(inner, _ptr(np.ascontiguousarray(wrow)), _ptr(np.ascontiguousarray(arow)), _ptr(s), _ptr(ch))
        return s, ch.reshape(-1, 4)

    def float_to_half(self, f: float) -> int:
        return int(self.lib.pxo_float_to_half(f))

    def half_to_float(self, h: int) -> float:
        return float(self.lib.pxo_half_to_float(h))


class Reference(_Lib):
    """Pixelina's own CPU kernels (oracle/_ref/libpixref.so)."""

    prefix = "pixref_"

    def __init__(self, path: str = REF_SO):
        super().__init__(path)
        self.lib.pixref_set_threads.argtypes = [C.c_size_t]
        self.lib.pixref_set_threads.restype = None
        self.lib.pixref_thread_count.argtypes = []
        self.lib.pixref_thread_count.restype = C.c_size_t

    def set_threads(self, n: int) -> None:
        self.lib.pixref_set_threads(n)

    def attention(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, heads: int, kv_heads: int, ranges, query_offset: int = 0):
        """tensor_attention's range overload; ranges [(begin, end, key_end, causal)].  None when it rejects the arguments."""
        q, k, v = (np.ascontiguousarray(a, dtype=np.float32) for a in (q, k, v))
        d = q.shape[1] // heads
        out = np.zeros_like(q)
        n = len(ranges)
        arrs = [np.array([r[i] for r in ranges], dtype=np.uint64) for i in range(3)]
        cz = np.array([1 if r[3] else 0 for r in ranges], dtype=np.int32)
        fn = self.lib.pixref_attention
        fn.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                       C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_size_t, C.c_void_p]
        fn.restype = C.c_int
        ok = fn(_ptr(q), q.shape[0], _ptr(k), _ptr(v), k.shape[0], heads, kv_heads, d, _ptr(arrs[0]), _ptr(arrs[1]), _ptr(arrs[2]),
                _ptr(cz), n, query_offset, _ptr(out))
        return out if ok else None

    def gguf_list(self, path: str, cap: int = 256):
        """PixModelFile::open on `path`: (result code, tensors in name order, metadata key count)."""

        class T(C.Structure):
            _fields_ = [("name", C.c_char * 256), ("type", C.c_uint32), ("rank", C.c_uint32), ("shape", C.c_uint64 * 5),
                        ("offset", C.c_uint64), ("bytes", C.c_uint64)]

        buf = (T * cap)()
        count, keys = C.c_size_t(0), C.c_size_t(0)
        fn = self.lib.pixref_gguf_list
        fn.argtypes = [C.c_char_p, C.c_void_p, C.c_size_t, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]
        fn.restype = C.c_int
        rc = fn(path.encode(), C.cast(buf, C.c_void_p), cap, C.byref(count), C.byref(keys))
        tensors = [{"name": buf[i].name.decode(), "type": int(buf[i].type), "shape": [int(v) for v in buf[i].shape[:buf[i].rank]],
                    "offset": int(buf[i].offset), "bytes": int(buf[i].bytes)} for i in range(min(count.value, cap))]
        return int(rc), tensors, int(keys.value)

    def thread_count(self) -> int:
        return int(self.lib.pixref_thread_count())


def oracle_available() -> bool:
    return os.path.exists(ORACLE_SO)


def reference_available() -> bool:
    return os.path.exists(REF_SO)


def q8_0_gemm_reference_blocks(oracle: Oracle, w_blocks: np.ndarray, xq_blocks: np.ndarray, inner: int) -> np.ndarray:
    """All exact int32 Q8_0 block dots, shape [columns, rows, blocks]."""
    rows = w_blocks.shape[0]
    cols = xq_blocks.shape[0]
    out = np.zeros((cols, rows, inner // 32), dtype=np.int32)
    for c in range(cols):
        for r in range(rows):
            out[c, r] = oracle.block_dots_q8_0(inner, w_blocks[r], xq_blocks[c])
    return out

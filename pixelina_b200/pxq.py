"""Python host mirror of the pxq C ABI (include/pxq.h).

The operator surface follows Pixelina's matmul boundary (paths within the
Pixelina source tree):

* ``quant_matmul``   -- cpu_quant_matmul (src/kernels_quant.cpp:369-412):
  host buffers in, host buffer out, ``(handled, output)`` like its bool.
* ``Weight``         -- a device-resident GGUF tensor, the Vulkan backend's
  weight cache entry (src/backend_vulkan.cpp:742-758).
* ``matmul``         -- cpu_matmul / vulkan_matmul (src/backend_cpu.cpp:103,
  src/backend_vulkan.cpp:1083) on device tensors, with the row-range view of
  tensor_linear_rows (src/tensor.cpp:529-544) and the bias of tensor_linear
  (src/tensor.cpp:156-172).
* ``quantize_q8_0`` / ``quantize_q8_K`` / ``decode`` -- the reference's
  quantizers and cpu_decode on device buffers.

torch is used only for device memory and streams.  Everything computes in
libpxq.so; importing this module on a machine without the built library or
without a B200 raises instead of falling back to any CPU path.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libpxq.so")

OK = 0
ERR_INVALID = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_NO_MEMORY = 4
ERR_NO_DEVICE = 5
ERR_DEVICE_STATUS = 6
ERR_IO = 7
ERR_FORMAT = 8
ERR_TIMEOUT = 9

TYPE_Q8_0 = 8
TYPE_Q5_K = 13
TYPE_Q6_K = 14
BLOCK_ELEMS = {TYPE_Q8_0: 32, TYPE_Q5_K: 256, TYPE_Q6_K: 256}
BLOCK_BYTES = {TYPE_Q8_0: 34, TYPE_Q5_K: 176, TYPE_Q6_K: 210}
Q8_0_BYTES = 34
Q8_K_BYTES = 292

# name -> (restype, argtypes); must list exactly the functions of include/pxq.h
_vp, _sz, _u32, _u64, _i = C.c_void_p, C.c_size_t, C.c_uint32, C.c_uint64, C.c_int
SIGNATURES = {
    "pxq_version": (_i, []),
    "pxq_last_error": (C.c_char_p, []),
    "pxq_init": (_i, [_i]),
    "pxq_weight_bytes": (_u64, [_u64, _u64, _u32]),
    "pxq_quantize_q8_0": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "pxq_quantize_q8_K": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "pxq_quantize_q8_K_matvec": (_i, [_vp, _vp, _sz, _sz, _vp]),
    "pxq_decode": (_i, [_vp, _u32, _sz, _vp, _vp]),
    "pxq_weight_upload": (_i, [_vp, _i, _u32, _sz, _sz, C.c_char_p, C.POINTER(_vp)]),
    "pxq_weight_upload_gated": (_i, [_vp, _vp, _i, _u32, _sz, _sz, C.c_char_p, C.POINTER(_vp)]),
    "pxq_matmul_gated": (_i, [_vp, _vp, _sz, _vp, _sz, _vp]),
    "pxq_weight_release": (_i, [_vp]),
    "pxq_weight_cache_clear": (_i, []),
    "pxq_weight_cache_limit": (_i, [_u64]),
    "pxq_weight_cache_usage": (_i, [C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u64)]),
    "pxq_matmul": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _sz, _vp, _vp]),
    "pxq_matvec": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _sz, _vp, _vp]),
    "pxq_gemm": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _sz, _vp, _vp]),
    "pxq_quant_matmul": (_i, [_vp, _u32, _vp, _vp, _sz, _sz, _sz]),
    "pxq_matmul_host": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _sz]),
    "pxq_synchronize": (_i, [_vp]),
    "pxq_gather_shards": (_i, [_vp, _sz, _sz, _sz, _vp, _sz, _vp]),
    "pxq_matmul_scatter": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _sz, _sz, _sz, _vp]),
    "pxq_ipc_alloc": (_i, [_sz, _vp, _vp]),
    "pxq_ipc_free": (_i, [_vp]),
    "pxq_ipc_open": (_i, [_vp, _vp]),
    "pxq_ipc_close": (_i, [_vp]),
    "pxq_gemm_block_dots": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _vp]),
    "pxq_activation_quantize": (_i, [_u32, _vp, _sz, _sz, C.POINTER(_vp), _vp]),
    "pxq_matmul_quantized": (_i, [_vp, _sz, _sz, _vp, _vp, _sz, _vp, _vp]),
    "pxq_activation_release": (_i, [_vp, _vp]),
    "pxq_kernel_launches": (_u64, []),
    "pxq_matvec_noalloc": (_i, [_vp, _sz, _sz, _vp, _sz, _vp, _sz, _vp, _vp]),
    "pxq_debug_matvec_stall": (_i, [_vp, _vp, _sz, _vp, _i, _vp]),
    "pxq_comm_unique_id": (_i, [_vp]),
    "pxq_comm_init": (_i, [_vp, _i, _i, _i, C.POINTER(_vp)]),
    "pxq_comm_size": (_i, [_vp, C.POINTER(_i), C.POINTER(_i)]),
    "pxq_comm_barrier": (_i, [_vp]),
    "pxq_comm_synchronize": (_i, [_vp, _vp]),
    "pxq_comm_destroy": (_i, [_vp]),
    "pxq_sharded_output_create": (_i, [_vp, _sz, _sz, C.POINTER(_vp), C.POINTER(_vp)]),
    "pxq_sharded_output_destroy": (_i, [_vp]),
    "pxq_sharded_matmul": (_i, [_vp, _vp, _sz, _vp, _sz, _vp, _vp, _sz, _vp]),
    "pxq_sharded_matmul_host": (_i, [_vp, _vp, _sz, _vp, _sz, _sz, _vp]),
    "pxq_attention": (_i, [_vp, _sz, _vp, _vp, _sz, _sz, _sz, _sz, _vp, _sz, _sz, _vp, _vp]),
    "pxq_gguf_open": (_i, [C.c_char_p, C.POINTER(_vp)]),
    "pxq_gguf_close": (_i, [_vp]),
    "pxq_gguf_tensor_count": (_sz, [_vp]),
    "pxq_gguf_metadata_count": (_sz, [_vp]),
    "pxq_gguf_data": (_vp, [_vp]),
    "pxq_gguf_tensor_at": (_i, [_vp, _sz, _vp]),
    "pxq_gguf_find": (_i, [_vp, C.c_char_p, _vp]),
    "pxq_gguf_upload": (_i, [_vp, C.c_char_p, _sz, _sz, C.POINTER(_vp)]),
    "pxq_gguf_upload_gated": (_i, [_vp, C.c_char_p, _sz, C.c_char_p, _sz, _sz, C.POINTER(_vp)]),
}


class GGUFTensor(C.Structure):
    """pxq_gguf_tensor (include/pxq.h)."""

    _fields_ = [("name", C.c_char_p), ("type", C.c_uint32), ("rank", C.c_uint32), ("shape", C.c_uint64 * 5),
                ("offset", C.c_uint64), ("bytes", C.c_uint64)]

    def as_dict(self) -> dict:
        return {"name": self.name.decode(), "type": int(self.type), "shape": [int(v) for v in self.shape[:self.rank]],
                "offset": int(self.offset), "bytes": int(self.bytes)}


class PxqError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"pxq error {code}: {msg}")
        self.code = code


_lib = None


def load(path: str = LIB_PATH):
    """Load libpxq.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(f"{path} is missing: build it with `python -c 'import __graft_entry__ as g; g.build()'`")
    lib = C.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


def _check(rc: int) -> None:
    if rc != OK:
        raise PxqError(rc, load().pxq_last_error().decode(errors="replace"))


def last_error() -> str:
    return load().pxq_last_error().decode(errors="replace")


def weight_bytes(inner: int, rows: int, wtype: int) -> int:
    return int(load().pxq_weight_bytes(inner, rows, wtype))


# ------------------------------------------------------------ device side ---

def _torch():
    import torch  # noqa: WPS433 (device memory and streams only)

    return torch


def _stream_ptr(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return C.c_void_p(s.cuda_stream)


def _ptr(t) -> C.c_void_p:
    return C.c_void_p(t.data_ptr()) if t is not None else C.c_void_p(0)


def init(device: int = 0) -> None:
    torch = _torch()
    torch.cuda.set_device(device)
    _check(load().pxq_init(device))


def quantize_q8_0(x, stream=None):
    """fp32 [rows, inner] cuda tensor -> uint8 [rows, inner/32*34] GGUF Q8_0 blocks."""
    torch = _torch()
    x = x.contiguous()
    rows, inner = x.shape
    out = torch.empty((rows, inner // 32 * Q8_0_BYTES), dtype=torch.uint8, device=x.device)
    _check(load().pxq_quantize_q8_0(_ptr(x), _ptr(out), rows, inner, _stream_ptr(stream)))
    return out


def quantize_q8_K(x, stream=None):
    """fp32 [rows, inner] cuda tensor -> uint8 [rows, inner/256*292] Q8_K blocks."""
    torch = _torch()
    x = x.contiguous()
    rows, inner = x.shape
    out = torch.empty((rows, inner // 256 * Q8_K_BYTES), dtype=torch.uint8, device=x.device)
    _check(load().pxq_quantize_q8_K(_ptr(x), _ptr(out), rows, inner, _stream_ptr(stream)))
    return out


Q8K_MATVEC_BYTES = 288


def quantize_q8_K_matvec(x, stream=None):
    """fp32 [rows <= 8, inner] cuda tensor -> uint8 [rows, inner/256*288] matvec
    records (the Q8_K quants, permuted, plus 32-element sums and d)."""
    torch = _torch()
    x = x.contiguous()
    rows, inner = x.shape
    out = torch.empty((rows, inner // 256 * Q8K_MATVEC_BYTES), dtype=torch.uint8, device=x.device)
    _check(load().pxq_quantize_q8_K_matvec(_ptr(x), _ptr(out), rows, inner, _stream_ptr(stream)))
    return out


def decode(data, wtype: int, count: int, stream=None):
    torch = _torch()
    out = torch.empty(count, dtype=torch.float32, device=data.device)
    _check(load().pxq_decode(_ptr(data), wtype, count, _ptr(out), _stream_ptr(stream)))
    return out


class Weight:
    """A GGUF weight tensor resident on the current device."""

    def __init__(self, data, wtype: int, inner: int, rows: int, key: Optional[str] = None):
        lib = load()
        self.wtype, self.inner, self.rows = wtype, inner, rows
        handle = C.c_void_p()
        if hasattr(data, "data_ptr"):  # torch tensor (host or device)
            on_dev = 1 if data.is_cuda else 0
            ptr = C.c_void_p(data.data_ptr())
            self._keep = data
        else:
            arr = np.ascontiguousarray(data, dtype=np.uint8)
            on_dev, ptr = 0, arr.ctypes.data_as(C.c_void_p)
            self._keep = arr
        kb = key.encode() if key else None
        _check(lib.pxq_weight_upload(ptr, on_dev, wtype, inner, rows, kb, C.byref(handle)))
        self.handle = handle
        self._keep = None

    def release(self) -> None:
        if self.handle:
            _check(load().pxq_weight_release(self.handle))
            self.handle = C.c_void_p()


class GatedWeight:
    """The gate and up projections of a gated feed-forward, resident on the
    current device as one weight (pxq_weight_upload_gated)."""

    def __init__(self, gate, up, wtype: int, inner: int, rows: int, key: Optional[str] = None):
        lib = load()
        self.wtype, self.inner, self.rows = wtype, inner, rows
        keep, ptrs, on_dev = [], [], 0
        for data in (gate, up):
            if hasattr(data, "data_ptr"):
                on_dev = 1 if data.is_cuda else 0
                ptrs.append(C.c_void_p(data.data_ptr()))
                keep.append(data)
            else:
                arr = np.ascontiguousarray(data, dtype=np.uint8)
                ptrs.append(arr.ctypes.data_as(C.c_void_p))
                keep.append(arr)
        handle = C.c_void_p()
        kb = key.encode() if key else None
        _check(lib.pxq_weight_upload_gated(ptrs[0], ptrs[1], on_dev, wtype, inner, rows, kb, C.byref(handle)))
        self.handle = handle

    def release(self) -> None:
        if self.handle:
            _check(load().pxq_weight_release(self.handle))
            self.handle = C.c_void_p()


class AttentionRange(C.Structure):
    """pxq_attention_range (include/pxq.h)."""

    _fields_ = [("query_begin", C.c_size_t), ("query_end", C.c_size_t), ("key_end", C.c_size_t), ("causal", C.c_int)]


def attention(q, k, v, heads: int, kv_heads: int, ranges=None, query_offset: int = 0, causal: bool = False, out=None,
              stream=None):
    """tensor_attention on device fp32 tensors q [rows][heads*d], k, v [keys][kv_heads*d].
    ranges: [(query_begin, query_end, key_end, causal)] (the second overload);
    None: one range over all rows and keys with `causal` (the first overload)."""
    torch = _torch()
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    rows, keys = q.shape[0], k.shape[0]
    d = q.shape[1] // heads
    if ranges is None:
        ranges = [(0, rows, keys, causal)]
    arr = (AttentionRange * len(ranges))(*[AttentionRange(b, e, ke, 1 if c else 0) for b, e, ke, c in ranges])
    if out is None:
        out = torch.empty_like(q)
    _check(load().pxq_attention(_ptr(q), rows, _ptr(k), _ptr(v), keys, heads, kv_heads, d, C.cast(arr, C.c_void_p), len(ranges),
                                query_offset, _ptr(out), _stream_ptr(stream)))
    return out


class _Uploaded:
    """A weight uploaded from a model file (pxq_gguf_upload*)."""

    def __init__(self, handle, wtype: int, inner: int, rows: int):
        self.handle, self.wtype, self.inner, self.rows = handle, wtype, inner, rows

    def release(self) -> None:
        if self.handle:
            _check(load().pxq_weight_release(self.handle))
            self.handle = C.c_void_p()


class GGUF:
    """A GGUF model file opened with pxq_gguf_open (a read-only mapping)."""

    def __init__(self, path: str):
        h = C.c_void_p()
        _check(load().pxq_gguf_open(path.encode(), C.byref(h)))
        self.handle, self.path = h, path

    def close(self) -> None:
        if self.handle:
            load().pxq_gguf_close(self.handle)
            self.handle = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def metadata_count(self) -> int:
        return int(load().pxq_gguf_metadata_count(self.handle))

    def tensors(self) -> list:
        lib = load()
        out = []
        for i in range(int(lib.pxq_gguf_tensor_count(self.handle))):
            t = GGUFTensor()
            _check(lib.pxq_gguf_tensor_at(self.handle, i, C.byref(t)))
            out.append(t.as_dict())
        return out

    def find(self, name: str) -> dict:
        t = GGUFTensor()
        _check(load().pxq_gguf_find(self.handle, name.encode(), C.byref(t)))
        return t.as_dict()

    def upload(self, name: str, row_first: int = 0, row_count: int = 0) -> _Uploaded:
        t = self.find(name)
        rows = 1
        for v in t["shape"][1:]:
            rows *= v
        h = C.c_void_p()
        _check(load().pxq_gguf_upload(self.handle, name.encode(), row_first, row_count, C.byref(h)))
        return _Uploaded(h, t["type"], t["shape"][0], row_count or rows - row_first)

    def upload_gated(self, gate: str, gate_first: int, up: str, up_first: int, rows: int) -> _Uploaded:
        t = self.find(gate)
        h = C.c_void_p()
        _check(load().pxq_gguf_upload_gated(self.handle, gate.encode(), gate_first, up.encode(), up_first, rows, C.byref(h)))
        return _Uploaded(h, t["type"], t["shape"][0], rows)


def matmul_gated(w: GatedWeight, x, out=None, ldy: Optional[int] = None, stream=None):
    """Y[c, r] = silu(x[c] . gate[r]) * (x[c] . up[r]) on the device."""
    torch = _torch()
    x = x.contiguous()
    columns, inner = x.shape
    if inner != w.inner:
        raise ValueError(f"input has {inner} features, weight expects {w.inner}")
    if out is None:
        out = torch.empty((columns, w.rows), dtype=torch.float32, device=x.device)
        ldy = w.rows
    elif ldy is None:
        ldy = out.stride(0)
    _check(load().pxq_matmul_gated(w.handle, _ptr(x), columns, _ptr(out), ldy, _stream_ptr(stream)))
    return out


def matmul(w: Weight, x, row_first: int = 0, row_count: Optional[int] = None, bias=None, out=None, ldy: Optional[int] = None,
           path: str = "auto", stream=None):
    """Y[c, r] = sum_k x[c, k] * W[row_first + r, k] (+ bias[r]) on the device."""
    torch = _torch()
    x = x.contiguous()
    columns, inner = x.shape
    if inner != w.inner:
        raise ValueError(f"input has {inner} features, weight expects {w.inner}")
    rc = w.rows - row_first if row_count is None else row_count
    if out is None:
        out = torch.empty((columns, rc), dtype=torch.float32, device=x.device)
        ldy = rc
    elif ldy is None:
        ldy = out.stride(0)
    fn = {"auto": load().pxq_matmul, "matvec": load().pxq_matvec, "gemm": load().pxq_gemm}[path]
    _check(fn(w.handle, row_first, rc, _ptr(x), columns, _ptr(out), ldy, _ptr(bias), _stream_ptr(stream)))
    return out


def gemm_block_dots(w: Weight, x, row_first: int = 0, row_count: Optional[int] = None, stream=None):
    """Exact per-block dots from the tensor-core GEMM: [items, columns, rows]."""
    torch = _torch()
    x = x.contiguous()
    columns, inner = x.shape
    rc = w.rows - row_first if row_count is None else row_count
    items = {TYPE_Q8_0: inner // 32, TYPE_Q5_K: 5 * (inner // 256), TYPE_Q6_K: 4 * (inner // 256)}[w.wtype]
    dump = torch.zeros((items, columns, rc), dtype=torch.float32, device=x.device)
    _check(load().pxq_gemm_block_dots(w.handle, row_first, rc, _ptr(x), columns, _ptr(dump), _stream_ptr(stream)))
    return dump


class Activation:
    """An activation quantized once for weights of one type (pxq_activation)."""

    def __init__(self, wtype: int, x, stream=None):
        self.x = x.contiguous()
        self.columns, self.inner = self.x.shape
        self.wtype = wtype
        h = C.c_void_p()
        _check(load().pxq_activation_quantize(wtype, _ptr(self.x), self.columns, self.inner, C.byref(h),
                                              _stream_ptr(stream)))
        self.handle = h

    def release(self, stream=None) -> None:
        if self.handle:
            _check(load().pxq_activation_release(self.handle, _stream_ptr(stream)))
            self.handle = C.c_void_p()


def matmul_quantized(w: Weight, a: Activation, row_first: int = 0, row_count: Optional[int] = None, bias=None, out=None,
                     ldy: Optional[int] = None, stream=None):
    torch = _torch()
    rc = w.rows - row_first if row_count is None else row_count
    if out is None:
        out = torch.empty((a.columns, rc), dtype=torch.float32, device=a.x.device)
        ldy = rc
    elif ldy is None:
        ldy = out.stride(0)
    _check(load().pxq_matmul_quantized(w.handle, row_first, rc, a.handle, _ptr(out), ldy, _ptr(bias), _stream_ptr(stream)))
    return out


def cache_limit(nbytes: int) -> None:
    """pxq_weight_cache_limit: the weight cache's budget on this device (0: default)."""
    _check(load().pxq_weight_cache_limit(nbytes))


def cache_usage() -> tuple[int, int, int]:
    """pxq_weight_cache_usage: (cached bytes, budget, entries) on this device."""
    b, l, n = C.c_uint64(), C.c_uint64(), C.c_uint64()
    _check(load().pxq_weight_cache_usage(C.byref(b), C.byref(l), C.byref(n)))
    return b.value, l.value, n.value


def kernel_launches() -> int:
    return int(load().pxq_kernel_launches())


def gather_shards(src, shards: int, columns: int, shard_rows: int, out=None, stream=None):
    torch = _torch()
    if out is None:
        out = torch.empty((columns, shards * shard_rows), dtype=torch.float32, device=src.device)
    _check(load().pxq_gather_shards(_ptr(src), shards, columns, shard_rows, _ptr(out), out.stride(0), _stream_ptr(stream)))
    return out


IPC_HANDLE_BYTES = 64


class IpcBuffer:
    """fp32 device buffer [rows][cols] that other processes of the node can
    map (pxq_ipc_alloc); ``handle`` is its 64-byte CUDA IPC handle and
    ``tensor`` a torch view of it on this device."""

    def __init__(self, rows: int, cols: int):
        torch = _torch()
        ptr, handle = C.c_void_p(), (C.c_uint8 * IPC_HANDLE_BYTES)()
        _check(load().pxq_ipc_alloc(rows * cols * 4, C.byref(ptr), C.cast(handle, C.c_void_p)))
        self.ptr, self.handle, self.shape = ptr.value, bytes(handle), (rows, cols)
        self.tensor = torch.as_tensor(_CudaArray(self.ptr, self.shape), device="cuda")

    def free(self) -> None:
        if self.ptr:
            self.tensor = None
            _check(load().pxq_ipc_free(C.c_void_p(self.ptr)))
            self.ptr = None


class IpcPeer:
    """Another process's IpcBuffer opened in this one (pxq_ipc_open)."""

    def __init__(self, handle: bytes):
        ptr = C.c_void_p()
        buf = (C.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(handle)
        _check(load().pxq_ipc_open(C.cast(buf, C.c_void_p), C.byref(ptr)))
        self.ptr = ptr.value

    def close(self) -> None:
        if self.ptr:
            _check(load().pxq_ipc_close(C.c_void_p(self.ptr)))
            self.ptr = None


class _CudaArray:
    """Minimal __cuda_array_interface__ over a raw fp32 device pointer."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": "<f4", "data": (ptr, False), "version": 2}


def matmul_scatter(W: "Weight", x, dst_ptrs, ldy: int, col_offset: int, row_first: int = 0, row_count=None, stream=None):
    """pxq_matmul_scatter: rows [row_first, row_first + row_count) of W times
    x (device fp32 [M][K], M > 8), every element written to each pointer of
    ``dst_ptrs`` at [m][col_offset + n] with row stride ``ldy``; dst_ptrs[0]
    is this GPU's own buffer, the rest the other ranks' (pxq_ipc_open)."""
    x = x.contiguous()
    row_count = W.rows - row_first if row_count is None else row_count
    arr = (C.c_void_p * len(dst_ptrs))(*[C.c_void_p(p) for p in dst_ptrs])
    _check(load().pxq_matmul_scatter(W.handle, row_first, row_count, _ptr(x), x.shape[0], C.cast(arr, C.c_void_p), len(dst_ptrs),
                                     ldy, col_offset, _stream_ptr(stream)))


def synchronize(stream=None) -> None:
    _check(load().pxq_synchronize(_stream_ptr(stream)))


# --------------------------------------------------------------- host side ---

def quant_matmul(weights: np.ndarray, wtype: int, x: np.ndarray, rows: int):
    """cpu_quant_matmul with host buffers: returns (handled, Y[columns, rows])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    columns, inner = x.shape
    w = np.ascontiguousarray(weights, dtype=np.uint8)
    y = np.empty((columns, rows), dtype=np.float32)
    rc = load().pxq_quant_matmul(w.ctypes.data_as(C.c_void_p), wtype, x.ctypes.data_as(C.c_void_p),
                                 y.ctypes.data_as(C.c_void_p), rows, columns, inner)
    if rc == ERR_UNSUPPORTED:
        return False, y
    _check(rc)
    return True, y


def quant_matmul_ptr(weights_ptr: int, wtype: int, x_ptr: int, y_ptr: int, rows: int, columns: int, inner: int) -> int:
    """Raw-pointer form of pxq_quant_matmul (host addresses); returns the status."""
    return int(load().pxq_quant_matmul(C.c_void_p(weights_ptr), wtype, C.c_void_p(x_ptr), C.c_void_p(y_ptr), rows, columns,
                                       inner))

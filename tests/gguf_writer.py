"""A GGUF v3 writer for the loader tests (test infrastructure).

Writes the container layout that Pixelina's loader reads
(src/model.cpp:196-232): magic, version, tensor and key counts, typed
metadata pairs, the tensor directory (name, rank, dims, type, offset relative
to the aligned data start), padding to the alignment, tensor data.  Every
field can be overridden to build the malformed files the tests need.
"""
from __future__ import annotations

import struct

# metadata value types (GGUF)
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q", I64: "<q",
           F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        etype, items = v
        out = struct.pack("<IQ", etype, len(items))
        for it in items:
            out += _value(etype, it)
        return out
    if vtype in _SCALAR:
        return struct.pack(_SCALAR[vtype], v)
    return b""  # an invalid type carries no payload


def write_gguf(path: str, tensors: list, metadata: list = (), alignment: int = 32, magic: bytes = b"GGUF", version: int = 3,
               count: int | None = None, offsets: list | None = None, truncate: int = 0) -> None:
    """tensors: [(name, type, shape, data_bytes)], shape in GGML order.
    metadata: [(key, vtype, value)].  offsets: relative data offsets to write
    instead of the packed ones (for misaligned / overlapping files)."""
    head = magic + struct.pack("<I", version)
    head += struct.pack("<QQ", len(tensors) if count is None else count, len(metadata))
    for key, vtype, v in metadata:
        head += _str(key) + struct.pack("<I", vtype) + _value(vtype, v)
    rel, pos = [], 0
    for name, ttype, shape, data in tensors:
        rel.append(pos)
        pos = (pos + len(data) + alignment - 1) // alignment * alignment
    if offsets is not None:
        rel = offsets
    for (name, ttype, shape, data), off in zip(tensors, rel):
        head += _str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in shape)
        head += struct.pack("<IQ", ttype, off)
    base = (len(head) + alignment - 1) // alignment * alignment
    blob = bytearray(head + b"\0" * (base - len(head)))
    end = max([o + len(t[3]) for o, t in zip(rel, tensors)] + [0])
    blob += b"\0" * end
    for (name, ttype, shape, data), off in zip(tensors, rel):
        blob[base + off:base + off + len(data)] = data
    if truncate:
        blob = blob[:len(blob) - truncate]
    with open(path, "wb") as f:
        f.write(bytes(blob))

"""Writes small GGUF files for the tests (test infrastructure).

Layout (little-endian): magic "GGUF", version, tensor count, KV count (64-bit
from version 2 on), the KVs (key string, value type, value), the tensor
directory (name, dimension count, dimensions, ggml type, offset into the data
section), padding to the alignment, then the data section with every tensor's
bytes at its aligned offset.
"""
from __future__ import annotations

import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q", I64: "<q",
        F64: "<d"}


def _len(n: int, version: int) -> bytes:
    return struct.pack("<Q" if version >= 2 else "<I", n)


def _str(s: str, version: int) -> bytes:
    b = s.encode()
    return _len(len(b), version) + b


def _value(ty: int, v, version: int) -> bytes:
    if ty == STRING:
        return _str(v, version)
    if ty == ARRAY:
        ety, items = v
        return struct.pack("<I", ety) + _len(len(items), version) + b"".join(_value(ety, x, version) for x in items)
    return struct.pack(_FMT[ty], v)


def gguf_bytes(kvs, tensors, version: int = 3, alignment: int = 32, offsets=None) -> bytes:
    """kvs: [(key, type, value)]; tensors: [(name, ggml_type, ne tuple, data bytes)].
    offsets (optional) overrides the data offsets (to build malformed files)."""
    head = b"GGUF" + struct.pack("<I", version) + _len(len(tensors), version) + _len(len(kvs), version)
    for key, ty, v in kvs:
        head += _str(key, version) + struct.pack("<I", ty) + _value(ty, v, version)
    offs, at = [], 0
    for _, _, _, data in tensors:
        at = (at + alignment - 1) // alignment * alignment
        offs.append(at)
        at += len(data)
    if offsets is not None:
        offs = list(offsets)
    for (name, ty, ne, _), off in zip(tensors, offs):
        head += _str(name, version) + struct.pack("<I", len(ne))
        head += b"".join(_len(d, version) for d in ne) + struct.pack("<I", ty) + struct.pack("<Q", off)
    head += b"\0" * ((-len(head)) % alignment)
    data = bytearray()
    for (_, _, _, payload), off in zip(tensors, offs):
        if len(data) < off:
            data += b"\0" * (off - len(data))
        data[off:off + len(payload)] = payload
    return head + bytes(data)


def write_gguf(path, kvs, tensors, **kw) -> None:
    with open(path, "wb") as f:
        f.write(gguf_bytes(kvs, tensors, **kw))

"""A GGUF v3 writer for tests: metadata key/value pairs and tensors laid out
as the format specifies (magic, version, counts, typed key/value pairs, the
tensor table, then the data section aligned to ``general.alignment``)."""

from __future__ import annotations

import struct

import numpy as np

U32, I32, F32, BOOL, STR, ARR, U64 = 4, 5, 6, 7, 8, 9, 10


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _val(vt: int, v) -> bytes:
    if vt == U32:
        return struct.pack("<I", v)
    if vt == I32:
        return struct.pack("<i", v)
    if vt == F32:
        return struct.pack("<f", v)
    if vt == BOOL:
        return struct.pack("<?", v)
    if vt == U64:
        return struct.pack("<Q", v)
    if vt == STR:
        return _str(v)
    raise ValueError(vt)


def write_gguf(path: str, metadata: dict, tensors: list, alignment: int = 32, version: int = 3) -> None:
    """metadata: key -> (type, value) or (ARR, element type, values);
    tensors: (gguf name, ggml type id, shape in NumPy order, bytes)."""
    kv = b""
    for key, spec in metadata.items():
        kv += _str(key)
        if spec[0] == ARR:
            _, et, values = spec
            kv += struct.pack("<IIQ", ARR, et, len(values)) + b"".join(_val(et, v) for v in values)
        else:
            kv += struct.pack("<I", spec[0]) + _val(spec[0], spec[1])
    table = b""
    data = b""
    for name, gtype, shape, raw in tensors:
        raw = bytes(np.ascontiguousarray(raw).view(np.uint8).reshape(-1))
        data += b"\0" * ((-len(data)) % alignment)
        dims = list(reversed(shape))  # GGUF lists the fastest axis first
        table += _str(name) + struct.pack(f"<I{len(dims)}Q", len(dims), *dims) + struct.pack("<IQ", gtype, len(data))
        data += raw
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(metadata)) + kv + table
    head += b"\0" * ((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head + data)

"""A minimal GGUF writer for the tests (the GPU box has no gguf-py): metadata values of the GGUF
value types, tensor records and an aligned data section, laid out as the format describes
(version 1 with 32-bit counts, versions 2/3 with 64-bit counts)."""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}


def _count(v: int, version: int) -> bytes:
    return struct.pack("<I" if version == 1 else "<Q", v)


def _string(s, version: int) -> bytes:
    b = s if isinstance(s, bytes) else s.encode()
    return _count(len(b), version) + b


def _value(vtype: int, v, version: int) -> bytes:
    if vtype == STR:
        return _string(v, version)
    if vtype == ARR:
        sub, items = v
        return struct.pack("<I", sub) + _count(len(items), version) + b"".join(_value(sub, x, version) for x in items)
    return struct.pack(_SCALAR[vtype], v)


def gguf_bytes(metadata, tensors, version: int = 3, alignment: int = 32, data: bytes | None = None,
               tail: bytes = b"") -> bytes:
    """metadata: [(key, vtype, value)] (arrays: value = (sub_type, items)).  tensors: [(name, dims,
    ggml_type, payload bytes)] laid out in order, each at an `alignment` boundary; or, with `data`
    given, [(name, dims, ggml_type, offset)] over that raw data section."""
    out = b"GGUF" + struct.pack("<I", version) + _count(len(tensors), version) + _count(len(metadata), version)
    for key, vt, v in metadata:
        out += _string(key, version) + struct.pack("<I", vt) + _value(vt, v, version)
    if data is None:
        section, offs = b"", []
        for _, _, _, payload in tensors:
            pad = (-len(section)) % alignment
            section += b"\0" * pad
            offs.append(len(section))
            section += bytes(payload)
        records = [(n, d, t, o) for (n, d, t, _), o in zip(tensors, offs)]
    else:
        section, records = data, tensors
    for name, dims, gtype, off in records:
        out += _string(name, version) + struct.pack("<I", len(dims))
        out += b"".join(_count(int(d), version) for d in dims)
        out += struct.pack("<I", gtype) + struct.pack("<Q", off)
    out += b"\0" * ((-len(out)) % alignment)
    return out + section + tail


def write_stage_gguf(path, tensors: dict, metadata=(), alignment: int = 32):
    """A GGUF of oracle tensors {name: (ggml_type, dims, array)}."""
    tl = [(n, d, t, np.ascontiguousarray(a).view(np.uint8).tobytes()) for n, (t, d, a) in tensors.items()]
    with open(path, "wb") as f:
        f.write(gguf_bytes(list(metadata), tl, alignment=alignment))
    return path

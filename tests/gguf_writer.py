"""A minimal GGUF (v3) writer for the loader tests — test infrastructure.

It lays files out the way the reference's own test fixtures write them
(har/crates/har-serve/src/gguf.rs:175-205, har/crates/har-package-slice/src/tests.rs:21-50):
magic, version, u64 tensor and metadata counts, metadata key/type/value
records, tensor infos (name, rank, u64 dims in GGML order, u32 type, u64
offset relative to the data section), zero padding to the alignment, then
the tensor payloads at their offsets."""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
        BOOL: "<?", U64: "<Q", I64: "<q", F64: "<d"}


def _str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def _value(vtype, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[vtype], v)


def write_gguf(path, metadata, tensors, alignment=32, version=3):
    """metadata: [(key, vtype, value)]; tensors: [(name, dims, ggml_type,
    payload bytes)].  Payloads are placed in order, each at an aligned offset.
    Returns {name: absolute file offset of the payload}."""
    out = bytearray(b"GGUF")
    out += struct.pack("<IQQ", version, len(tensors), len(metadata))
    for key, vt, val in metadata:
        out += _str(key) + struct.pack("<I", vt) + _value(vt, val)
    tensors = [(n, d, t, np.ascontiguousarray(p).view(np.uint8).tobytes()) for n, d, t, p in tensors]
    rel, off = [], 0
    for name, dims, gtype, payload in tensors:
        rel.append(off)
        out += _str(name) + struct.pack("<I", len(dims))
        out += b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gtype, off)
        off += len(payload)
        off = (off + alignment - 1) // alignment * alignment
    while len(out) % alignment:
        out.append(0)
    data = len(out)
    where = {}
    for (name, _, _, payload), r in zip(tensors, rel):
        while len(out) < data + r:
            out.append(0)
        where[name] = len(out)
        out += payload
    with open(path, "wb") as f:
        f.write(out)
    return where

"""In-memory GGUF builder for tests, following the byte layout of woolly's
MockGGUFBuilder (crates/woolly-gguf/tests/load_model.rs:51-144): header,
metadata, tensor table with running (unaligned) offsets, 32-byte pad, data."""
import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)


def _val(t, v):
    fmt = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f",
           U64: "<Q", I64: "<q", F64: "<d"}
    if t in fmt:
        return struct.pack(fmt[t], v)
    if t == BOOL:
        return struct.pack("<B", 1 if v else 0)
    if t == STR:
        b = v.encode()
        return struct.pack("<Q", len(b)) + b
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_val(et, x) for x in items)
    raise ValueError(t)


def build(metadata=(), tensors=(), version=3):
    """metadata: [(key, type, value)]; tensors: [(name, shape, ggml_type, nbytes, data)]."""
    out = bytearray(b"GGUF")
    out += struct.pack("<IQQ", version, len(tensors), len(metadata))
    for k, t, v in metadata:
        kb = k.encode()
        out += struct.pack("<Q", len(kb)) + kb + struct.pack("<I", t) + _val(t, v)
    off = 0
    for name, shape, gt, nbytes, _ in tensors:
        nb = name.encode()
        out += struct.pack("<Q", len(nb)) + nb + struct.pack("<I", len(shape))
        out += b"".join(struct.pack("<Q", d) for d in shape)
        out += struct.pack("<IQ", gt, off)
        off += nbytes
    pad = (len(out) + 31) // 32 * 32 - len(out)
    out += bytes(pad)
    for *_, data in tensors:
        out += data
    return bytes(out)

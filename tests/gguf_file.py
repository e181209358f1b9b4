"""Test helper: a GGUF v2/v3 file writer in plain Python (the container format as the reference's src/gguf.c reads and
writes it), able to produce layouts the reference's writer never does -- tensor infos out of data order, explicit
offsets, any key/value type, nested arrays -- for the reader's tests."""
import struct

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q", I64: "<q",
        F64: "<d"}
T_EXPERTS = 120  # INZ_T_EXPERTS (src/quant.h:36)


def _str(s):
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[t], v)


def _header(kvs, tensors, alignment, version, order):
    offs, pos = [], 0
    for _, data in tensors:
        offs.append(pos)
        pos += (len(data) + alignment - 1) // alignment * alignment
    kvs = [("general.alignment", U32, alignment)] + list(kvs)  # as the reference's writer does
    head = struct.pack("<IIQQ", 0x46554747, version, len(tensors), len(kvs))
    head += b"".join(_str(k) + struct.pack("<I", t) + _value(t, v) for k, t, v in kvs)
    for i in (order if order is not None else range(len(tensors))):
        name, data = tensors[i]
        head += _str(name) + struct.pack("<I", 1) + struct.pack("<Q", len(data)) + struct.pack("<IQ", T_EXPERTS, offs[i])
    start = (len(head) + alignment - 1) // alignment * alignment
    return head, start, offs, pos


def gguf_bytes(kvs, tensors, alignment=32, version=3, order=None):
    """kvs: [(key, type, value)]; arrays are (elem_type, [items]). tensors: [(name, data)] in data order, data any
    bytes-like object; order: the order of their infos in the header (default: data order). Offsets are packed at
    `alignment`, which the file records as "general.alignment". Returns (file bytes, data start, offsets)."""
    head, start, offs, pos = _header(kvs, tensors, alignment, version, order)
    body = bytearray(start + pos)
    body[:len(head)] = head
    for (_, data), o in zip(tensors, offs):
        body[start + o:start + o + len(data)] = bytes(data)
    return bytes(body), start, offs


def write(path, kvs, tensors, alignment=32, version=3, order=None):
    """gguf_bytes streamed to `path` (tensor data written in place, no whole-file copy in memory)."""
    tensors = [(n, memoryview(d).cast("B")) for n, d in tensors]
    head, start, offs, pos = _header(kvs, tensors, alignment, version, order)
    with open(path, "wb") as f:
        f.write(head)
        f.write(b"\0" * (start - len(head)))
        for (_, data), o in zip(tensors, offs):
            assert f.tell() == start + o
            f.write(data)
            f.write(b"\0" * ((len(data) + alignment - 1) // alignment * alignment - len(data)))
    return start, offs

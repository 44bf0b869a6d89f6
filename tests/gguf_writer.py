"""Minimal GGUF v3 writer for hand-built test models (F32/F16/quantized
payloads given as bytes), in the layout of tools/nexus-convert/main.rs:345-383."""
import struct

import numpy as np

VT_U32, VT_F32, VT_STR = 4, 6, 8


def write_gguf(path, metadata: dict, tensors: list, alignment: int = 32):
    """metadata: key -> int (U32) | float (F32) | str; tensors: (name, shape, type_id, bytes)."""
    out = bytearray(b"GGUF")
    out += struct.pack("<IQQ", 3, len(tensors), len(metadata) + 1)
    items = dict(metadata)
    items["general.alignment"] = alignment
    for key in sorted(items):
        v = items[key]
        out += struct.pack("<Q", len(key)) + key.encode()
        if isinstance(v, str):
            out += struct.pack("<IQ", VT_STR, len(v)) + v.encode()
        elif isinstance(v, float):
            out += struct.pack("<If", VT_F32, v)
        else:
            out += struct.pack("<II", VT_U32, v)
    off = 0
    offsets = []
    for name, shape, ty, data in tensors:
        out += struct.pack("<Q", len(name)) + name.encode() + struct.pack("<I", len(shape))
        for d in shape:
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", ty, off)
        offsets.append(off)
        off += (len(data) + alignment - 1) // alignment * alignment
    while len(out) % alignment:
        out.append(0)
    for (_, _, _, data) in tensors:
        out += bytes(data)
        while len(out) % alignment:
            out.append(0)
    with open(path, "wb") as f:
        f.write(out)


def f32_bytes(values) -> bytes:
    return np.asarray(values, np.float32).tobytes()

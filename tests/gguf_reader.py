"""Tiny GGUF v3 reader for tests (F32 tensors only)."""
import struct

import numpy as np


def _str(b, p):
    n = struct.unpack_from("<Q", b, p)[0]
    return b[p + 8:p + 8 + n].decode(), p + 8 + n


def read_tensor(path, name):
    b = open(path, "rb").read()
    assert b[:4] == b"GGUF"
    _, tc, kc = struct.unpack_from("<IQQ", b, 4)
    p = 24
    align = 32
    for _ in range(kc):
        key, p = _str(b, p)
        vt = struct.unpack_from("<I", b, p)[0]
        p += 4
        if vt in (4, 5, 6):
            val = struct.unpack_from("<I", b, p)[0]
            p += 4
        elif vt == 8:
            val, p = _str(b, p)
        else:
            raise ValueError(vt)
        if key == "general.alignment":
            align = val
    infos = {}
    for _ in range(tc):
        tname, p = _str(b, p)
        nd = struct.unpack_from("<I", b, p)[0]
        p += 4
        shape = struct.unpack_from("<" + "Q" * nd, b, p)
        p += 8 * nd
        ty, off = struct.unpack_from("<IQ", b, p)
        p += 12
        infos[tname] = (shape, ty, off)
    base = (p + align - 1) // align * align
    shape, ty, off = infos[name]
    assert ty == 0
    n = int(np.prod(shape))
    return np.frombuffer(b, np.float32, n, base + off)

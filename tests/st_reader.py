"""Minimal safetensors reader (numpy) for tests: returns raw arrays by name."""
import json
import struct

import numpy as np

_DT = {"U32": np.uint32, "F32": np.float32, "BF16": np.uint16}


def read_tensors(path: str, names):
    out = {}
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
        base = 8 + n
        for name in names:
            t = hdr["language_model.model." + name]
            a, b = t["data_offsets"]
            f.seek(base + a)
            out[name] = np.frombuffer(f.read(b - a), _DT[t["dtype"]]).reshape(t["shape"]).copy()
    return out

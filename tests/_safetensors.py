"""Minimal safetensors reader/writer for the tests (the format the prefix
cache's disk tier shares with the reference: an 8-byte little-endian header
length, a JSON header of {name: {dtype, shape, data_offsets}} and an optional
"__metadata__", then the raw tensor bytes)."""
import json
import struct

import numpy as np

_NP = {"U8": np.uint8, "F16": np.uint16, "BF16": np.uint16, "F32": np.float32}


def read(path):
    with open(path, "rb") as f:
        (n,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, t in header.items():
        if name == "__metadata__":
            continue
        a, b = t["data_offsets"]
        arr = np.frombuffer(data[a:b], dtype=_NP[t["dtype"]]).reshape(t["shape"])
        out[name] = (t["dtype"], arr)
    return out, header


def write(path, tensors, metadata=None):
    """tensors: name -> (dtype string, numpy array)."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, (dt, arr) in tensors.items():
        raw = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    js = json.dumps(header).encode()
    js += b" " * ((8 - len(js) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(js)))
        f.write(js)
        for b in blobs:
            f.write(b)

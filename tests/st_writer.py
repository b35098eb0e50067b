"""Writes safetensors files for the tests (format: u64 header length, JSON header with
dtype / shape / data_offsets per tensor, then the data block)."""
import json
import struct

import numpy as np

_DT = {np.dtype(np.uint16): "BF16", np.dtype(np.float32): "F32", np.dtype(np.uint32): "U32",
       np.dtype(np.int32): "I32", np.dtype(np.float16): "F16", np.dtype(np.uint8): "U8"}


def write_safetensors(path, tensors: dict, metadata: dict | None = None, bf16_keys=()):
    """tensors: name -> numpy array (uint16 arrays are written as BF16)."""
    header, blobs, off = {}, [], 0
    if metadata:
        header["__metadata__"] = metadata
    for name, a in tensors.items():
        a = np.asarray(a)  # (np.ascontiguousarray would turn a 0-d array into shape [1])
        a = a if a.flags.c_contiguous else a.copy()
        b = a.tobytes()
        header[name] = {"dtype": _DT[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)

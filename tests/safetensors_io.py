"""A small safetensors writer and reader for the checkpoint tests: an 8-byte little-endian
header length, a JSON header {name: {"dtype", "shape", "data_offsets": [start, end]}}
(offsets from the end of the header; optional "__metadata__"), then the tensor bytes in
header order with no gaps. The header is padded with spaces to a multiple of 8 bytes."""
import json
import struct

import numpy as np

DTYPES = {"U8": np.uint8, "BF16": np.uint16, "F16": np.float16, "F32": np.float32}


def write_shard(path, tensors, metadata=None, order=None):
    """tensors: name -> (dtype name, shape, numpy array of that many elements)."""
    names = order or list(tensors)
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name in names:
        dt, shape, arr = tensors[name]
        b = np.ascontiguousarray(arr, DTYPES[dt]).tobytes()
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read_header(path):
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        return json.loads(f.read(n)), 8 + n

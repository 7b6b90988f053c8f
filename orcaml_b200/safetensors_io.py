"""The safetensors container, read and written without dependencies.

Layout (the format orca-serialize reads and writes through the `safetensors`
crate, orca-serialize/src/lib.rs:6-79): an 8-byte little-endian header size
N, N bytes of JSON -- {name: {"dtype", "shape", "data_offsets": [begin, end]},
optional "__metadata__": {str: str}} padded with spaces to a multiple of 8 --
then the tensors' raw little-endian bytes, offsets relative to the end of the
header.
"""
from __future__ import annotations

import json
import struct
from typing import Dict, Optional, Tuple

ITEM_BYTES = {"F32": 4, "F64": 8, "F16": 2, "BF16": 2, "I32": 4, "I64": 8, "U8": 1, "BOOL": 1}

Entry = Tuple[str, list, bytes]   # (dtype, shape, raw bytes)


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= int(d)
    return n


def write(path: str, entries: Dict[str, Entry], metadata: Optional[Dict[str, str]] = None):
    header, blobs, offset = {}, [], 0
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    for name in sorted(entries):
        dtype, shape, data = entries[name]
        if dtype not in ITEM_BYTES:
            raise ValueError(f"unsupported dtype {dtype!r} for {name!r}")
        if len(data) != _numel(shape) * ITEM_BYTES[dtype]:
            raise ValueError(f"{name!r}: {len(data)} bytes for shape {list(shape)}")
        header[str(name)] = {"dtype": dtype, "shape": [int(d) for d in shape],
                             "data_offsets": [offset, offset + len(data)]}
        blobs.append(data)
        offset += len(data)
    raw = json.dumps(header, separators=(",", ":")).encode()
    raw += b" " * ((8 - len(raw) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(raw)))
        f.write(raw)
        for b in blobs:
            f.write(b)


def read(path: str) -> Tuple[Dict[str, Entry], Dict[str, str]]:
    with open(path, "rb") as f:
        buf = f.read()
    if len(buf) < 8:
        raise ValueError("not a safetensors file")
    (n,) = struct.unpack("<Q", buf[:8])
    if 8 + n > len(buf):
        raise ValueError("truncated safetensors header")
    header = json.loads(buf[8:8 + n].decode())
    data = memoryview(buf)[8 + n:]
    metadata = header.pop("__metadata__", {}) or {}
    out = {}
    for name, meta in header.items():
        dtype = meta.get("dtype")
        if dtype not in ITEM_BYTES:
            raise ValueError(f"Unsupported safetensor dtype {dtype!r}")
        shape = [int(d) for d in meta["shape"]]
        b0, b1 = meta["data_offsets"]
        if not (0 <= b0 <= b1 <= len(data)) or b1 - b0 != _numel(shape) * ITEM_BYTES[dtype]:
            raise ValueError(f"bad data offsets for {name!r}")
        out[name] = (dtype, shape, bytes(data[b0:b1]))
    return out, metadata

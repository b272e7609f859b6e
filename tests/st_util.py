"""A minimal safetensors writer and reader in plain Python (test helpers, independent of the
library's C++ reader): 8-byte little-endian header length, JSON header {name: {dtype, shape,
data_offsets}}, then the tensor bytes (the layout src/safetensors/safetensors.cc:43-83 reads)."""
from __future__ import annotations

import json
import struct

import numpy as np

NP_DTYPE = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I8": np.int8, "I32": np.int32, "U8": np.uint8}


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bfloat16 bits by round-to-nearest-even (how checkpoints are usually made)."""
    u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(a, np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def bf16_widen(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bits -> fp32, exactly (SafeTensorsLoader::bf16_to_f32)."""
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def write(path: str, tensors: dict, metadata: dict | None = None, pad: bool = True) -> None:
    """tensors: name -> (dtype string, numpy array).  Data in insertion order, no gaps."""
    hdr, blobs, off = {}, [], 0
    if metadata is not None:
        hdr["__metadata__"] = metadata
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        hdr[name] = {"dtype": dt, "shape": list(np.shape(arr)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(hdr).encode()
    if pad:
        h += b" " * ((8 - (8 + len(h)) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def read(path: str):
    """(metadata dict, {name: (dtype, shape, bytes)}) of a safetensors file."""
    with open(path, "rb") as f:
        raw = f.read()
    (n,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    meta = hdr.pop("__metadata__", {})
    out = {}
    for name, t in hdr.items():
        b, e = t["data_offsets"]
        out[name] = (t["dtype"], tuple(t["shape"]), data[b:e])
    return meta, out


def array(entry) -> np.ndarray:
    dt, shape, b = entry
    return np.frombuffer(b, dtype=NP_DTYPE[dt]).reshape(shape)

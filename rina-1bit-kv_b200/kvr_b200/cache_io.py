"""Packed-cache container: save / load the compressed KV state.

The reference keeps its index in memory only (no checkpoint / resume).  This
module stores the packed state in a self-describing file that any language can
read without Python pickling:

    bytes 0..7    magic  b"KVRCACHE"
    bytes 8..11   uint32 format version (1), little-endian
    bytes 12..15  uint32 length H of the header
    bytes 16..    H bytes of UTF-8 JSON:
                  {"meta": {...}, "tensors": [{"name", "dtype", "shape",
                   "offset", "nbytes"}, ...]}
    then the raw little-endian tensor bytes, each starting at its `offset`
    (from the start of the file, 64-byte aligned).

dtype names: uint8, int32, int64, float16, float32.  Tensors are written in
C order.  `meta` holds plain JSON values (counters, codec, shapes).
"""
from __future__ import annotations

import json
import struct

import numpy as np
import torch

MAGIC = b"KVRCACHE"
VERSION = 1
_ALIGN = 64
_DTYPES = {torch.uint8: "uint8", torch.int32: "int32", torch.int64: "int64", torch.float16: "float16",
           torch.float32: "float32"}
_NP = {"uint8": np.uint8, "int32": np.int32, "int64": np.int64, "float16": np.float16, "float32": np.float32}


def _align(n):
    return (n + _ALIGN - 1) // _ALIGN * _ALIGN


def write_cache(path, meta: dict, tensors: dict):
    """meta: JSON-serialisable dict; tensors: name -> torch.Tensor (any device)."""
    host = {}
    for name, t in tensors.items():
        if t.dtype not in _DTYPES:
            raise TypeError(f"{name}: unsupported dtype {t.dtype}")
        host[name] = t.detach().contiguous().cpu()
    entries, offset = [], 0
    for name, t in host.items():
        nb = t.numel() * t.element_size()
        entries.append({"name": name, "dtype": _DTYPES[t.dtype], "shape": list(t.shape), "offset": offset,
                        "nbytes": nb})
        offset = _align(offset + nb)
    # the header's length depends on the offsets it records: fix the data base first
    probe = json.dumps({"meta": meta, "tensors": entries}).encode()
    base = _align(16 + len(probe) + 16 * len(entries) + 64)
    for e in entries:
        e["offset"] += base
    header = json.dumps({"meta": meta, "tensors": entries}).encode()
    if 16 + len(header) > base:
        raise RuntimeError("cache header overflow")
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<II", VERSION, len(header)) + header)
        f.write(b"\0" * (base - 16 - len(header)))
        pos = base
        for e in entries:
            f.write(b"\0" * (e["offset"] - pos))
            f.write(host[e["name"]].numpy().tobytes())
            pos = e["offset"] + e["nbytes"]


def read_cache(path, device="cpu"):
    """-> (meta, {name: tensor on `device`})."""
    with open(path, "rb") as f:
        raw = f.read()
    if raw[:8] != MAGIC:
        raise ValueError(f"{path}: not a KVR cache file")
    version, hlen = struct.unpack("<II", raw[8:16])
    if version != VERSION:
        raise ValueError(f"{path}: cache format version {version}, expected {VERSION}")
    head = json.loads(raw[16:16 + hlen].decode())
    out = {}
    for e in head["tensors"]:
        a = np.frombuffer(raw, dtype=_NP[e["dtype"]], count=int(np.prod(e["shape"], dtype=np.int64)),
                          offset=e["offset"]).reshape(e["shape"])
        out[e["name"]] = torch.from_numpy(a.copy()).to(device)
    return head["meta"], out

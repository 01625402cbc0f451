"""Packed-cache container (kvr_b200.cache_io): byte-exact round trip on the
host, header layout, error on foreign files."""
import json
import struct

import pytest
import torch


def test_round_trip_all_dtypes(tmp_path):
    from kvr_b200.cache_io import MAGIC, read_cache, write_cache
    g = torch.Generator().manual_seed(0)
    tensors = {
        "u8": torch.randint(0, 256, (7, 3), generator=g, dtype=torch.int64).to(torch.uint8),
        "i32": torch.randint(-2**31, 2**31 - 1, (2, 5, 4), generator=g, dtype=torch.int64).to(torch.int32),
        "i64": torch.arange(11, dtype=torch.int64) * -3,
        "f16": torch.randn(3, 128, generator=g).half(),
        "f32": torch.randn(9, generator=g),
        "empty": torch.zeros(0, 8, dtype=torch.float16),
    }
    meta = {"codec": "sd1", "n": 3, "nested": {"a": [1, 2]}}
    p = tmp_path / "c.kvrc"
    write_cache(p, meta, tensors)
    raw = p.read_bytes()
    assert raw[:8] == MAGIC
    version, hlen = struct.unpack("<II", raw[8:16])
    head = json.loads(raw[16:16 + hlen])
    assert version == 1 and head["meta"] == meta
    for e in head["tensors"]:
        assert e["offset"] % 64 == 0 and e["offset"] >= 16 + hlen
    m2, t2 = read_cache(p)
    assert m2 == meta and set(t2) == set(tensors)
    for k, v in tensors.items():
        assert t2[k].dtype == v.dtype and t2[k].shape == v.shape
        assert torch.equal(t2[k].view(torch.uint8) if v.numel() else t2[k], v.view(torch.uint8) if v.numel() else v)


def test_foreign_file_is_rejected(tmp_path):
    from kvr_b200.cache_io import read_cache
    p = tmp_path / "x.bin"
    p.write_bytes(b"not a cache file at all")
    with pytest.raises(ValueError):
        read_cache(p)

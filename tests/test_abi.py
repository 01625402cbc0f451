"""CPU checks of the C ABI boundary: the in-tree library loads without a GPU
and exports every entry point include/kvr_b200.h declares; the Python binding
knows each one.  No compute calls here."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HDR = os.path.join(ROOT, "include", "kvr_b200.h")


def declared():
    src = open(HDR).read()
    return sorted(set(re.findall(r"^KVR_API\s+(?:int|size_t|const char \*)\s*(kvr_\w+)\(", src, re.M)))


def test_header_declares_entry_points():
    names = declared()
    assert len(names) >= 25
    assert "kvr_sd1_decode_step" in names and "kvr_compute_scores" in names


def test_library_exports_every_declared_symbol():
    from kvr_b200 import _native
    if not os.path.exists(_native.LIB_PATH):
        pytest.fail("native library not built: run __graft_entry__.build()")
    lib = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(declared()) == set(_native.SIGNATURES), set(declared()) ^ set(_native.SIGNATURES)
    assert _native.lib().kvr_abi_version() >> 16 == 1


def test_workspace_size_helpers_need_no_gpu():
    from kvr_b200 import _native as N
    assert N.call("kvr_sd1_workspace_bytes", 1, 32, 8, 504, 64, 16, 512, 0) > 0
    assert N.call("kvr_decode_attn_workspace_bytes", 32, 8, 128, 1536) > 0
    assert N.call("kvr_sd1_select_workspace_bytes", 32, 8, 252) % 256 == 0


def test_operators_refuse_cpu_tensors():
    import torch
    from kvr_b200 import kernels
    with pytest.raises(ValueError, match="CUDA"):
        kernels.transform(torch.zeros(2, 128))

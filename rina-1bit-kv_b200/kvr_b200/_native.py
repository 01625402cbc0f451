"""ctypes binding of the C ABI in include/kvr_b200.h (libkvr_b200.so, in-tree).

There is no fallback: if the library is missing, importing an operator raises.
Tensors are passed as raw device pointers; every call runs on the current
torch CUDA stream and raises ``KvrError`` on a non-zero status.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

# KVR_B200_LIB: load another build of the same library (A/B measurements of
# kernel variants); default: the in-tree build.
LIB_PATH = os.environ.get("KVR_B200_LIB") or os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib",
                                                           "libkvr_b200.so")

KVR_F32, KVR_F16, KVR_BF16 = 0, 1, 2
KVR_HADAMARD, KVR_DCT = 0, 1
STATUS = {0: "KVR_OK", 1: "KVR_EINVAL", 2: "KVR_ECUDA", 3: "KVR_ENOTSUP", 4: "KVR_ETIMEOUT"}

_DT = {torch.float32: KVR_F32, torch.float16: KVR_F16, torch.bfloat16: KVR_BF16}
TRANSFORMS = {"hadamard": KVR_HADAMARD, "dct": KVR_DCT}


class KvrError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS.get(code, code)}: {msg}")
        self.code = code


P, I, I64, F, SZ = C.c_void_p, C.c_int, C.c_int64, C.c_float, C.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "kvr_last_error": (C.c_char_p, []),
    "kvr_abi_version": (I, []),
    "kvr_absmax_scales": (I, [P, I, I64, I64, F, P, P]),
    "kvr_int4w_encode_k": (I, [P, I, I64, I, I, I64, P, P, P]),
    "kvr_int4w_encode_vres": (I, [P, I, P, I64, I, I, P, P, P]),
    "kvr_compute_scores": (I, [P, P, P, P, P, I, I, I64, P, P]),
    "kvr_int4w_token_scores": (I, [P, I, P, P, P, P, I64, I, I, I, I64, P, I64, P]),
    "kvr_int4w_chunk_scores": (I, [P, I, P, P, P, P, I64, I, I, I, I64, I, P, I64, P]),
    "kvr_topk_rows": (I, [P, I, I64, I64, I, I64, I64, P, P, I64, I64, P]),
    "kvr_int4w_token_topk_workspace_bytes": (SZ, [I, I64, I]),
    "kvr_int4w_token_topk": (I, [P, I, P, P, P, P, I64, I, I, I, I64, I, I64, I64, P, P, SZ, P]),
    "kvr_int4w_gather": (I, [P, P, P, I, I, I, P, P, I64, P, P, P, P, P]),
    "kvr_int4w_vpredict_weights_bytes": (SZ, [I, I]),
    "kvr_int4w_vpredict_prepare": (I, [P, P, P, P, I, I, P, P, P, P]),
    "kvr_int4w_vpredict": (I, [P, P, P, I, I, I, P, P, P, P, P, P, P]),
    "kvr_int4w_attractor_workspace_bytes": (SZ, [I64, I]),
    "kvr_int4w_attractor_select": (I, [P, I, I, P, P, P, P, I64, P, I, P, I64, I, I64, I64, P, P, P, SZ, P]),
    "kvr_int4w_assign_basins": (I, [P, P, I, I64, I64, P, I, P, P]),
    "kvr_decode_attn_counted": (I, [P, I, I, I, I, P, P, I, I, I64, I64, P, P, I, I, I64, I64, P, F, P, I, P, SZ,
                                    P]),
    "kvr_int4w_vres_add": (I, [P, P, P, P, I, I, I, P, P]),
    "kvr_window_write": (I, [P, P, I, I64, I, I, P, P, I64, I64, P]),
    "kvr_decode_store_update": (I, [P, P, P, I, I, I, I, P, P, I64, I64, P, P, P, I64, I64, P, P, I64, I, P]),
    "kvr_decode_attn_workspace_bytes": (SZ, [I, I, I, I64]),
    "kvr_decode_attn": (I, [P, I, I, I, I, P, P, I, I, I64, I64, P, P, I, I, I64, I64, F, P, I, P, SZ, P]),
    "kvr_transform": (I, [P, P, I64, I, I, P]),
    "kvr_sd1_encode": (I, [P, P, I, I, I, I64, I, I64, I64, P, P, I64, I64, I, P, P, P, P, I64, I64, P]),
    "kvr_sd1_tile_scores": (I, [P, I, I, I, I, P, P, I64, I64, I, I, P, P]),
    "kvr_sd1_decode_tiles": (I, [P, P, P, P, I64, I, I, I, I, P, I, P, P, P]),
    "kvr_sd1_select_workspace_bytes": (SZ, [I, I, I64]),
    "kvr_sd1_select": (I, [P, I, I, I, I, P, P, I64, I64, I, I, I, I64, I64, I64, P, P, P, P, SZ, P]),
    "kvr_sd1_attend_workspace_bytes": (SZ, [I, I, I, I, I, I64, I64]),
    "kvr_sd1_attend": (I, [P, I, P, I, I, I, P, P, I64, I64, P, P, I64, P, P, P, P, I64, I, I, P, I, F, P, I, P,
                           P, SZ, P]),
    "kvr_sd1_workspace_bytes": (SZ, [I, I, I, I64, I, I, I64, I64]),
    "kvr_set_sd1_step_path": (I, [I]),
    "kvr_sd1_decode_step_update": (I, [P, P, P, I, I, I, P, P, I64, I64, P, P, P, I64, I64, I64, P, P, I64, I,
                                       P, P, P, P, I64, I64, I, I, I, I64, I64, F, P, I, P, P, SZ, P]),
    "kvr_sd1_decode_step": (I, [P, I, I, I, I, P, P, I64, I64, P, P, I64, P, P, P, P, I64, I64, I, I, I, I64, I64,
                                F, P, I, P, P, SZ, P]),
    "kvr_lse_merge": (I, [P, I, I, I, P, I, P]),
    "kvr_merge_candidates": (I, [P, P, I, I, I, I, I64, I64, P, P, P]),
    "kvr_peer_buffer_bytes": (SZ, []),
    "kvr_peer_handle_bytes": (SZ, []),
    "kvr_peer_alloc": (I, [P]),
    "kvr_peer_free": (I, [P]),
    "kvr_peer_handle": (I, [P, P]),
    "kvr_peer_open": (I, [P, P]),
    "kvr_peer_close": (I, [P]),
    "kvr_peer_merge_candidates": (I, [P, I, I, P, P, I, I, I, I64, I64, P, P, P]),
    "kvr_peer_lse_merge": (I, [P, I, I, P, I, I, P, I, P]),
    "kvr_sd1_prefill_workspace_bytes": (SZ, [I64, I]),
    "kvr_sd1_prefill_scores": (I, [P, I, I64, I, I, P, P, I64, I64, I, I, P, P, SZ, P]),
    "kvr_kmeans_workspace_bytes": (SZ, [I64, I]),
    "kvr_kmeans": (I, [P, I64, I, I, I, P, P, P, SZ, P]),
    "kvr_int4w_vpredict_status": (I, [P]),
    "kvr_workspace_status": (I, [P, P]),
    "kvr_selftest_bounded_wait": (I, [P, C.c_uint32, P]),
    "kvr_decode_attn_noalloc_max_scratch_bytes": (SZ, []),
    "kvr_decode_attn_noalloc": (I, [P, I, I, I, I, P, P, I, I, I64, I64, P, P, I, I, I64, I64, F, P, I, P]),
}

_lib = None


def lib():
    """Load libkvr_b200.so once; raise if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"kvr_b200 native library not built: {LIB_PATH} is missing "
                               "(run __graft_entry__.build() or python -m kvr_b200._build)")
        h = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(h, name)
            fn.restype = res
            fn.argtypes = args
        _lib = h
    return _lib


_FN: dict = {}


def call(name: str, *args) -> int:
    """Call an entry point; a non-zero status raises KvrError (functions that
    return sizes or strings are returned as they are)."""
    ent = _FN.get(name)
    if ent is None:
        ent = _FN[name] = (getattr(lib(), name), name.endswith("_bytes") or name in ("kvr_last_error",
                                                                                    "kvr_abi_version"))
    rc = ent[0](*args)
    if ent[1]:
        return rc
    if rc != 0:
        raise KvrError(rc, lib().kvr_last_error().decode())
    return rc


def ptr(t) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("kvr_b200 operators need CUDA tensors (this build has no CPU path)")
    return t.data_ptr()


def dtype_code(t) -> int:
    try:
        return _DT[t.dtype]
    except KeyError as e:
        raise TypeError(f"unsupported dtype {t.dtype}") from e


def stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class Workspace:
    """A zero-initialised device scratch buffer that grows on demand.  The
    kernels leave it zeroed after every successful call, so it is reused
    across calls without clearing."""

    def __init__(self, device=None):
        self.buf = None
        self.device = device

    def get(self, nbytes: int, device) -> torch.Tensor:
        nbytes = max(int(nbytes), 256)
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        return self.buf


_WS: dict = {}


def workspace(tag: str, nbytes: int, device) -> torch.Tensor:
    device = device if isinstance(device, torch.device) else torch.device(device)
    ws = _WS.get((tag, device))
    if ws is None:
        ws = _WS[(tag, device)] = Workspace()
    return ws.get(nbytes, device)

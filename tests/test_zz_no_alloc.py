"""The allocation-free attention entry point, for callers that cannot call
cudaMalloc (a plugin inside a host that owns the GPU heap, or a path where an
allocation would stall the device).  Called through the C ABI, it must give the
same result as kvr_decode_attn with a caller workspace, on two calls in a row
(the shared scratch array keeps the previous call's contents), and must refuse
a call whose scratch need exceeds its fixed maximum.  Collected last on purpose."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _args(q, k0, v0, k1, v1):
    from kvr_b200 import _native as N
    P = N.ptr
    return [P(q), N.dtype_code(q), q.shape[0], k0.shape[1], 128,
            P(k0), P(v0), N.dtype_code(k0), N.dtype_code(v0), k0.shape[0], k0.stride(0),
            P(k1), P(v1), N.dtype_code(k1), N.dtype_code(v1), k1.shape[0], k1.stride(0), 0.0]


def test_noalloc_matches_workspace_entry_point_twice():
    from kvr_b200 import _native as N
    dev = "cuda"
    for seed, (n0, n1) in enumerate([(512, 1024), (300, 77)]):
        g = torch.Generator(device=dev).manual_seed(seed)
        q = torch.randn(32, 128, device=dev, generator=g)
        k0 = torch.randn(n0, 8, 128, device=dev, generator=g).half()
        v0 = torch.randn(n0, 8, 128, device=dev, generator=g).half()
        k1 = torch.randn(n1, 8, 128, device=dev, generator=g)
        v1 = torch.randn(n1, 8, 128, device=dev, generator=g).half()
        ref = torch.empty(32, 128, device=dev)
        got = torch.empty(32, 128, device=dev)
        ws_bytes = N.call("kvr_decode_attn_workspace_bytes", 32, 8, 128, n0 + n1)
        ws = torch.zeros(ws_bytes + 256, dtype=torch.uint8, device=dev)
        s = N.stream()
        N.call("kvr_decode_attn", *_args(q, k0, v0, k1, v1), N.ptr(ref), N.KVR_F32, N.ptr(ws), ws.numel(), s)
        N.call("kvr_decode_attn_noalloc", *_args(q, k0, v0, k1, v1), N.ptr(got), N.KVR_F32, s)
        torch.cuda.synchronize()
        a, b = got.cpu().numpy(), ref.cpu().numpy()
        assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max()


def _noalloc_need(n_q, n_kv, n_tok):
    """Scratch bytes the allocation-free call needs for n_tok tokens (a
    multiple of 64): kvr_decode_attn_workspace_bytes counts two spare 64-token
    units that the allocation-free call does not reserve."""
    from kvr_b200 import _native as N
    assert n_tok % 64 == 0 and n_tok >= 128
    return N.call("kvr_decode_attn_workspace_bytes", n_q, n_kv, 128, n_tok - 128)


def test_noalloc_larger_then_smaller_head_count():
    """A call with more KV heads leaves counters and partials in the shared
    array beyond what a later call with fewer heads uses; the later call must
    not pick them up."""
    from kvr_b200 import _native as N
    dev = "cuda"
    s = N.stream()
    for seed, (n_kv, g_, n) in enumerate([(8, 4, 640), (2, 4, 256), (8, 8, 128), (1, 2, 64)]):
        gen = torch.Generator(device=dev).manual_seed(100 + seed)
        n_q = n_kv * g_
        q = torch.randn(n_q, 128, device=dev, generator=gen)
        k = torch.randn(n, n_kv, 128, device=dev, generator=gen).half()
        v = torch.randn(n, n_kv, 128, device=dev, generator=gen).half()
        ref = torch.empty(n_q, 128, device=dev)
        got = torch.empty(n_q, 128, device=dev)
        ws = torch.zeros(N.call("kvr_decode_attn_workspace_bytes", n_q, n_kv, 128, n) + 256, dtype=torch.uint8,
                         device=dev)
        N.call("kvr_decode_attn", *_args(q, k, v, k[:0], v[:0]), N.ptr(ref), N.KVR_F32, N.ptr(ws), ws.numel(), s)
        N.call("kvr_decode_attn_noalloc", *_args(q, k, v, k[:0], v[:0]), N.ptr(got), N.KVR_F32, s)
        torch.cuda.synchronize()
        a, b = got.cpu().numpy(), ref.cpu().numpy()
        assert np.abs(a - b).max() <= 1e-5 * np.abs(b).max(), (n_kv, g_, n)


def test_noalloc_rejects_oversized_calls():
    from kvr_b200 import _native as N
    dev = "cuda"
    limit = N.call("kvr_decode_attn_noalloc_max_scratch_bytes")
    n = 128
    while _noalloc_need(64, 8, n) <= limit:
        n *= 2
    assert _noalloc_need(64, 8, n) > limit
    q = torch.zeros(64, 128, device=dev)
    k = torch.zeros(n, 8, 128, device=dev, dtype=torch.float16)
    out = torch.empty(64, 128, device=dev)
    with pytest.raises(N.KvrError, match="scratch"):
        N.call("kvr_decode_attn_noalloc", *_args(q, k, k, k[:0], k[:0]), N.ptr(out), N.KVR_F32, N.stream())

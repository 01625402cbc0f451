"""Torch-facing wrappers of the native kernels (one per C-ABI entry point).

All tensors must live on a CUDA device; outputs are allocated here with torch
(the C ABI itself never allocates).  Shapes follow the reference
(modules/kvr_retrieval.py, modules/kvr_window.py) unless noted.
"""
from __future__ import annotations

import contextlib
import math

import torch

from . import _native as N
from ._native import call, dtype_code, ptr, stream

D = 128


def _c(t):
    return t if t.is_contiguous() else t.contiguous()


# ------------------------------------------------------------------ int4w --


def absmax_scales(x: torch.Tensor, clamp_min: float = 1e-8) -> torch.Tensor:
    """calibrate()'s k_scales (kvr_retrieval.py:99): (n, ...) -> (...) fp32."""
    x = _c(x)
    n = x.shape[0]
    out = torch.empty(x.shape[1:], dtype=torch.float32, device=x.device)
    call("kvr_absmax_scales", ptr(x), dtype_code(x), n, out.numel(), clamp_min, ptr(out), stream())
    return out


def int4w_encode_k(k: torch.Tensor, k_scales: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """(n, n_kv, d) -> packed (n, n_kv, d/2) uint8 (kvr_retrieval.py:190-193)."""
    n, n_kv, d = k.shape
    if k.stride(2) != 1 or k.stride(1) != d:
        k = k.contiguous()
    ks = _c(k_scales.float())
    if out is None:
        out = torch.empty(n, n_kv, d // 2, dtype=torch.uint8, device=k.device)
    call("kvr_int4w_encode_k", ptr(k), dtype_code(k), n, n_kv, d, k.stride(0), ptr(ks), ptr(out), stream())
    return out


def int4w_encode_vres(v, v_pred, vr_scales, out=None):
    """(n, n_kv, d) -> packed (n, n_kv, d/4) uint8 (kvr_retrieval.py:196-203)."""
    v = _c(v)
    n, n_kv, d = v.shape
    vp = _c(v_pred.float())
    vr = _c(vr_scales.float().reshape(-1))
    if out is None:
        out = torch.empty(n, n_kv, d // 4, dtype=torch.uint8, device=v.device)
    call("kvr_int4w_encode_vres", ptr(v), dtype_code(v), ptr(vp), n, n_kv, d, ptr(vr), ptr(out), stream())
    return out


def compute_scores(q_avg, k_packed, k_scales, cos_tbl, sin_tbl, n_stored=None):
    """Drop-in for the reference native kernel (kvr_cuda.cu:53-77)."""
    n_kv, d = k_packed.shape[1], k_packed.shape[2] * 2
    n = k_packed.shape[0] if n_stored is None else n_stored
    q = _c(q_avg.float())
    out = torch.empty(n, n_kv, dtype=torch.float32, device=q.device)
    call("kvr_compute_scores", ptr(q), ptr(_c(k_packed)), ptr(_c(k_scales.float())), ptr(_c(cos_tbl.float())),
         ptr(_c(sin_tbl.float())), n_kv, d, n, ptr(out), stream())
    return out


def _rope_args(cos, sin):
    if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.stride(0) != sin.stride(0):
        cos, sin = cos.contiguous(), sin.contiguous()
    return cos, sin, cos.stride(0)


def int4w_token_scores(q_post, k_packed, k_scales, cos, sin, n_stored, halves_equal=False, out=None):
    """compute_all_scores (kvr_retrieval.py:265-289) -> HEAD-MAJOR (n_kv, n_stored)."""
    n_kv = k_packed.shape[1]
    q = _c(q_post.float())
    cos, sin, rs = _rope_args(cos.float(), sin.float())
    if out is None:
        out = torch.empty(n_kv, n_stored, dtype=torch.float32, device=q.device)
    call("kvr_int4w_token_scores", ptr(q), q.shape[0], ptr(_c(k_packed)), ptr(_c(k_scales.float())), ptr(cos),
         ptr(sin), rs, int(halves_equal), n_kv, D, n_stored, ptr(out), out.stride(0), stream())
    return out


def int4w_token_topk(q_post, k_packed, k_scales, cos, sin, n_stored, k, halves_equal=False, ex_start=0, ex_end=0):
    """Token branch of retrieve_topk in one call (scores + exclusion + top-k,
    kvr_retrieval.py:265-289, 389-392) -> idx (k, n_kv) int64."""
    n_kv = k_packed.shape[1]
    q = _c(q_post.float())
    cos, sin, rs = _rope_args(cos.float(), sin.float())
    idx = torch.empty(k, n_kv, dtype=torch.int64, device=q.device)
    ws = N.workspace("int4w_topk", call("kvr_int4w_token_topk_workspace_bytes", n_kv, n_stored, k), q.device)
    call("kvr_int4w_token_topk", ptr(q), q.shape[0], ptr(_c(k_packed)), ptr(_c(k_scales.float())), ptr(cos),
         ptr(sin), rs, int(halves_equal), n_kv, D, n_stored, k, ex_start, ex_end, ptr(idx), ptr(ws), ws.numel(),
         stream())
    return idx


def int4w_chunk_scores(q_post, k_packed, k_scales, cos, sin, n_stored, chunk, halves_equal=False):
    """compute_chunk_scores (kvr_retrieval.py:291-315) -> HEAD-MAJOR (n_kv, n_stored // chunk)."""
    n_kv = k_packed.shape[1]
    q = _c(q_post.float())
    cos, sin, rs = _rope_args(cos.float(), sin.float())
    nc = n_stored // chunk
    out = torch.empty(n_kv, nc, dtype=torch.float32, device=q.device)
    call("kvr_int4w_chunk_scores", ptr(q), q.shape[0], ptr(_c(k_packed)), ptr(_c(k_scales.float())), ptr(cos),
         ptr(sin), rs, int(halves_equal), n_kv, D, n_stored, chunk, ptr(out), out.stride(0), stream())
    return out


def topk_rows(scores: torch.Tensor, k: int, ex_start: int = 0, ex_end: int = 0, transpose_out: bool = False):
    """Per-row top-k of (rows, n) fp32, (score desc, index asc); entries in
    [ex_start, ex_end) and NaN count as -inf.  Returns (idx int64, vals fp32)
    shaped (rows, k), or (k, rows) when transpose_out."""
    assert scores.dim() == 2 and scores.stride(1) == 1 and scores.dtype == torch.float32
    rows, n = scores.shape
    shape = (k, rows) if transpose_out else (rows, k)
    idx = torch.empty(shape, dtype=torch.int64, device=scores.device)
    vals = torch.empty(shape, dtype=torch.float32, device=scores.device)
    ors, oes = (1, rows) if transpose_out else (k, 1)
    call("kvr_topk_rows", ptr(scores), rows, n, scores.stride(0), k, ex_start, ex_end, ptr(idx), ptr(vals), ors, oes,
         stream())
    return idx, vals


def int4w_gather(k_packed, k_scales, top, cos, sin, k_mean=None, want_x=True, count=None, ret_k=None):
    """-> (ret_k (k, n_kv, d) fp32 post-RoPE, x (n_kv, k, n_kv*d) fp32 = deq
    K_pre - K_mean, or None when want_x is False).  count: optional device
    int32 row count (rows past it are left untouched)."""
    k, n_kv = top.shape
    cos, sin, rs = _rope_args(cos.float(), sin.float())
    if ret_k is None:
        ret_k = torch.empty(k, n_kv, D, dtype=torch.float32, device=top.device)
    x = torch.empty(n_kv, k, n_kv * D, dtype=torch.float32, device=top.device) if want_x else None
    km = _c(k_mean.float().reshape(-1)) if want_x else None
    call("kvr_int4w_gather", ptr(_c(k_packed)), ptr(_c(k_scales.float())), ptr(_c(top)), k, n_kv, D, ptr(cos),
         ptr(sin), rs, ptr(km), ptr(ret_k), ptr(x), ptr(count), stream())
    return ret_k, x


def int4w_vpredict_prepare(W, k_mean, v_mean, k_scales, n_kv):
    """Once per calibration: (w3, unscale fp32 (n_kv*d), bias fp32 (n_kv*d))
    for int4w_vpredict; w3 holds the fp16 hi/lo parts of W' = W diag(step) in
    the kernel's tensor-core operand layout (n_kv*2*d*n_kv*d halves)."""
    dev = W.device
    KD = n_kv * D
    w3 = torch.empty(n_kv, 2, D, KD, dtype=torch.float16, device=dev)
    unscale = torch.empty(KD, dtype=torch.float32, device=dev)
    bias = torch.empty(KD, dtype=torch.float32, device=dev)
    call("kvr_int4w_vpredict_prepare", ptr(_c(W.float())), ptr(_c(k_mean.float().reshape(-1))),
         ptr(_c(v_mean.float().reshape(-1))), ptr(_c(k_scales.float().reshape(-1))), n_kv, D, ptr(w3),
         ptr(unscale), ptr(bias), stream())
    return w3, unscale, bias


def int4w_vpredict(k_packed, top, prep, vr_packed, vr_scales, count=None, out=None):
    """ret_v (k, n_kv, d) fp16 = W-predicted V + int2 residual of the tokens
    top (k, n_kv) int64 (kvr_retrieval.py:394-402), on the tensor cores."""
    k, n_kv = top.shape
    w3, unscale, bias = prep
    if out is None:
        out = torch.empty(k, n_kv, D, dtype=torch.float16, device=top.device)
    call("kvr_int4w_vpredict", ptr(_c(k_packed)), ptr(_c(top)), ptr(count), k, n_kv, D, ptr(w3), ptr(unscale),
         ptr(bias), ptr(_c(vr_packed)), ptr(_c(vr_scales.float().reshape(-1))), ptr(out), stream())
    return out


def int4w_vpredict_status():
    """Raises if a bounded device-side wait of the V-predict kernel gave up
    since the last check (synchronises the current stream)."""
    call("kvr_int4w_vpredict_status", stream())


def int4w_attractor_select(q, n_kv, k_packed, k_scales, cos, sin, centroids, labels, n_labelled, top_a=48,
                           ex_start=0, ex_end=0):
    """Attractor branch selection (kvr_retrieval.py:332-367) on the device:
    labels int32 (>= n_labelled) -> (top (top_a*16, n_kv) int64, count (1,)
    int32 device tensor)."""
    q = _c(q.float())
    n_q = q.shape[0]
    cos, sin, rs = _rope_args(cos.float(), sin.float())
    rows = top_a * 16
    top = torch.empty(rows, n_kv, dtype=torch.int64, device=q.device)
    count = torch.empty(1, dtype=torch.int32, device=q.device)
    ws = N.workspace("attractor", call("kvr_int4w_attractor_workspace_bytes", n_labelled, top_a), q.device)
    call("kvr_int4w_attractor_select", ptr(q), n_q, n_kv, ptr(_c(k_packed)), ptr(_c(k_scales.float())), ptr(cos),
         ptr(sin), rs, ptr(_c(centroids.float())), centroids.shape[0], ptr(_c(labels)), n_labelled, top_a, ex_start,
         ex_end, ptr(top), ptr(count), ptr(ws), ws.numel(), stream())
    return top, count


def int4w_assign_basins(k_packed, k_scales, t0, t1, centroids, labels):
    """labels[t0:t1] (int32, in place) = nearest basin of each token's head-0 K."""
    call("kvr_int4w_assign_basins", ptr(_c(k_packed)), ptr(_c(k_scales.float())), k_packed.shape[1], t0, t1,
         ptr(_c(centroids.float())), centroids.shape[0], ptr(labels), stream())


# ----------------------------------------------------------------- window --


def window_write(k, v, ring_k, ring_v, pos: int):
    """Ring write of n tokens at slots (pos + i) % cap (kvr_window.py:19-41)."""
    k, v = _c(k), _c(v)
    if v.dtype != k.dtype:
        v = v.to(k.dtype)
    n = k.shape[0]
    n_kv, d = ring_k.shape[1], ring_k.shape[2]
    call("kvr_window_write", ptr(k), ptr(v), dtype_code(k), n, n_kv, d, ptr(ring_k), ptr(ring_v), ring_k.shape[0],
         pos, stream())


def decode_store_update(q, k, v, cos, sin, pos, ring_k, ring_v, slot, tail_k=None, tail_v=None, tail_row=0,
                        write_kv=True, q_out=None):
    """One decode step's RoPE + window write (+ eviction of the slot's old row
    into the sd1 tail) in one launch.  q (n_q, d), k/v (n_kv, d) of the model
    dtype -> q_out = RoPE(q) (same dtype)."""
    q, k, v = _c(q), _c(k), _c(v)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k and v must share a dtype")
    cos, sin, rs = _rope_args(cos, sin)
    if q_out is None:
        q_out = torch.empty_like(q)
    call("kvr_decode_store_update", ptr(q), ptr(k), ptr(v), dtype_code(q), q.shape[0], k.shape[0], D, ptr(cos),
         ptr(sin), rs, pos, ptr(q_out), ptr(ring_k), ptr(ring_v), ring_k.shape[0], slot, ptr(tail_k), ptr(tail_v),
         tail_row, int(write_kv), stream())
    return q_out


# -------------------------------------------------------------- attention --


def _seg_rows(k, v, d):
    if k.stride(-1) != 1 or k.stride(-2) != d:
        k = k.contiguous()
    if v.stride(-1) != 1 or v.stride(-2) != d or v.stride(0) != k.stride(0):
        v = v.contiguous()
        if v.stride(0) != k.stride(0):
            k = k.contiguous()
    return k, v


def decode_attn(q, segments, scale=None, out_dtype=None, n_kv=None, n1_count=None, out=None):
    """Exact attention of q (n_q, d) over up to two K/V segments
    [(k0, v0), (k1, v1)], each (n_i, n_kv, d) with contiguous rows.
    n1_count: optional device int32 holding how many rows of the second
    segment are valid (kvr_decode_attn_counted)."""
    q = _c(q)
    n_q, d = q.shape
    if n_kv is None:
        n_kv = segments[0][0].shape[1]
    segs = [_seg_rows(k, v, d) if k.shape[0] else None for k, v in segments]
    if n1_count is None:
        segs = [sg for sg in segs if sg is not None]
    while len(segs) < 2:
        segs.append(None)
    if segs[1] is None:
        n1_count = None
    out_dtype = out_dtype or q.dtype
    if out is None:
        out = torch.empty(n_q, d, dtype=out_dtype, device=q.device)
    n_tot = sum(sg[0].shape[0] for sg in segs if sg is not None)
    ws = N.workspace("attn", call("kvr_decode_attn_workspace_bytes", n_q, n_kv, d, n_tot), q.device)
    args = []
    for sg in segs:
        if sg is not None:
            k, v = sg
            args.append([ptr(k), ptr(v), dtype_code(k), dtype_code(v), k.shape[0], k.stride(0)])
        else:
            args.append([None, None, 0, 0, 0, 0])
    if n1_count is not None:
        call("kvr_decode_attn_counted", ptr(q), dtype_code(q), n_q, n_kv, d, *args[0], *args[1], ptr(n1_count),
             float(scale or 0.0), ptr(out), dtype_code(out), ptr(ws), ws.numel(), stream())
    else:
        call("kvr_decode_attn", ptr(q), dtype_code(q), n_q, n_kv, d, *args[0], *args[1], float(scale or 0.0),
             ptr(out), dtype_code(out), ptr(ws), ws.numel(), stream())
    return out


def lse_merge(partials: torch.Tensor, out_dtype=torch.float32):
    """partials (P, n_q, d+2) [m, l, o] -> (n_q, d)."""
    p = _c(partials.float())
    P_, n_q, dd = p.shape
    out = torch.empty(n_q, dd - 2, dtype=out_dtype, device=p.device)
    call("kvr_lse_merge", ptr(p), P_, n_q, dd - 2, ptr(out), dtype_code(out), stream())
    return out


def merge_candidates(scores, idx, k_sel, tile_base=0, n_local=0, global_out=True):
    """scores fp32 / idx int32 (N, B, H, k_local) gathered candidates ->
    (global_sel (B, H, k_sel) int32 or None, local_sel (B, H, k_sel) int32)."""
    N_, B, H, kl = scores.shape
    sc, ix = _c(scores.float()), _c(idx.to(torch.int32))
    lsel = torch.empty(B, H, k_sel, dtype=torch.int32, device=sc.device)
    gsel = torch.empty_like(lsel) if global_out else None
    call("kvr_merge_candidates", ptr(sc), ptr(ix), N_, B * H, kl, k_sel, tile_base, n_local, ptr(gsel), ptr(lsel),
         stream())
    return gsel, lsel


# -------------------------------------------------------------------- sd1 --


def transform(x: torch.Tensor, kind: str = "hadamard", inverse: bool = False) -> torch.Tensor:
    """Orthonormal Hadamard / DCT along the last axis (d = 128), fp32."""
    x = _c(x.float())
    y = torch.empty_like(x)
    call("kvr_transform", ptr(x), ptr(y), x.numel() // D, N.TRANSFORMS[kind], int(inverse), stream())
    return y


class Sd1Store:
    """Device buffers of one layer's 1-bit store for `batch` sequences x n_kv heads.

    kbits/vbits (B, n_kv, nt_cap, tile, 4) uint32 (stored as int32 tensors),
    kscale/vscale (B, n_kv, nt_cap, 128) fp16.  `n_tiles` full tiles are valid."""

    def __init__(self, batch, n_kv, nt_cap, tile=64, kind="hadamard", device="cuda"):
        if tile not in (32, 64, 128):
            raise ValueError("tile must be 32, 64 or 128")
        self.batch, self.n_kv, self.nt_cap, self.tile, self.kind = batch, n_kv, nt_cap, tile, kind
        self.kbits = torch.zeros(batch, n_kv, nt_cap, tile, 4, dtype=torch.int32, device=device)
        self.vbits = torch.zeros_like(self.kbits)
        self.kscale = torch.zeros(batch, n_kv, nt_cap, D, dtype=torch.float16, device=device)
        self.vscale = torch.zeros_like(self.kscale)
        self.n_tiles = 0

    @property
    def nbytes(self):
        return sum(t.numel() * t.element_size() for t in (self.kbits, self.vbits, self.kscale, self.vscale))

    def grow(self, nt_cap):
        if nt_cap <= self.nt_cap:
            return
        def ext(t):
            z = torch.zeros(*t.shape[:2], nt_cap - self.nt_cap, *t.shape[3:], dtype=t.dtype, device=t.device)
            return torch.cat([t, z], 2)
        self.kbits, self.vbits = ext(self.kbits), ext(self.vbits)
        self.kscale, self.vscale = ext(self.kscale), ext(self.vscale)
        self.nt_cap = nt_cap


def sd1_encode(store: Sd1Store, k, v, n_tiles=None, tile0=None, cos=None, sin=None, pos0=0):
    """Encode full tiles of k, v ((B, n, n_kv, d) or (n, n_kv, d)) into the store
    starting at tile `tile0` (default: store.n_tiles, then advances n_tiles)."""
    if k.dim() == 3:
        k, v = k.unsqueeze(0), v.unsqueeze(0)
    B, n, n_kv, d = k.shape
    if v.dtype != k.dtype:
        v = v.to(k.dtype)
    if k.stride(-1) != 1 or k.stride(-2) != d:
        k = k.contiguous()
    if v.stride() != k.stride():
        k, v = k.contiguous(), v.contiguous()
    nt = n // store.tile if n_tiles is None else n_tiles
    t0 = store.n_tiles if tile0 is None else tile0
    if cos is not None:
        cos, sin, rs = _rope_args(cos.float(), sin.float())
    else:
        rs = 0
    call("kvr_sd1_encode", ptr(k), ptr(v), dtype_code(k), B, n_kv, nt, store.tile, k.stride(0), k.stride(1),
         ptr(cos), ptr(sin), rs, pos0, N.TRANSFORMS[store.kind], ptr(store.kbits), ptr(store.kscale),
         ptr(store.vbits), ptr(store.vscale), store.nt_cap, t0, stream())
    if tile0 is None:
        store.n_tiles = t0 + nt
    return nt


def sd1_tile_scores(store: Sd1Store, q):
    """q (B, n_q, d) -> (B, n_kv, n_tiles) fp32 selection scores."""
    q = _c(q if q.dim() == 3 else q.unsqueeze(0))
    B, n_q, _ = q.shape
    out = torch.empty(B, store.n_kv, max(store.n_tiles, 0), dtype=torch.float32, device=q.device)
    call("kvr_sd1_tile_scores", ptr(q), dtype_code(q), B, n_q, store.n_kv, ptr(store.kbits), ptr(store.kscale),
         store.nt_cap, store.n_tiles, store.tile, N.TRANSFORMS[store.kind], ptr(out), stream())
    return out


def sd1_select(store: Sd1Store, q, k_sel, ex_t0=0, ex_t1=0, tile_base=0, n_tiles=None):
    """-> (sel (B, n_kv, k_sel) int32, sel_scores fp32, qprime (B, n_q, d) fp32)."""
    q = _c(q if q.dim() == 3 else q.unsqueeze(0))
    B, n_q, _ = q.shape
    nt = store.n_tiles if n_tiles is None else n_tiles
    sel = torch.empty(B, store.n_kv, k_sel, dtype=torch.int32, device=q.device)
    sc = torch.empty(B, store.n_kv, k_sel, dtype=torch.float32, device=q.device)
    qp = torch.empty(B, n_q, D, dtype=torch.float32, device=q.device)
    ws = N.workspace("sd1_select", call("kvr_sd1_select_workspace_bytes", B, store.n_kv, nt), q.device)
    call("kvr_sd1_select", ptr(q), dtype_code(q), B, n_q, store.n_kv, ptr(store.kbits), ptr(store.kscale),
         store.nt_cap, nt, store.tile, N.TRANSFORMS[store.kind], k_sel, ex_t0, ex_t1, tile_base, ptr(sel), ptr(sc),
         ptr(qp), ptr(ws), ws.numel(), stream())
    return sel, sc, qp


def _win_args(win_k, win_v, n_win):
    if win_k is None or n_win == 0:
        return None, None, 1, 0
    return ptr(win_k), ptr(win_v), win_k.shape[-3], n_win


def sd1_attend(store: Sd1Store, q, qprime, sel, win_k=None, win_v=None, n_win=0, tail_k=None, tail_v=None,
               n_tail=0, scale=None, out_dtype=None, partial=False):
    """Attention over window (B, cap, n_kv, d) fp16 + tail (B, t, n_kv, d) fp16 +
    selected tiles.  Returns out (B, n_q, d) or partial rows (B, n_q, d+2)."""
    q = _c(q if q.dim() == 3 else q.unsqueeze(0))
    B, n_q, _ = q.shape
    k_sel = sel.shape[-1]
    out_dtype = out_dtype or q.dtype
    if partial:
        part = torch.empty(B, n_q, D + 2, dtype=torch.float32, device=q.device)
        out = None
    else:
        out = torch.empty(B, n_q, D, dtype=out_dtype, device=q.device)
        part = None
    wk, wv, wcap, nw = _win_args(win_k, win_v, n_win)
    tk, tv = (ptr(tail_k), ptr(tail_v)) if n_tail else (None, None)
    ws = N.workspace("sd1_attend", call("kvr_sd1_attend_workspace_bytes", B, n_q, store.n_kv, store.tile, k_sel, nw,
                                        n_tail), q.device)
    call("kvr_sd1_attend", ptr(q), dtype_code(q), ptr(qprime), B, n_q, store.n_kv, wk, wv, wcap, nw, tk, tv, n_tail,
         ptr(store.kbits), ptr(store.kscale), ptr(store.vbits), ptr(store.vscale), store.nt_cap, store.tile,
         N.TRANSFORMS[store.kind], ptr(_c(sel)), k_sel, float(scale or 0.0), ptr(out),
         dtype_code(out) if out is not None else 0, ptr(part), ptr(ws), ws.numel(), stream())
    return part if partial else out


_STEP_WS: dict = {}


@contextlib.contextmanager
def sd1_step_path(path):
    """Within the block, kvr_sd1_decode_step runs the one-kernel cluster path
    where shapes allow ("cluster", the default; "cluster8": 8-CTA clusters
    only) or always the selection + attention kernels ("split").
    Process-wide; restores the previous value."""
    fn = N.lib().kvr_set_sd1_step_path  # returns the previous value, not a status
    prev = fn({"cluster": 0, "split": 1, "cluster8": 2}[path])
    try:
        yield
    finally:
        fn(prev)


def sd1_decode_step(store: Sd1Store, q, k_sel, win_k=None, win_v=None, n_win=0, tail_k=None, tail_v=None,
                    n_tail=0, ex_t0=0, ex_t1=0, scale=None, out=None, sel_out=None, ws=None):
    """Tile selection + attention in one call: one cluster kernel for few rows,
    else the selection and attention kernels.  Returns out (B, n_q, d)."""
    q = _c(q if q.dim() == 3 else q.unsqueeze(0))
    B, n_q, _ = q.shape
    if out is None:
        out = torch.empty(B, n_q, D, dtype=q.dtype, device=q.device)
    wk, wv, wcap, nw = _win_args(win_k, win_v, n_win)
    tk, tv = (ptr(tail_k), ptr(tail_v)) if n_tail else (None, None)
    if ws is None:
        key = (B, n_q, store.n_kv, store.n_tiles, store.tile, k_sel, nw, n_tail)
        need = _STEP_WS.get(key)
        if need is None:
            need = _STEP_WS[key] = call("kvr_sd1_workspace_bytes", *key)
            if len(_STEP_WS) > 4096:
                _STEP_WS.clear()
        ws = N.workspace("sd1_step", need, q.device)
    call("kvr_sd1_decode_step", ptr(q), dtype_code(q), B, n_q, store.n_kv, wk, wv, wcap, nw, tk, tv, n_tail,
         ptr(store.kbits), ptr(store.kscale), ptr(store.vbits), ptr(store.vscale), store.nt_cap, store.n_tiles,
         store.tile, N.TRANSFORMS[store.kind], k_sel, ex_t0, ex_t1, float(scale or 0.0), ptr(out), dtype_code(out),
         ptr(sel_out), ptr(ws), ws.numel(), stream())
    return out


def sd1_decode_step_update(store: Sd1Store, q, k, v, cos, sin, pos, k_sel, win_k, win_v, n_win, slot,
                           tail_k=None, tail_v=None, n_tail=0, evict=False, ex_t0=0, ex_t1=0, scale=None,
                           out=None, q_out=None, sel_out=None, ws=None):
    """The layer's store update fused with its decode step (batch 1).

    q (n_q, d), k and v (n_kv, d): the new token's pre-RoPE rows, one dtype.
    The rotated K / V land in window slot `slot` (one of the n_win rows
    attended, n_win counting the new row); with `evict` the slot's old row
    first moves to tail row n_tail - 1.  Returns (out (1, n_q, d) of q's
    dtype, q_out = RoPE(q))."""
    q, k, v = _c(q), _c(k), _c(v)
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise TypeError("q, k and v must share a dtype")
    n_q, n_kv = q.shape[0], k.shape[0]
    cos, sin, rs = _rope_args(cos, sin)
    if out is None:
        out = torch.empty(1, n_q, D, dtype=q.dtype, device=q.device)
    if q_out is None:
        q_out = torch.empty_like(q)
    if ws is None:
        key = (1, n_q, n_kv, store.n_tiles, store.tile, k_sel, n_win, n_tail)
        need = _STEP_WS.get(key)
        if need is None:
            need = _STEP_WS[key] = call("kvr_sd1_workspace_bytes", *key)
            if len(_STEP_WS) > 4096:
                _STEP_WS.clear()
        ws = N.workspace("sd1_step", need, q.device)
    call("kvr_sd1_decode_step_update", ptr(q), ptr(k), ptr(v), dtype_code(q), n_q, n_kv, ptr(cos), ptr(sin), rs,
         pos, ptr(q_out), ptr(win_k), ptr(win_v), win_k.shape[-3], n_win, slot, ptr(tail_k), ptr(tail_v), n_tail,
         int(evict), ptr(store.kbits), ptr(store.kscale), ptr(store.vbits), ptr(store.vscale), store.nt_cap,
         store.n_tiles, store.tile, N.TRANSFORMS[store.kind], k_sel, ex_t0, ex_t1, float(scale or 0.0), ptr(out),
         dtype_code(out), ptr(sel_out), ptr(ws), ws.numel(), stream())
    return out, q_out


def sd1_decode_tiles(store: Sd1Store, sel):
    """sel (B, n_kv, k) int64 -> (K (B, k*t, n_kv, d) fp32, V fp16)."""
    sel = _c(sel.long())
    B, n_kv, k = sel.shape
    ok = torch.empty(B, k * store.tile, n_kv, D, dtype=torch.float32, device=sel.device)
    ov = torch.empty(B, k * store.tile, n_kv, D, dtype=torch.float16, device=sel.device)
    call("kvr_sd1_decode_tiles", ptr(store.kbits), ptr(store.kscale), ptr(store.vbits), ptr(store.vscale),
         store.nt_cap, B, n_kv, store.tile, N.TRANSFORMS[store.kind], ptr(sel), k, ptr(ok), ptr(ov), stream())
    return ok, ov


def sd1_prefill_scores(store: Sd1Store, q):
    """Tensor-core tile scores for a block of prefill queries (batch-1 store):
    q (nq, n_q, d) -> (nq, n_kv, n_tiles) fp32."""
    if store.batch != 1:
        raise ValueError("prefill scoring takes a batch-1 store")
    q = _c(q)
    nq, n_q, _ = q.shape
    out = torch.empty(nq, store.n_kv, store.n_tiles, dtype=torch.float32, device=q.device)
    ws = N.workspace("sd1_prefill", call("kvr_sd1_prefill_workspace_bytes", nq, store.n_kv), q.device)
    call("kvr_sd1_prefill_scores", ptr(q), dtype_code(q), nq, n_q, store.n_kv, ptr(store.kbits), ptr(store.kscale),
         store.nt_cap, store.n_tiles, store.tile, N.TRANSFORMS[store.kind], ptr(out), ptr(ws), ws.numel(), stream())
    return out


def kmeans(x, k=128, iters=10):
    """Deterministic Lloyd k-means on the device: x (n, 128) -> (labels (n,)
    int32, centroids (k, 128) fp32)."""
    x = _c(x.float())
    n = x.shape[0]
    c = torch.empty(k, D, dtype=torch.float32, device=x.device)
    lab = torch.empty(n, dtype=torch.int32, device=x.device)
    ws = N.workspace("kmeans", call("kvr_kmeans_workspace_bytes", n, k), x.device)
    call("kvr_kmeans", ptr(x), n, D, k, iters, ptr(c), ptr(lab), ptr(ws), ws.numel(), stream())
    return lab, c


def workspace_status(ws: torch.Tensor):
    call("kvr_workspace_status", ptr(ws), stream())


def default_scale(d=D):
    return math.sqrt(d)

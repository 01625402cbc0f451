"""CPU oracle for the reference-faithful ``int4w`` codec — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy (byte/integer work) and plain torch-CPU (the one
place where the reference leans on a LAPACK routine, ``calibrate``), the
algorithm of the reference's compressed-KV path:

* ``modules/kvr_retrieval.py`` — int4 K codes, int2 V-residual codes, scoring,
  chunk scoring, top-k retrieval and V reconstruction;
* ``modules/kvr_window.py``    — fp16 ring window and its exact attention;
* ``modules/kvr_cuda.cu``      — the (dead-in-the-live-path) interleaved-RoPE
  score kernel;
* ``modules/kvr_hook.py``      — the concatenated window+retrieved softmax.

Each function cites the reference file:line it follows.  Parity of this
restatement is PINNED against fixtures produced by running the reference itself
(``tests/golden/make_golden.py`` -> ``tests/golden/int4w_golden.npz``; checked by
``tests/test_oracle_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
may import this module, and only as the checker.  The product path never
routes through it.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32

# --------------------------------------------------------------------------
# bit packing (kvr_retrieval.py:69-91)
# --------------------------------------------------------------------------


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:69-72 — u = code+8; even element -> high nibble, odd -> low."""
    u = (codes.astype(np.int16) + 8).astype(np.uint8)
    return ((u[..., 0::2] << 4) | u[..., 1::2]).astype(np.uint8)


def unpack_int4(p: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:74-78."""
    hi = (p >> 4).astype(np.int8) - 8
    lo = (p & 0x0F).astype(np.int8) - 8
    return np.stack([hi, lo], axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)


def pack_int2(codes: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:80-83 — u = code+2; element 0 in bits 7-6 ... element 3 in bits 1-0."""
    u = (codes.astype(np.int16) + 2).astype(np.uint8)
    return ((u[..., 0::4] << 6) | (u[..., 1::4] << 4) | (u[..., 2::4] << 2) | u[..., 3::4]).astype(np.uint8)


def unpack_int2(p: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:85-91."""
    parts = [((p >> s) & 0x03).astype(np.int8) - 2 for s in (6, 4, 2, 0)]
    return np.stack(parts, axis=-1).reshape(*p.shape[:-1], p.shape[-1] * 4)


# --------------------------------------------------------------------------
# calibration (kvr_retrieval.py:95-122) — torch CPU, the reference's own numerics
# --------------------------------------------------------------------------


def calibrate(k_pre: np.ndarray, v: np.ndarray | None):
    """kvr_retrieval.py:95-122.

    Returns a dict with k_scales (n_kv, d), W (D, D), K_mean (1, D), V_mean (1, D),
    vr_scales (n_kv, 1), all float32.  ``torch.linalg.pinv`` has no pinned
    algorithm in the reference, so the restatement calls the same torch routine.
    """
    import torch

    k_t = torch.from_numpy(np.ascontiguousarray(k_pre))
    n, n_kv, d = k_t.shape
    D = n_kv * d
    k2 = k_t.reshape(n, D).float()
    out = {"k_scales": k_t.abs().max(dim=0).values.clamp(min=1e-8).float().numpy()}
    if v is not None and n > 10:
        v2 = torch.from_numpy(np.ascontiguousarray(v)).reshape(n, D).float()
        half = n // 2
        k_tr, v_tr = k2[:half], v2[:half]
        K_mean = k_tr.mean(0, keepdim=True)
        V_mean = v_tr.mean(0, keepdim=True)
        kc = k_tr - K_mean
        vc = v_tr - V_mean
        W = (kc.T @ vc).T @ torch.linalg.pinv(kc.T @ kc)
        v_pred_all = (k2 - K_mean) @ W.T + V_mean
        v_res = v2 - v_pred_all
        vr_scales = v_res.view(-1, n_kv, d).abs().amax(dim=(0, 2)).unsqueeze(1).clamp(min=1e-8)
        out.update(W=W.numpy(), K_mean=K_mean.numpy(), V_mean=V_mean.numpy(), vr_scales=vr_scales.numpy())
    else:
        out.update(W=np.eye(D, dtype=F32), K_mean=np.zeros((1, D), F32),
                   V_mean=np.zeros((1, D), F32), vr_scales=np.ones((n_kv, 1), F32))
    return out


# --------------------------------------------------------------------------
# encoder (kvr_retrieval.py:162-207)
# --------------------------------------------------------------------------


def k_step(k_scales: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:126,167,190 — step = 2*scale/16 (exact in fp32)."""
    return (F32(2.0) * k_scales.astype(F32)) / F32(16.0)


def quantize_k(k_pre: np.ndarray, k_scales: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:190-191 — clamp(round_half_even(k/step), -8, 7)."""
    q = np.rint(k_pre.astype(F32) / k_step(k_scales))
    return np.clip(q, -8, 7).astype(np.int8)


def predict_v(k_flat: np.ndarray, W, K_mean, V_mean) -> np.ndarray:
    """kvr_retrieval.py:131-134 — (k - mu_k) @ W^T + mu_v (torch CPU matmul)."""
    import torch

    kt = torch.from_numpy(np.ascontiguousarray(k_flat, dtype=F32))
    r = (kt - torch.from_numpy(K_mean)) @ torch.from_numpy(W).T + torch.from_numpy(V_mean)
    return r.numpy()


def vr_step(vr_scales: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:146,176,200 — 2*vr_scale/4."""
    return (F32(2.0) * vr_scales.astype(F32)) / F32(4.0)


def quantize_vres(v: np.ndarray, v_pred: np.ndarray, vr_scales: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:199-201 — clamp(round((v - v_pred)/vr_step), -2, 1)."""
    res = v.astype(F32) - v_pred.astype(F32)
    q = np.rint(res / vr_step(vr_scales)[None])
    return np.clip(q, -2, 1).astype(np.int8)


def batch_append(k_pre: np.ndarray, v: np.ndarray, cal: dict):
    """kvr_retrieval.py:187-207.  Returns (k_packed, vr_packed, v_pred) with the
    reference's zero padding of max(1024, n//2) rows."""
    n, n_kv, d = k_pre.shape
    extra = max(1024, n // 2)
    kq = quantize_k(k_pre, cal["k_scales"])
    kp = np.concatenate([pack_int4(kq), np.zeros((extra, n_kv, d // 2), np.uint8)], 0)
    v_pred = predict_v(k_pre.reshape(n, -1), cal["W"], cal["K_mean"], cal["V_mean"]).reshape(n, n_kv, d)
    vrq = quantize_vres(v, v_pred, cal["vr_scales"])
    vp = np.concatenate([pack_int2(vrq), np.zeros((extra, n_kv, d // 4), np.uint8)], 0)
    return kp, vp, v_pred


# --------------------------------------------------------------------------
# RoPE (kvr_retrieval.py:27-37, 136-141)
# --------------------------------------------------------------------------


def rotate_half(x: np.ndarray) -> np.ndarray:
    """kvr_retrieval.py:27-29."""
    d2 = x.shape[-1] // 2
    return np.concatenate([-x[..., d2:], x[..., :d2]], axis=-1)


def apply_rotary(x, cos, sin):
    """kvr_retrieval.py:32-33 (rows of cos/sin broadcast per token)."""
    return x * cos + rotate_half(x) * sin


def reverse_rotary(x, cos, sin):
    """kvr_retrieval.py:36-37."""
    return x * cos - rotate_half(x) * sin


def rope_tables(max_pos: int, d: int, theta: float = 500000.0):
    """HF-Llama-style (max_pos, d) tables with duplicated halves (kvr_hook.py:49-55
    takes them from the model's rotary module; this is the default-rope formula)."""
    inv_freq = (1.0 / (theta ** (np.arange(0, d, 2, dtype=np.int64).astype(F32) / F32(d)))).astype(F32)
    freqs = np.arange(max_pos, dtype=F32)[:, None] * inv_freq[None, :]
    emb = np.concatenate([freqs, freqs], -1).astype(F32)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


# --------------------------------------------------------------------------
# scoring (kvr_retrieval.py:124-129, 265-315; kvr_cuda.cu:9-49)
# --------------------------------------------------------------------------


def deq_k(k_packed: np.ndarray, k_scales: np.ndarray, n_stored: int) -> np.ndarray:
    """kvr_retrieval.py:124-129 (all heads at once): (n, n_kv, d) fp32."""
    return unpack_int4(k_packed[:n_stored]).astype(F32) * k_step(k_scales)[None]


def q_group_mean(q: np.ndarray, n_kv: int) -> np.ndarray:
    """kvr_retrieval.py:270 — mean over each GQA group: (n_kv, d)."""
    n_q, d = q.shape
    return q.astype(F32).reshape(n_kv, n_q // n_kv, d).mean(axis=1, dtype=np.float64).astype(F32)


def _cosine(qa: np.ndarray, keys: np.ndarray) -> np.ndarray:
    qn = qa / (np.linalg.norm(qa.astype(np.float64)) + 1e-8)
    kn = keys / (np.linalg.norm(keys.astype(np.float64), axis=-1, keepdims=True) + 1e-8)
    return kn.astype(np.float64) @ qn.astype(np.float64)


def token_scores(q_post, k_packed, k_scales, cos, sin, n_stored):
    """kvr_retrieval.py:265-289 — cosine(q_avg, RoPE(deq K)) per (token, head); NaN -> -inf.
    Returns (n_stored, n_kv) float64 (the checker compares at rel 1e-5)."""
    n_kv = k_packed.shape[1]
    qa = q_group_mean(q_post, n_kv)
    kp = deq_k(k_packed, k_scales, n_stored)
    c, s = cos[:n_stored, None, :], sin[:n_stored, None, :]
    kr = apply_rotary(kp, c, s).astype(F32)
    out = np.stack([_cosine(qa[h], kr[:, h]) for h in range(n_kv)], 1)
    out[np.isnan(out)] = -np.inf
    return out


def chunk_scores(q_post, k_packed, k_scales, cos, sin, n_stored, cs):
    """kvr_retrieval.py:291-315 — cosine against the mean of each full chunk of
    ``cs`` RoPE'd tokens; trailing partial chunk dropped (:297)."""
    n_kv = k_packed.shape[1]
    n_chunks = n_stored // cs
    if n_chunks < 1:
        return token_scores(q_post, k_packed, k_scales, cos, sin, n_stored)
    qa = q_group_mean(q_post, n_kv)
    kp = deq_k(k_packed, k_scales, n_stored)
    kr = apply_rotary(kp, cos[:n_stored, None, :], sin[:n_stored, None, :]).astype(F32)
    d = kr.shape[-1]
    means = kr[: n_chunks * cs].reshape(n_chunks, cs, n_kv, d).astype(np.float64).mean(1)
    out = np.stack([_cosine(qa[h], means[:, h]) for h in range(n_kv)], 1)
    out[np.isnan(out)] = -np.inf
    return out


def scores_interleaved(q_avg, k_packed, k_scales, cos_half, sin_half, n_stored):
    """kvr_cuda.cu:9-49 — interleaved-pair RoPE with (n, d/2) tables, dot / sqrt(d).
    Computed in float64; (n_stored, n_kv)."""
    n_kv, d = q_avg.shape
    p = k_packed[:n_stored].astype(np.int32)
    hi = ((p >> 4) - 8).astype(np.float64)
    lo = ((p & 0x0F) - 8).astype(np.float64)
    sc = k_scales.astype(np.float64)
    k_even = hi * sc[None, :, 0::2] / 8.0
    k_odd = lo * sc[None, :, 1::2] / 8.0
    c = cos_half[:n_stored, None, :].astype(np.float64)
    s = sin_half[:n_stored, None, :].astype(np.float64)
    k0r = k_even * c - k_odd * s
    k1r = k_even * s + k_odd * c
    q = q_avg.astype(np.float64)
    return ((k0r * q[None, :, 0::2]).sum(-1) + (k1r * q[None, :, 1::2]).sum(-1)) / np.sqrt(d)


# --------------------------------------------------------------------------
# selection (kvr_retrieval.py:370-392) with the stated tie-break
# --------------------------------------------------------------------------


def topk_rule(scores: np.ndarray, k: int) -> np.ndarray:
    """Column-wise top-k of (n, H) scores, ordered by (score desc, index asc).
    NaN counts as -inf and -0.0 equals +0.0.  This is the deterministic rule the
    kernels implement in place of torch.topk's unspecified tie order
    (kvr_retrieval.py:392)."""
    s = np.where(np.isnan(scores), -np.inf, scores.astype(np.float64))
    n, H = s.shape
    idx = np.arange(n)
    out = np.empty((k, H), np.int64)
    for h in range(H):
        order = np.lexsort((idx, -s[:, h]))
        out[:, h] = order[:k]
    return out


def near_tie_ok(scores, got_idx, want_idx, rel=1e-6) -> bool:
    """Selected sets may differ only among entries whose score lies within
    ``rel`` (relative) of the k-th selected score (the parity rule's near-tie
    clause)."""
    s = np.where(np.isnan(scores), -np.inf, scores.astype(np.float64))
    for h in range(s.shape[1]):
        a, b = set(got_idx[:, h].tolist()), set(want_idx[:, h].tolist())
        if a == b:
            continue
        kth = s[want_idx[-1, h], h]
        tol = rel * max(abs(kth), 1e-30)
        for i in a ^ b:
            if not (abs(s[i, h] - kth) <= tol or (np.isinf(kth) and s[i, h] == kth)):
                return False
    return True


def retrieve_token_branch(q_post, st: dict, cos, sin, top_k, ex_start=0, ex_end=0):
    """kvr_retrieval.py:317-330 (guards) + 389-412 (token branch) with attractors
    disabled.  ``st`` holds k_packed, vr_packed, n_stored and the calibration.
    Returns (ret_k fp32 post-RoPE, ret_v fp16, top_indices)."""
    nr = st["n_stored"]
    n_kv = st["k_packed"].shape[1]
    d = st["k_packed"].shape[2] * 2
    if nr == 0 or ex_start >= nr or (ex_start <= 0 and ex_end >= nr):
        z = np.zeros((0, n_kv, d), np.float16)
        return z, z, np.zeros((0, n_kv), np.int64)
    top_k = min(top_k, nr)
    sc = token_scores(q_post, st["k_packed"], st["k_scales"], cos, sin, nr)
    sc[ex_start:ex_end, :] = -np.inf
    top = topk_rule(sc, top_k)
    return gather_selected(st, top, cos, sin) + (top,)


def chunk_branch_indices(q_post, st, cos, sin, top_k, cs, ex_start=0, ex_end=0):
    """The intended chunk branch of kvr_retrieval.py:370-388 (the reference's own
    body raises UnboundLocalError: ``scores``/``cs`` are never bound), using
    compute_chunk_scores (:291-315) as the score source."""
    nr = st["n_stored"]
    sc = chunk_scores(q_post, st["k_packed"], st["k_scales"], cos, sin, nr, cs)
    n_chunks = sc.shape[0]
    ec_start = ex_start // cs
    ec_end = min((ex_end + cs - 1) // cs, n_chunks)
    if ec_start >= ec_end:
        ec_start = ec_end = 0
    if ec_start < n_chunks:
        sc[ec_start:ec_end, :] = -np.inf
    top_chunks = min(max(1, min(top_k, nr) // cs), n_chunks)
    cidx = topk_rule(sc, top_chunks)
    tok = cidx[:, None, :] * cs + np.arange(cs)[None, :, None]
    return tok.reshape(top_chunks * cs, -1), cidx, sc


def gather_selected(st, top, cos, sin):
    """kvr_retrieval.py:394-412 — V = W-predict(deq K_pre of all heads) + int2
    residual; K gathered per head and re-rotated at its own position."""
    n_kv = st["k_packed"].shape[1]
    d = st["k_packed"].shape[2] * 2
    kpre = unpack_int4(st["k_packed"][top]).astype(F32) * k_step(st["k_scales"])[None, None]  # (k, H, H, d)
    k = top.shape[0]
    ret_k = np.empty((k, n_kv, d), F32)
    ret_v = np.empty((k, n_kv, d), F32)
    vstep = vr_step(st["vr_scales"])  # (H, 1)
    for h in range(n_kv):
        tid = top[:, h]
        rows = kpre[:, h]  # (k, H, d): all heads of the selected tokens
        vb = predict_v(rows.reshape(k, -1), st["W"], st["K_mean"], st["V_mean"]).reshape(k, n_kv, d)[:, h]
        res = unpack_int2(st["vr_packed"][tid][:, h]).astype(F32) * vstep[h]
        ret_v[:, h] = vb + res
        ret_k[:, h] = apply_rotary(rows[:, h], cos[tid], sin[tid])
    return ret_k, ret_v.astype(np.float16)


def attractor_select(q_post, st, cos, sin, labels, centroids, top_a=48, per_basin=16, ex_start=0, ex_end=0):
    """kvr_retrieval.py:248-263 + 332-367 — the attractor branch given the
    basins (labels, centroids): cosine of the head-0 group-mean query with each
    centroid, the top_a basins, in each basin with more than per_basin tokens
    the per_basin best by head-0 cosine of RoPE(deq K) at the token's own
    position, the sorted union, minus [ex_start, ex_end) when that range is
    non-empty.  Ties by index ascending (torch leaves them unspecified).
    Returns (tokens ascending, basin scores, {basin: token scores})."""
    n_kv = st["k_packed"].shape[1]
    qa = q_group_mean(q_post, n_kv)[0]
    bs = _cosine(qa, centroids.astype(F32))
    bs = np.where(np.isnan(bs), -np.inf, bs)
    basins = topk_rule(bs[:, None], min(top_a, len(bs)))[:, 0]
    k0 = deq_k(st["k_packed"], st["k_scales"], len(labels))[:, 0]
    chosen, tok_scores = [], {}
    for b in basins:
        tidx = np.nonzero(labels == b)[0]
        if len(tidx) <= per_basin:
            chosen.append(tidx)
            continue
        kr = apply_rotary(k0[tidx], cos[tidx], sin[tidx]).astype(F32)
        sc = _cosine(qa, kr)
        tok_scores[int(b)] = (tidx, sc)
        chosen.append(tidx[topk_rule(sc[:, None], per_basin)[:, 0]])
    toks = np.unique(np.concatenate(chosen)) if chosen else np.zeros(0, np.int64)
    if ex_end > ex_start:
        toks = toks[(toks < ex_start) | (toks >= ex_end)]
    return toks, bs, tok_scores


# --------------------------------------------------------------------------
# attention (kvr_window.py:43-69, kvr_hook.py:274-282, kvr_triton.py:42-79)
# --------------------------------------------------------------------------


def softmax_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float | None = None):
    """Exact softmax(q.k^T/scale).v per Q head with GQA kvh = hi // g.
    q (n_q, d); k, v (n_tok, n_kv, d).  float64 result."""
    n_q, d = q.shape
    n_kv = k.shape[1]
    g = n_q // n_kv
    scale = scale or d ** 0.5
    q64, k64, v64 = (x.astype(np.float64) for x in (q, k, v))
    out = np.zeros((n_q, d))
    if k.shape[0] == 0:
        return out
    for hi in range(n_q):
        h = hi // g
        s = k64[:, h] @ q64[hi] / scale
        w = np.exp(s - s.max())
        out[hi] = (w / w.sum()) @ v64[:, h]
    return out


def window_ring_write(ring_k, ring_v, pos, k_new, v_new):
    """kvr_window.py:19-41 — slot = pos % cap; wrapped writes in fp16.
    Returns the new ``pos``; ``n`` is min(n + count, cap)."""
    cap = ring_k.shape[0]
    for i in range(k_new.shape[0]):
        slot = (pos + i) % cap
        ring_k[slot] = k_new[i].astype(np.float16)
        ring_v[slot] = v_new[i].astype(np.float16)
    return pos + k_new.shape[0]


def kmeans_lloyd(x, k, iters):
    """Specification of the device k-means that replaces the reference's host
    MiniBatchKMeans (modules/kvr_retrieval.py:234-246; not a restatement of
    it: sklearn's mini-batch algorithm is version-dependent).  x (n, d)
    float32.  centroid j starts at x[j*n//k]; each iteration assigns every
    point to argmin_j ||c_j||^2 - 2 x.c_j (lowest j on ties) and moves each
    non-empty cluster's centroid to the mean of its points; a final assignment
    gives the labels.  Returns (labels int64, centroids float32), float64
    arithmetic (the device accumulates in fp32: compare labels on separated
    data, centroids with a tolerance)."""
    x = np.asarray(x, np.float64)
    n = x.shape[0]
    c = x[(np.arange(k) * n) // k].copy()

    def assign(c):
        d = (c * c).sum(1)[None, :] - 2.0 * x @ c.T
        return d.argmin(1)

    for _ in range(iters):
        lab = assign(c)
        for j in range(k):
            m = lab == j
            if m.any():
                c[j] = x[m].mean(0)
    return assign(c).astype(np.int64), c.astype(np.float32)

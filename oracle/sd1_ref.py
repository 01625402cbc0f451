"""CPU oracle for the ``sd1`` 1-bit codec — TEST INFRASTRUCTURE ONLY.

PARITY UNPINNED VS REFERENCE: the reference (Misaka477/RINA-1bit-KV) contains no
1-bit, Hadamard/DCT or sigma-delta code at all (its codec is int4 K + int2
V-residual, modules/kvr_retrieval.py:2-4).  This file IS the written
specification of the sd1 codec that the CUDA kernels implement, stated as
numpy float32 code whose every operation order is fixed so that the kernels can
be checked bit-exactly against it.  It is pinned against itself by known-answer
tests (tests/test_sd1_oracle.py: orthonormality vs a float64 matrix, round
trips, hand-worked sigma-delta cases) and quality is judged against exact
attention.

The scoring side mirrors the reference's design points:
* the query used for selection is the GQA-group mean of the post-RoPE query
  (modules/kvr_retrieval.py:270, 296);
* tokens are grouped into fixed tiles and only full tiles are scored
  (the chunk scorer, modules/kvr_retrieval.py:291-315, drops the partial tail);
* selection is a per-KV-head top-k with an exclusion range
  (modules/kvr_retrieval.py:370-392).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import
this module.

Spec summary (d = 128, tile t in {32, 64, 128}):
1. RoPE (optional): k_post = (k*cos) + (rotate_half(k)*sin), three roundings,
   cos/sin rows from HF-style (max_pos, d) tables at the token's position.
2. Transform along head_dim, orthonormal: Walsh-Hadamard (Sylvester order,
   butterfly stages of stride 1,2,...,64, then x*fp32(1/sqrt(d))) or DCT-II
   (Lee's recursive factorisation, fixed below, then x*fp32(sqrt(1/d)) for
   k=0 and x*fp32(sqrt(2/d)) otherwise).
3. Per (tile, channel) scale s = fp16_rn(min((sum_j |x_j|) * (1/t), 65504)),
   sum sequential in j.
4. First-order sigma-delta along the tile's tokens, per channel, e0 = 0:
   u = x_j + e; bit = (u >= 0); y = bit ? s : -s; e = u - y.
5. Bits token-major: token j owns 4 uint32 words; channel c is bit c%32 of
   word c//32.  Scales fp16 per (tile, channel).  Same for V.
6. Selection score of a tile for KV head h: q' = T(q_avg), w_c = q'_c * s_c,
   M = max|w_c|, wq_c = rint(w_c * (127/M)) (0 if M == 0), per token
   S_j = 2*sum_c wq_c*bit_jc - sum_c wq_c (integer, computed from bit planes
   with popcount), tile score = float(max_j S_j) * (M/127).
7. Top-k tiles per head by (score desc, tile index asc); NaN = -inf.
8. Attention: exact softmax over the fp16 window, the fp16 pending tail and
   the decoded selected tiles, k_hat_j = T^T(s (2 bit_j - 1)), same for V.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
F16 = np.float16
D = 128

# ----------------------------------------------------------------------------
# transforms
# ----------------------------------------------------------------------------


def hadamard_fwd(x: np.ndarray) -> np.ndarray:
    """Orthonormal WHT along the last axis, butterfly strides 1, 2, ..., d/2."""
    y = np.array(x, dtype=F32, copy=True)
    d = y.shape[-1]
    h = 1
    while h < d:
        y = y.reshape(*y.shape[:-1], d // (2 * h), 2, h)
        a = y[..., 0, :].copy()
        b = y[..., 1, :].copy()
        y[..., 0, :] = a + b
        y[..., 1, :] = a - b
        y = y.reshape(*y.shape[:-3], d)
        h *= 2
    return y * F32(1.0 / np.sqrt(d))


def lee_factors(d: int = D) -> dict:
    """f[M][j] = fp32(1 / (2 cos(pi (2j+1) / (2M)))) for block sizes M = d, d/2, ..., 2."""
    out = {}
    M = d
    while M >= 2:
        j = np.arange(M // 2, dtype=np.float64)
        out[M] = (1.0 / (2.0 * np.cos(np.pi * (2.0 * j + 1.0) / (2.0 * M)))).astype(F32)
        M //= 2
    return out


def dct_consts(d: int = D):
    return F32(np.sqrt(1.0 / d)), F32(np.sqrt(2.0 / d))


def dct_fwd(x: np.ndarray) -> np.ndarray:
    """Orthonormal DCT-II along the last axis by Lee's algorithm.

    Split levels M = d..2 (blocks of size M at offsets multiple of M):
        a_j = x_j + x_{M-1-j};  b_j = (x_j - x_{M-1-j}) * f[M][j];  block <- [a, b]
    Merge levels M = 2..d:
        out_{2k} = A_k;  out_{2k+1} = B_k + B_{k+1} (k < M/2-1);  out_{M-1} = B_{M/2-1}
    then scale element 0 by sqrt(1/d), the rest by sqrt(2/d)."""
    y = np.array(x, dtype=F32, copy=True)
    lead = y.shape[:-1]
    d = y.shape[-1]
    f = lee_factors(d)
    M = d
    while M >= 2:
        blk = y.reshape(*lead, d // M, M)
        lo = blk[..., : M // 2]
        hi_rev = blk[..., ::-1][..., : M // 2]
        a = lo + hi_rev
        b = (lo - hi_rev) * f[M]
        y = np.concatenate([a, b], -1).reshape(*lead, d)
        M //= 2
    M = 2
    while M <= d:
        blk = y.reshape(*lead, d // M, M)
        A = blk[..., : M // 2]
        B = blk[..., M // 2:]
        out = np.empty_like(blk)
        out[..., 0::2] = A
        odd = B.copy()
        odd[..., :-1] = B[..., :-1] + B[..., 1:]
        out[..., 1::2] = odd
        y = out.reshape(*lead, d)
        M *= 2
    c0, c1 = dct_consts(d)
    y[..., 0] = y[..., 0] * c0
    y[..., 1:] = y[..., 1:] * c1
    return y


def dct_inv(y: np.ndarray) -> np.ndarray:
    """Orthonormal DCT-III (inverse of dct_fwd) by the transposed Lee graph."""
    x = np.array(y, dtype=F32, copy=True)
    lead = x.shape[:-1]
    d = x.shape[-1]
    f = lee_factors(d)
    c0, c1 = dct_consts(d)
    x[..., 0] = x[..., 0] * c0
    x[..., 1:] = x[..., 1:] * c1
    M = d
    while M >= 2:
        blk = x.reshape(*lead, d // M, M)
        A = blk[..., 0::2]
        odd = blk[..., 1::2]
        B = odd.copy()
        B[..., 1:] = odd[..., 1:] + odd[..., :-1]
        x = np.concatenate([A, B], -1).reshape(*lead, d)
        M //= 2
    M = 2
    while M <= d:
        blk = x.reshape(*lead, d // M, M)
        a = blk[..., : M // 2]
        fb = blk[..., M // 2:] * f[M]
        out = np.empty_like(blk)
        out[..., : M // 2] = a + fb
        out[..., M // 2:] = (a - fb)[..., ::-1]
        x = out.reshape(*lead, d)
        M *= 2
    return x


def transform(x, kind: str, inverse: bool = False):
    if kind == "hadamard":
        return hadamard_fwd(x)  # symmetric orthonormal: its own inverse
    if kind == "dct":
        return dct_inv(x) if inverse else dct_fwd(x)
    raise ValueError(kind)


def transform_matrix(kind: str, d: int = D) -> np.ndarray:
    """float64 orthonormal matrix T with y = T x (for checking only)."""
    if kind == "hadamard":
        H = np.array([[1.0]])
        while H.shape[0] < d:
            H = np.block([[H, H], [H, -H]])
        return H / np.sqrt(d)
    n = np.arange(d)
    T = np.cos(np.pi * (2 * n[None, :] + 1) * n[:, None] / (2 * d)) * np.sqrt(2.0 / d)
    T[0] *= np.sqrt(0.5)
    return T


# ----------------------------------------------------------------------------
# encoder
# ----------------------------------------------------------------------------


def rope_apply_f32(k, cos, sin):
    """(k*cos) + (rotate_half(k)*sin) in float32 with three roundings."""
    d2 = k.shape[-1] // 2
    rh = np.concatenate([-k[..., d2:], k[..., :d2]], -1)
    return (k * cos).astype(F32) + (rh * sin).astype(F32)


def sigma_delta_tile(x: np.ndarray):
    """x: (..., t, d) float32 transformed values of one tile.
    Returns (bits bool (..., t, d), scale fp16 (..., d))."""
    t = x.shape[-2]
    acc = np.zeros(x.shape[:-2] + x.shape[-1:], F32)
    for j in range(t):
        acc = acc + np.abs(x[..., j, :])
    mean = acc * F32(1.0 / t)
    s16 = np.minimum(mean, F32(65504.0)).astype(F16)
    s = s16.astype(F32)
    e = np.zeros_like(acc)
    bits = np.zeros(x.shape, bool)
    for j in range(t):
        u = x[..., j, :] + e
        b = u >= 0
        y = np.where(b, s, -s)
        e = u - y
        bits[..., j, :] = b
    return bits, s16


def pack_bits(bits: np.ndarray) -> np.ndarray:
    """bool (..., d) -> uint32 (..., d/32); channel c -> bit c%32 of word c//32."""
    d = bits.shape[-1]
    b = bits.reshape(*bits.shape[:-1], d // 32, 32).astype(np.uint64)
    w = (b << np.arange(32, dtype=np.uint64)).sum(-1)
    return w.astype(np.uint32)


def unpack_bits(words: np.ndarray) -> np.ndarray:
    w = words.astype(np.uint64)[..., None]
    b = (w >> np.arange(32, dtype=np.uint64)) & 1
    return b.reshape(*words.shape[:-1], words.shape[-1] * 32).astype(bool)


def encode(k, v, tile: int, kind: str, cos=None, sin=None, pos0: int = 0):
    """Encode full tiles.  k, v: (n, d) float32 (one head; n a multiple of tile).
    If cos/sin are given, k is pre-RoPE and is rotated at positions pos0+i.
    Returns dict(kbits (nt, t, d/32) u32, kscale (nt, d) f16, vbits, vscale)."""
    n, d = k.shape
    assert n % tile == 0
    k = k.astype(F32)
    if cos is not None:
        k = rope_apply_f32(k, cos[pos0:pos0 + n], sin[pos0:pos0 + n])
    kt = transform(k, kind).reshape(n // tile, tile, d)
    vt = transform(v.astype(F32), kind).reshape(n // tile, tile, d)
    kb, ks = sigma_delta_tile(kt)
    vb, vs = sigma_delta_tile(vt)
    return {"kbits": pack_bits(kb), "kscale": ks, "vbits": pack_bits(vb), "vscale": vs}


def decode_tiles(bits, scale, kind):
    """Reconstruct (nt, t, d) float64 vectors: T^T(s * (2 bit - 1))."""
    b = unpack_bits(bits).astype(np.float64) * 2.0 - 1.0
    y = b * scale.astype(np.float64)[:, None, :]
    T = transform_matrix(kind, y.shape[-1])
    return y @ T  # (row-vector) y T == (T^T y^T)^T


# ----------------------------------------------------------------------------
# selection
# ----------------------------------------------------------------------------


def q_group_mean_f32(q: np.ndarray, n_kv: int) -> np.ndarray:
    """Sequential fp32 sum over the g heads of each group, then / g."""
    n_q, d = q.shape
    g = n_q // n_kv
    qg = q.astype(F32).reshape(n_kv, g, d)
    acc = qg[:, 0].copy()
    for i in range(1, g):
        acc = acc + qg[:, i]
    return acc / F32(g)


def tile_scores(qprime: np.ndarray, kbits: np.ndarray, kscale: np.ndarray) -> np.ndarray:
    """qprime (d,) fp32 transformed group-mean query; kbits (nt, t, d/32); kscale (nt, d).
    Returns (nt,) float32 tile scores per the spec (step 6)."""
    w = (qprime[None, :] * kscale.astype(F32)).astype(F32)  # (nt, d)
    M = np.abs(w).max(-1)
    with np.errstate(divide="ignore", invalid="ignore"):
        inv = np.where(M > 0, F32(127.0) / M, F32(0.0)).astype(F32)
    wq = np.rint((w * inv[:, None]).astype(F32)).astype(np.int64)
    bits = unpack_bits(kbits).astype(np.int64)  # (nt, t, d)
    P = (bits * wq[:, None, :]).sum(-1)
    S = 2 * P - wq.sum(-1)[:, None]
    Smax = S.max(-1).astype(F32)
    delta = (M / F32(127.0)).astype(F32)
    return (Smax * delta).astype(F32)


def select_tiles(scores: np.ndarray, k: int, ex_t0: int = 0, ex_t1: int = 0) -> np.ndarray:
    """scores (nt,) -> indices of the top-min(k, nt) tiles, (score desc, index asc);
    tiles in [ex_t0, ex_t1) are scored -inf."""
    s = np.where(np.isnan(scores), -np.inf, scores.astype(np.float64))
    s[ex_t0:ex_t1] = -np.inf
    s = np.where(s == 0, 0.0, s)
    order = np.lexsort((np.arange(len(s)), -s))
    return order[: min(k, len(s))]


# ----------------------------------------------------------------------------
# attention
# ----------------------------------------------------------------------------


def decode_attention(q, win_k, win_v, tiles_k, tiles_v, scale=None):
    """q (g, d) fp32 (the Q heads of one KV head); win_k/v (n_w, d) (window plus
    pending tail, exact); tiles_k/v (n_r, d) decoded selected tokens.
    float64 exact softmax result (g, d)."""
    k = np.concatenate([win_k.astype(np.float64), tiles_k.astype(np.float64)], 0)
    v = np.concatenate([win_v.astype(np.float64), tiles_v.astype(np.float64)], 0)
    d = q.shape[-1]
    scale = scale or np.sqrt(d)
    s = q.astype(np.float64) @ k.T / scale
    s = s - s.max(-1, keepdims=True)
    w = np.exp(s)
    return (w / w.sum(-1, keepdims=True)) @ v


# ----------------------------------------------------------------------------
# prefill-sized tile scoring (tensor cores)
# ----------------------------------------------------------------------------


def prefill_qprime_f16(q: np.ndarray, n_kv: int, kind: str) -> np.ndarray:
    """q (Nq, n_q, d) post-RoPE queries of a prefill block -> (Nq, n_kv, d) fp16:
    the GQA-group mean (q_group_mean_f32 order) transformed by T, rounded to fp16."""
    out = np.stack([transform(q_group_mean_f32(qi, n_kv), kind) for qi in q.astype(F32)])
    return out.astype(F16)


def prefill_tile_scores(qp16: np.ndarray, kbits: np.ndarray, kscale: np.ndarray) -> np.ndarray:
    """qp16 (Nq, d) fp16 transformed queries of one KV head; kbits (nt, t, d/32),
    kscale (nt, d).  Score of tile i for query r = max over the tile's tokens j of
    the exact dot q'_r . k_hat_j, k_hat_j = s (2 bit_j - 1) (transformed domain,
    exact products; the kernels accumulate in fp32).  float64 (Nq, nt)."""
    b = unpack_bits(kbits).astype(np.float64) * 2.0 - 1.0          # (nt, t, d)
    khat = b * kscale.astype(np.float64)[:, None, :]
    s = np.einsum("rd,ntd->rnt", qp16.astype(np.float64), khat)
    return s.max(-1)

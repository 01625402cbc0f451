"""CPU timing port of the reference decode path — TEST/BENCH INFRASTRUCTURE ONLY.

Restates, in torch-CPU operations (the reference's own library and numerics),
one layer of the reference's decode step so bench.py can time the reference
algorithm on the host cores:

* RetrievalIndex.compute_all_scores (modules/kvr_retrieval.py:265-289): per KV
  head dequantise int4 K, rotate_half RoPE via table gathers, cosine with the
  GQA-group mean query;
* exclusion + torch.topk (:389-392);
* V reconstruction of the unique selected tokens through W plus the int2
  residual, and per-head K gather + RoPE (:394-412);
* the hook's softmax over cat(window, retrieved) (modules/kvr_hook.py:274-282).

Only bench.py's CPU-baseline / reference arm and tests may import this module.
Its output agrees with oracle/int4w_ref.py (checked in tests/test_cpu_port.py).
"""
import math

import torch


def _rotate_half(x):
    d2 = x.shape[-1] // 2
    return torch.cat([-x[..., d2:], x[..., :d2]], dim=-1)


def _apply_rotary(x, cos, sin):
    return x * cos[:x.shape[0]] + _rotate_half(x) * sin[:x.shape[0]]


def _unpack_int4(p):
    hi = ((p >> 4).to(torch.int8) - 8)
    lo = ((p & 0x0F).to(torch.int8) - 8)
    return torch.stack([hi, lo], dim=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)


def _unpack_int2(p):
    v = [((p >> s) & 0x03).to(torch.int8) - 2 for s in (6, 4, 2, 0)]
    return torch.stack(v, dim=-1).reshape(*p.shape[:-1], p.shape[-1] * 4)


def make_case(seed, n_stored, window, n_kv=8, n_q=32, d=128, theta=500000.0, n_queries=64):
    """Synthetic config-0 K/V, calibrated and packed like the reference
    (kvr_retrieval.py:95-122, 187-207)."""
    g = torch.Generator().manual_seed(seed)
    n = n_stored + window
    scale = torch.exp(torch.randn(n_kv, d, generator=g))
    for h in range(n_kv):
        scale[h, torch.randperm(d, generator=g)[:4]] *= 20
    k = torch.randn(n, n_kv, d, generator=g) * scale
    v = torch.randn(n, n_kv, d, generator=g)
    inv = 1.0 / (theta ** (torch.arange(0, d, 2).float() / d))
    fr = torch.arange(n).float()[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    cos, sin = emb.cos(), emb.sin()
    D = n_kv * d
    ks = k[:n_stored]
    k_scales = ks.abs().max(0).values.clamp(min=1e-8)
    step = 2 * k_scales / 16
    kq = torch.round(ks / step).clamp(-8, 7).to(torch.int8)
    u = kq.to(torch.uint8) + 8
    k_packed = (u[..., 0::2] << 4) | u[..., 1::2]
    # calibration on a bounded sample (the pinv is a one-off, not the timed path)
    m = min(n_stored, 8192)
    k2, v2 = ks[:m].reshape(m, D), v[:m].reshape(m, D)
    half = m // 2
    K_mean, V_mean = k2[:half].mean(0, keepdim=True), v2[:half].mean(0, keepdim=True)
    kc, vc = k2[:half] - K_mean, v2[:half] - V_mean
    W = (kc.T @ vc).T @ torch.linalg.pinv(kc.T @ kc)
    vpred = (ks.reshape(n_stored, D) - K_mean) @ W.T + V_mean
    vres = v[:n_stored] - vpred.view(n_stored, n_kv, d)
    vr_scales = vres.abs().amax(dim=(0, 2)).unsqueeze(1).clamp(min=1e-8)
    vrq = torch.round(vres / (2 * vr_scales / 4)).clamp(-2, 1).to(torch.int8)
    u2 = vrq.to(torch.uint8) + 2
    vr_packed = (u2[..., 0::4] << 6) | (u2[..., 1::4] << 4) | (u2[..., 2::4] << 2) | u2[..., 3::4]
    kpost = _apply_rotary(k[n_stored:].reshape(-1, d), cos[n_stored:].repeat_interleave(n_kv, 0),
                          sin[n_stored:].repeat_interleave(n_kv, 0)).view(window, n_kv, d)
    return {"k_packed": k_packed, "k_scales": k_scales, "vr_packed": vr_packed, "vr_scales": vr_scales, "W": W,
            "K_mean": K_mean, "V_mean": V_mean, "cos": cos, "sin": sin, "n_stored": n_stored,
            "win_k": kpost.half(), "win_v": v[n_stored:].half(), "n_kv": n_kv, "n_q": n_q, "d": d,
            "q": torch.randn(n_queries, n_q, d, generator=g)}


@torch.no_grad()
def decode_layer(c, top_k, q_index=0):
    """One layer of the reference decode step; returns (n_q, d) fp32."""
    n_kv, n_q, d, nr = c["n_kv"], c["n_q"], c["d"], c["n_stored"]
    q = c["q"][q_index % c["q"].shape[0]]
    g = n_q // n_kv
    step = 2 * c["k_scales"] / 16
    q_avg = q.view(n_kv, g, d).mean(dim=1)
    aidx = torch.arange(nr)
    scores = torch.empty(nr, n_kv)
    for h in range(n_kv):                                   # kvr_retrieval.py:281-286
        kp = _unpack_int4(c["k_packed"][:nr, h, :]).float() * step[h]
        kp2 = _apply_rotary(kp, c["cos"][aidx], c["sin"][aidx])
        qn = q_avg[h] / (q_avg[h].norm() + 1e-8)
        kn = kp2 / (kp2.norm(dim=-1, keepdim=True) + 1e-8)
        scores[:, h] = qn @ kn.T
    top = torch.topk(scores, min(top_k, nr), dim=0)[1]      # :392
    all_tidx = top.T.reshape(-1)                           # :395-402
    uniq, inverse = all_tidx.unique(sorted=False, return_inverse=True)
    kpre_u = _unpack_int4(c["k_packed"][uniq]).float() * step.unsqueeze(0)
    vbase = ((kpre_u.reshape(-1, n_kv * d) - c["K_mean"]) @ c["W"].T + c["V_mean"]).reshape(-1, n_kv, d)
    vdq = _unpack_int2(c["vr_packed"][uniq]).float() * (2 * c["vr_scales"] / 4).unsqueeze(0)
    v_all = (vbase + vdq)[inverse].reshape(n_kv, top.shape[0], n_kv, d)
    ks, vs = [], []
    for h in range(n_kv):                                   # :404-412
        tidx = top[:, h]
        kt = _unpack_int4(c["k_packed"][tidx, h]).float() * step[h]
        ks.append(_apply_rotary(kt, c["cos"][tidx], c["sin"][tidx]))
        vs.append(v_all[h, :, h, :])
    rk = torch.stack(ks, 1)
    rv = torch.stack(vs, 1).half()
    k_cat = torch.cat([c["win_k"].float(), rk], 0)          # kvr_hook.py:274-282
    v_cat = torch.cat([c["win_v"].float(), rv.float()], 0)
    qg = q.view(n_kv, g, d)
    sc = torch.einsum("hgd, thd -> h g t", qg, k_cat)
    w = torch.softmax(sc / math.sqrt(d), dim=-1)
    return torch.einsum("h g t, t h d -> h g d", w, v_cat).reshape(n_q, d)


@torch.no_grad()
def encode_layer_timed(seed, n, n_kv=8, d=128, reps=3):
    """The reference's prefill encode of one layer on the host cores:
    RetrievalIndex.calibrate (absmax scales, W fit with pinv on the first
    half, residual scales; modules/kvr_retrieval.py:95-122) followed by
    batch_append (quantise + pack K, V-predict GEMM, int2 residual;
    :187-207), timed separately; returns medians over `reps` runs."""
    import time

    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(torch.randn(n_kv, d, generator=g))
    k = torch.randn(n, n_kv, d, generator=g) * scale
    v = torch.randn(n, n_kv, d, generator=g)
    D_ = n_kv * d
    cal, app = [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        k_scales = k.abs().max(0).values.clamp(min=1e-8)              # :99
        k2, v2 = k.reshape(n, D_), v.reshape(n, D_)
        half = n // 2
        K_mean, V_mean = k2[:half].mean(0, keepdim=True), v2[:half].mean(0, keepdim=True)
        kc, vc = k2[:half] - K_mean, v2[:half] - V_mean
        W = (kc.T @ vc).T @ torch.linalg.pinv(kc.T @ kc)               # :105-112
        vres = v2 - ((k2 - K_mean) @ W.T + V_mean)
        vr_scales = vres.view(-1, n_kv, d).abs().amax(dim=(0, 2)).unsqueeze(1).clamp(min=1e-8)  # :116
        t1 = time.perf_counter()
        step = 2 * k_scales / 16                                       # :190-193
        kq = torch.round(k / step).clamp(-8, 7).to(torch.int8)
        u = kq.to(torch.uint8) + 8
        k_packed = torch.zeros(n + max(1024, n // 2), n_kv, d // 2, dtype=torch.uint8)
        k_packed[:n] = (u[..., 0::2] << 4) | u[..., 1::2]
        v_pred = ((k2 - K_mean) @ W.T + V_mean).view(n, n_kv, d)       # :196-198
        vrq = torch.round((v - v_pred) / (2 * vr_scales / 4)).clamp(-2, 1).to(torch.int8)
        u2 = vrq.to(torch.uint8) + 2
        vr_packed = torch.zeros(n + max(1024, n // 2), n_kv, d // 4, dtype=torch.uint8)
        vr_packed[:n] = (u2[..., 0::4] << 6) | (u2[..., 1::4] << 4) | (u2[..., 2::4] << 2) | u2[..., 3::4]
        t2 = time.perf_counter()
        cal.append(t1 - t0)
        app.append(t2 - t1)
    cal.sort()
    app.sort()
    tot = sorted(c + a for c, a in zip(cal, app))
    return {"calibrate_s": cal[len(cal) // 2], "append_s": app[len(app) // 2], "median_s": tot[len(tot) // 2]}

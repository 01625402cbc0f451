"""Generate golden fixtures by running the REFERENCE implementation on CPU.

Run in a container where the reference checkout is importable:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference package ``modules`` (``RetrievalIndex``,
``WindowBuffer``), drives it on seeded synthetic inputs with the config-0
distribution (per-channel log-normal scales, 4 outlier channels x20, RoPE
theta 5e5 tables, V ~ N(0,1)) at a size the CPU finishes instantly, and writes
``int4w_golden.npz`` next to this script.  Nothing else reads the reference:
the tests and the GPU box only see the .npz.

Reference shims applied here (harness side, never in the reference):
* attractors disabled (``labels = attractors = None``), as the reference's own
  scripts/evaluation/_test_int4.py:33-36 does;
* ``chunk_size=0`` so ``retrieve_topk`` takes its token branch (the chunk
  branch at kvr_retrieval.py:370-388 raises UnboundLocalError).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def make_inputs(seed, n, n_kv, d, n_q, max_pos, theta=500000.0):
    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(torch.randn(n_kv, d, generator=g))
    for h in range(n_kv):
        ch = torch.randperm(d, generator=g)[:4]
        scale[h, ch] *= 20.0
    k_pre = (torch.randn(n, n_kv, d, generator=g) * scale).half().float()
    v = torch.randn(n, n_kv, d, generator=g).half().float()
    q = torch.randn(n_q, d, generator=g).half().float()
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    freqs = torch.arange(max_pos).float()[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], -1)
    return k_pre, v, q, emb.cos(), emb.sin()


def main(ref_root):
    sys.path.insert(0, ref_root)
    from modules.kvr_retrieval import RetrievalIndex, _apply_rotary
    from modules.kvr_window import WindowBuffer

    torch.manual_seed(0)
    n, n_kv, d, n_q, top_k, cs = 384, 2, 128, 8, 64, 32
    n_app = 5
    max_pos = n + n_app
    k_pre, v, q_pre, cos, sin = make_inputs(1234, n + n_app, n_kv, d, n_q, max_pos)
    out = {"k_pre": k_pre.half().numpy(), "v": v.half().numpy(), "q_pre": q_pre.half().numpy(),
           "cos": cos.numpy(), "sin": sin.numpy(), "n": n, "top_k": top_k, "cs": cs}

    # ---- encoder: calibrate + batch_append + append (kvr_retrieval.py:95-207)
    ri = RetrievalIndex(n_kv, d, top_k=top_k, device="cpu", chunk_size=0)
    ri.set_rotary_tables(cos, sin)
    ri.calibrate(k_pre[:n], v[:n])
    ri.batch_append(k_pre[:n], v[:n])
    out.update(k_scales=ri.k_scales.numpy(), W=ri.W.numpy(), K_mean=ri.K_mean.numpy(),
               V_mean=ri.V_mean.numpy(), vr_scales=ri.vr_scales.numpy(),
               k_packed_batch=ri.k_packed.numpy().copy(), vr_packed_batch=ri.vr_packed.numpy().copy())
    for i in range(n_app):
        ri.append(k_pre[n + i], v[n + i])
    out.update(k_packed=ri.k_packed.numpy(), vr_packed=ri.vr_packed.numpy(), n_stored=ri.n_stored)
    # calibrate without V (kvr_retrieval.py:117-121)
    ri0 = RetrievalIndex(n_kv, d, device="cpu", chunk_size=0)
    ri0.calibrate(k_pre[:8])
    out.update(noV_vr_scales=ri0.vr_scales.numpy(), noV_W_is_eye=bool(torch.equal(ri0.W, torch.eye(n_kv * d))))

    # ---- post-RoPE query at the next position
    # (the query is used as given: the scorers only need a post-RoPE q)
    q_post = q_pre.clone()
    out["q_post"] = q_post.numpy()

    # ---- scorers (kvr_retrieval.py:265-315)
    out["scores_all"] = ri.compute_all_scores(q_post).numpy()
    ri.chunk_size = cs
    out["scores_chunk"] = ri.compute_chunk_scores(q_post).numpy()
    ri.chunk_size = 0

    # ---- retrieve_topk, token branch, with and without an exclusion range
    ri.labels = ri.attractors = None
    rk, rv = ri.retrieve_topk(q_post, n_q=n_q)
    out.update(ret_k=rk.numpy(), ret_v=rv.numpy())
    rk2, rv2 = ri.retrieve_topk(q_post, n_q=n_q, exclude_start=200, exclude_end=389)
    out.update(ret_k_ex=rk2.numpy(), ret_v_ex=rv2.numpy())
    e1 = ri.retrieve_topk(q_post, n_q=n_q, exclude_start=0, exclude_end=10**6)
    out["empty_when_all_excluded"] = bool(e1[0].shape[0] == 0)

    # ---- window ring (kvr_window.py) and the hook's concatenated softmax (kvr_hook.py:274-282)
    wb = WindowBuffer(n_kv, d, window_size=64, device="cpu")
    k_post = _apply_rotary(k_pre.reshape(-1, d), cos[:n + n_app].repeat_interleave(n_kv, 0),
                           sin[:n + n_app].repeat_interleave(n_kv, 0)).view(n + n_app, n_kv, d)
    wb.batch_append(k_post[:100], v[:100])
    for i in range(100, 103):
        wb.append(k_post[i], v[i])
    out.update(win_k=wb.k.numpy(), win_v=wb.v.numpy(), win_pos=wb.pos, win_n=wb.n,
               win_attn=wb.attention(q_post, n_q=n_q).numpy())
    k_cat = torch.cat([wb.k[:wb.n].float(), rk], 0)
    v_cat = torch.cat([wb.v[:wb.n].float(), rv.float()], 0)
    qg = q_post.float().view(n_kv, n_q // n_kv, d)
    sc = torch.einsum("hgd, thd -> h g t", qg, k_cat)
    w = torch.softmax(sc / d ** 0.5, dim=-1)
    out["hook_attn"] = torch.einsum("h g t, t h d -> h g d", w, v_cat).reshape(n_q, d).numpy()

    path = os.path.join(HERE, "int4w_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path to the reference checkout>")
    main(sys.argv[1])

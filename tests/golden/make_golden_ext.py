"""Generate the configs[0] and generator-level golden fixtures by running the
REFERENCE implementation on CPU.

    python tests/golden/make_golden_ext.py /path/to/reference

Writes next to this script:
* config0_golden.npz — BASELINE configs[0] (tests/golden/inputs.py
  config0_case): the prefill stores of modules/kvr_hook.py:85-134 (window =
  last 256 tokens; calibrate on the whole prompt; batch_append of the 3840
  evicted tokens), then for each of the 16 queries the token-branch top-512
  indices (compute_all_scores + torch.topk, kvr_retrieval.py:265-289, 389-392)
  and the hook's softmax over cat(window, retrieve_topk)
  (kvr_hook.py:250-282).  Stores the reference's outputs only: k_scales, the
  sha256 of the packed K codes, the packed int2 residual codes, the indices
  and the attention outputs; the inputs are regenerated from the seed.
* generator_golden.npz — KVRGenerator (modules/kvr_generator.py:41-161) on
  the tiny fp16 Llama of inputs.tiny_llama: prefill of 320 tokens, window 96,
  top_k 16, then 12 steps fed with fixed token ids (the window is full from
  the first step, so every step evicts into the index); the lm_head logits of
  every step.

Shims (harness side only, never in the reference), as in the survey's probe:
* transformers 5 has no ``self_attn.rotary_emb``: the model's rotary module is
  attached to every attention module before KVRHook is built;
* ``run_fused_attn`` is Triton (GPU only): modules.kvr_generator's binding is
  replaced by the same exact softmax in torch, computed in fp32 and returned in
  the input dtype;
* attractors stay off (the tiny store has fewer than 256 tokens; configs[0]
  sets labels = attractors = None as scripts/evaluation/_test_int4.py:33-36).
"""
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs  # noqa: E402


def config0(ref_root):
    from modules.kvr_retrieval import RetrievalIndex
    from modules.kvr_window import WindowBuffer

    c = inputs.config0_case()
    n, n_kv, d, n_q, win, top_k, n_ret = c["n"], c["n_kv"], c["d"], c["n_q"], c["window"], c["top_k"], c["n_ret"]
    wb = WindowBuffer(n_kv, d, window_size=win, device="cpu")
    wb.batch_append(c["k_post"], c["v"])
    ri = RetrievalIndex(n_kv, d, top_k=top_k, device="cpu", chunk_size=0)
    ri.set_rotary_tables(c["cos"], c["sin"])
    ri.calibrate(c["k_pre"], c["v"])
    ri.batch_append(c["k_pre"][:n_ret], c["v"][:n_ret])
    ri.labels = ri.attractors = None
    out = {"k_scales": ri.k_scales.numpy(),
           "k_packed_sha256": np.frombuffer(hashlib.sha256(ri.k_packed[:n_ret].numpy().tobytes()).digest(), np.uint8),
           "vr_packed": ri.vr_packed[:n_ret].numpy(), "win_pos": wb.pos, "win_n": wb.n,
           "planted_pos": np.array(c["planted_pos"])}
    tops, outs = [], []
    ctx = n
    ex0, ex1 = max(0, ctx - wb.n), min(ri.n_stored, ctx)
    if ex0 >= ex1:
        ex0 = ex1 = 0
    for qi in range(c["queries"].shape[0]):
        q = c["queries"][qi]
        sc = ri.compute_all_scores(q)
        sc[ex0:ex1] = float("-inf")
        tops.append(torch.topk(sc, top_k, dim=0)[1].numpy().astype(np.int16))
        rk, rv = ri.retrieve_topk(q, n_q=n_q, exclude_start=ex0, exclude_end=ex1)
        k_cat = torch.cat([wb.k[:wb.n].float(), rk], 0)
        v_cat = torch.cat([wb.v[:wb.n].float(), rv.float()], 0)
        qg = q.float().view(n_kv, n_q // n_kv, d)
        w = torch.softmax(torch.einsum("hgd, thd -> h g t", qg, k_cat) / d ** 0.5, dim=-1)
        outs.append(torch.einsum("h g t, t h d -> h g d", w, v_cat).reshape(n_q, d).numpy())
    out.update(top=np.stack(tops), attn=np.stack(outs), ex=np.array([ex0, ex1]))
    path = os.path.join(HERE, "config0_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


def generator(ref_root):
    import modules.kvr_generator as G
    from modules.kvr_generator import KVRGenerator

    def fused_attn_cpu(q, k, v):
        n_q, d = q.shape
        n_kv = k.shape[1]
        qg = q.float().view(n_kv, n_q // n_kv, d)
        w = torch.softmax(torch.einsum("hgd, thd -> h g t", qg, k.float()) / d ** 0.5, dim=-1)
        return torch.einsum("h g t, t h d -> h g d", w, v.float()).reshape(n_q, d).to(q.dtype)

    G.run_fused_attn = fused_attn_cpu
    model, prompt, steps = inputs.tiny_llama()
    for layer in model.model.layers:
        layer.self_attn.rotary_emb = model.model.rotary_emb
    gen = KVRGenerator(model, window_size=inputs.TINY["window"], top_k=inputs.TINY["top_k"], device="cpu")
    logits = []
    h = model.lm_head.register_forward_hook(lambda m, a, o: logits.append(o.detach().float().reshape(-1).clone()))
    gen.prefill(prompt)
    logits.clear()
    n_stored = [gen.kvr.retrievals[0].n_stored]
    for i in range(inputs.TINY["n_steps"]):
        tok = int(prompt[0, -1]) if i == 0 else int(steps[i])
        gen.step(token_id=tok)
        n_stored.append(gen.kvr.retrievals[0].n_stored)
    h.remove()
    out = {"logits": torch.stack(logits).numpy(), "n_stored": np.array(n_stored),
           "tokens": np.array([int(prompt[0, -1])] + [int(s) for s in steps[1:]])}
    path = os.path.join(HERE, "generator_golden.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden_ext.py <path to the reference checkout>")
    sys.path.insert(0, sys.argv[1])
    config0(sys.argv[1])
    generator(sys.argv[1])

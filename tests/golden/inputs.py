"""Seeded synthetic inputs shared by the fixture generator (which runs the
reference on them) and the GPU tests (which regenerate them and run this
library on them).  torch's CPU generator is deterministic for a given torch
version, so only the reference's OUTPUTS need to be stored.

config0_case: BASELINE configs[0] — one layer, 32 query / 8 KV heads,
head_dim 128, 4096-token context, fp32; K ~ N(0,1) x per-channel log-normal
scale with 4 outlier channels x20 per head, RoPE theta 5e5; V ~ N(0,1);
window 256, top 8 tiles of 64 (top_k = 512 tokens); 16 queries N(0,1), 4 of
them planted at cosine 0.9 to a random past (evicted) key.

tiny_llama: a small random-init fp16 Llama (head_dim 128) for the
generator-level fixture (see TINY).
"""
import math

import torch

C0 = dict(n=4096, n_kv=8, d=128, n_q=32, window=256, top_k=512, n_queries=16, n_planted=4, theta=500000.0)


def rope_tables(max_pos, d, theta):
    inv_freq = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    freqs = torch.arange(max_pos).float()[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos(), emb.sin()


def _rot(x, cos, sin):
    d2 = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., d2:], x[..., :d2]], -1) * sin


def config0_case(seed=4242):
    c = C0
    n, n_kv, d, n_q = c["n"], c["n_kv"], c["d"], c["n_q"]
    g = torch.Generator().manual_seed(seed)
    scale = torch.exp(torch.randn(n_kv, d, generator=g))
    for h in range(n_kv):
        scale[h, torch.randperm(d, generator=g)[:4]] *= 20.0
    k_pre = torch.randn(n, n_kv, d, generator=g) * scale
    v = torch.randn(n, n_kv, d, generator=g)
    cos, sin = rope_tables(n + 1, d, c["theta"])
    k_post = _rot(k_pre, cos[:n, None, :], sin[:n, None, :])
    n_ret = n - c["window"]
    qs = torch.randn(c["n_queries"], n_q, d, generator=g)
    planted = []
    gq = n_q // n_kv
    for i in range(c["n_planted"]):
        p = int(torch.randint(0, n_ret, (1,), generator=g))
        planted.append(p)
        for hq in range(n_q):
            kk = k_post[p, hq // gq]
            kh = kk / kk.norm()
            u = torch.randn(d, generator=g)
            u = u - (u @ kh) * kh
            u = u / u.norm()
            qs[i, hq] = (0.9 * kh + math.sqrt(1 - 0.81) * u) * math.sqrt(d)
    return {"k_pre": k_pre, "v": v, "k_post": k_post, "cos": cos, "sin": sin, "queries": qs,
            "planted_pos": planted, "n_ret": n_ret, **c}


# one KV head (n_kv*d = 128) and a 320-token prompt, so that the V-predict
# fit of calibrate (kvr_retrieval.py:105-112, pinv on the first half of the
# prompt: 160 samples of 128 dims) is well conditioned and the W of different
# LAPACK implementations agree; 224 evicted tokens stay below the 256 that
# would trigger the reference's host k-means.
TINY = dict(vocab_size=256, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
            num_key_value_heads=1, head_dim=128, max_position_embeddings=512, rope_theta=500000.0,
            window=96, top_k=16, n_prompt=320, n_steps=12)


def tiny_llama(seed=7):
    """fp16 LlamaForCausalLM with random weights (std 0.02 init, seeded), on CPU."""
    from transformers import LlamaConfig, LlamaForCausalLM

    cfg = LlamaConfig(vocab_size=TINY["vocab_size"], hidden_size=TINY["hidden_size"],
                      intermediate_size=TINY["intermediate_size"], num_hidden_layers=TINY["num_hidden_layers"],
                      num_attention_heads=TINY["num_attention_heads"],
                      num_key_value_heads=TINY["num_key_value_heads"], head_dim=TINY["head_dim"],
                      max_position_embeddings=TINY["max_position_embeddings"], rope_theta=TINY["rope_theta"],
                      attn_implementation="eager")
    torch.manual_seed(seed)
    model = LlamaForCausalLM(cfg).half().eval()
    g = torch.Generator().manual_seed(seed + 1)
    prompt = torch.randint(0, TINY["vocab_size"], (1, TINY["n_prompt"]), generator=g)
    steps = torch.randint(0, TINY["vocab_size"], (TINY["n_steps"],), generator=g)
    return model, prompt, steps

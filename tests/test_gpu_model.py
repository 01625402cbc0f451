"""Model integration (KVRHook / KVRGenerator drop-ins) on a tiny random-init
fp16 Llama with head_dim 128, on the GPU."""
import numpy as np
import pytest
import torch

from oracle import int4w_ref as R

pytestmark = pytest.mark.gpu
DEV = "cuda"


def tiny_llama(layers=2, n_q=4, n_kv=2, vocab=500, max_pos=4096, seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    cfg = LlamaConfig(vocab_size=vocab, hidden_size=n_q * 128, intermediate_size=1024, num_hidden_layers=layers,
                      num_attention_heads=n_q, num_key_value_heads=n_kv, head_dim=128,
                      max_position_embeddings=max_pos, rope_theta=500000.0)
    return LlamaForCausalLM(cfg).half().to(DEV).eval()


@pytest.mark.parametrize("codec", ["int4w", "sd1"])
def test_generator_matches_hf_when_window_holds_everything(codec):
    from kvr_b200 import KVRGenerator
    m = tiny_llama()
    prompt = torch.randint(0, 500, (1, 100), device=DEV)
    x = torch.tensor([[7]], device=DEV)
    gen = KVRGenerator(m, window_size=256, top_k=64, codec=codec, attractors=False)
    gen.prefill(prompt)
    gen._is_first = False  # x is a new token at position 100: store it, then attend
    ours = gen.logits_step(x)
    with torch.no_grad():
        want = m(torch.cat([prompt, x], 1)).logits[0, -1].float()
    assert torch.allclose(ours, want, rtol=2e-2, atol=2e-2), (ours - want).abs().max()


def test_hook_retrieval_wiring_matches_oracle():
    from kvr_b200 import KVRGenerator
    m = tiny_llama()
    prompt = torch.randint(0, 500, (1, 400), device=DEV)
    gen = KVRGenerator(m, window_size=128, top_k=96, codec="int4w", attractors=False)
    gen.prefill(prompt)
    kvr = gen.kvr
    assert kvr._retrieval_built and kvr.retrievals[0].n_stored == 272
    win, ret = kvr.windows[0], kvr.retrievals[0]
    q = torch.randn(4, 128, device=DEV)
    ours = kvr.attend(0, q).cpu().numpy()
    st = {"k_packed": ret.k_packed.cpu().numpy(), "vr_packed": ret.vr_packed.cpu().numpy(),
          "k_scales": ret.k_scales.cpu().numpy(), "vr_scales": ret.vr_scales.cpu().numpy(),
          "W": ret.W.cpu().numpy(), "K_mean": ret.K_mean.cpu().numpy(), "V_mean": ret.V_mean.cpu().numpy(),
          "n_stored": ret.n_stored}
    cos, sin = kvr.cos_tbl.cpu().numpy(), kvr.sin_tbl.cpu().numpy()
    ex = (max(0, 400 - win.n), min(ret.n_stored, 400))
    ex = (0, 0) if ex[0] >= ex[1] else ex
    rk, rv, _ = R.retrieve_token_branch(q.cpu().numpy(), st, cos, sin, 96, *ex)
    kc = np.concatenate([win.k[:win.n].float().cpu().numpy(), rk])
    vc = np.concatenate([win.v[:win.n].float().cpu().numpy(), rv.astype(np.float32)])
    want = R.softmax_attention(q.cpu().numpy(), kc, vc)
    assert np.abs(ours - want).max() <= 2e-3 * np.abs(want).max()


@pytest.mark.parametrize("codec", ["int4w", "sd1"])
def test_generator_runs_with_eviction(codec):
    from kvr_b200 import KVRGenerator
    m = tiny_llama()
    prompt = torch.randint(0, 500, (1, 300), device=DEV)
    gen = KVRGenerator(m, window_size=128, top_k=128, codec=codec, attractors=False)
    gen.prefill(prompt)
    n0 = gen.kvr.retrievals[0].n_tokens
    gen.step(prompt[0, -1])
    ids = gen.generate(5, temperature=0.7, top_k=20)
    assert ids.shape == (5,) and gen.kvr._context_len == 306
    # every step past the first evicts one window token into the index
    assert gen.kvr.retrievals[0].n_tokens == n0 + 5
    assert torch.isfinite(gen.logits_step(ids[-1])).all()


def test_hook_path_runs():
    from kvr_b200 import KVRHook
    m = tiny_llama()
    prompt = torch.randint(0, 500, (1, 200), device=DEV)
    hook = KVRHook(m, window_size=128, top_k=64, codec="sd1", attractors=False, num_denoise_steps=0)
    hook.prefill(prompt)
    hook.register()
    hook._step = 1
    hook._context_len = 201
    with torch.no_grad():
        out = m(torch.cat([prompt, prompt[:, :1]], 1)).logits
    hook.remove()
    assert torch.isfinite(out).all()


@pytest.mark.parametrize("n_prompt", [300, 90])
def test_sd1_fused_prefill_builds_the_same_stores(n_prompt):
    """The sd1 prefill that encodes inside the projection hooks (no fp32
    capture of the prompt) leaves exactly the window rings and 1-bit stores
    of the capture-then-encode path (ragged tail included)."""
    from kvr_b200 import KVRHook
    m = tiny_llama(layers=2)
    prompt = torch.randint(0, 500, (1, n_prompt), device=DEV)
    hooks = []
    for fused in (False, True):
        h = KVRHook(m, window_size=128, top_k=64, codec="sd1", transform="dct", attractors=False,
                    fused_prefill=fused, num_denoise_steps=0)
        h.prefill(prompt)
        hooks.append(h)
    a, b = hooks
    assert a._retrieval_built == b._retrieval_built and a._context_len == b._context_len == n_prompt
    for li in range(2):
        wa, wb = a.windows[li], b.windows[li]
        assert (wa.pos, wa.n) == (wb.pos, wb.n)
        assert torch.equal(wa.k, wb.k) and torch.equal(wa.v, wb.v)
        ra, rb = a.retrievals[li], b.retrievals[li]
        assert (ra.n_stored, ra.n_tail) == (rb.n_stored, rb.n_tail)
        if ra.n_stored:
            nt = ra.store.n_tiles
            assert nt == rb.store.n_tiles and nt > 0
            for name in ("kbits", "kscale", "vbits", "vscale"):
                assert torch.equal(getattr(ra.store, name)[:, :, :nt], getattr(rb.store, name)[:, :, :nt]), name
            assert torch.equal(ra.tail_k[:, :ra.n_tail], rb.tail_k[:, :rb.n_tail])
            assert torch.equal(ra.tail_v[:, :ra.n_tail], rb.tail_v[:, :rb.n_tail])


@pytest.mark.parametrize("codec", ["int4w", "sd1"])
def test_save_and_resume_decoding(codec, tmp_path):
    """save_cache / load_cache: a fresh generator that loads the compressed
    state continues with exactly the logits of the one that saved it."""
    from kvr_b200 import KVRGenerator
    m = tiny_llama()
    prompt = torch.randint(0, 500, (1, 300), device=DEV)
    gen = KVRGenerator(m, window_size=128, top_k=128, codec=codec, transform="dct", attractors=False)
    gen.prefill(prompt)
    gen.step(prompt[0, -1])
    gen.step(torch.tensor(5, device=DEV))
    path = tmp_path / f"{codec}.kvrc"
    gen.save_cache(path)
    gen2 = KVRGenerator(m, window_size=128, top_k=128, codec=codec, transform="dct", attractors=False)
    gen2.load_cache(path)
    x = torch.tensor(11, device=DEV)
    assert torch.equal(gen.logits_step(x), gen2.logits_step(x))
    assert gen.kvr._context_len == gen2.kvr._context_len

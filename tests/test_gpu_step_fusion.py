"""The fused per-layer decode store update (kvr_decode_store_update): RoPE of
q and k bit-identical to the eager torch arithmetic of
modules/kvr_generator.py:91-94 in every model dtype, the window write and the
eviction into the 1-bit tail; and KVRGenerator with the fused kernel against
the step-by-step path."""
import os
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import inputs  # noqa: E402


@pytest.mark.parametrize("heads", [(32, 8), (64, 8), (4, 1)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_rope_and_window_write_bit_exact(dtype, heads):
    n_q, n_kv = heads
    from kvr_b200 import kernels as K
    from kvr_b200.kvr_retrieval import _apply_rotary
    g = torch.Generator(device="cuda").manual_seed(0)
    cos, sin = inputs.rope_tables(1000, 128, 500000.0)
    cos, sin = cos.cuda(), sin.cuda()
    q = (torch.randn(n_q, 128, device="cuda", generator=g) * 3).to(dtype)
    k = (torch.randn(n_kv, 128, device="cuda", generator=g) * 3).to(dtype)
    v = torch.randn(n_kv, 128, device="cuda", generator=g).to(dtype)
    ring_k = torch.randn(16, n_kv, 128, device="cuda", generator=g).half()
    ring_v = torch.randn(16, n_kv, 128, device="cuda", generator=g).half()
    ring_k0, ring_v0 = ring_k.clone(), ring_v.clone()
    tail_k = torch.zeros(64, n_kv, 128, device="cuda", dtype=torch.float16)
    tail_v = torch.zeros_like(tail_k)
    old_k, old_v = ring_k[5].clone(), ring_v[5].clone()
    pos = 777
    c, s = cos[pos:pos + 1].to(dtype), sin[pos:pos + 1].to(dtype)
    q_rot = K.decode_store_update(q, k, v, cos, sin, pos, ring_k, ring_v, 5, tail_k, tail_v, 9)
    torch.cuda.synchronize()
    assert torch.equal(q_rot, _apply_rotary(q, c, s))
    assert torch.equal(ring_k[5], _apply_rotary(k, c, s).to(torch.float16))
    assert torch.equal(ring_v[5], v.to(torch.float16))
    assert torch.equal(tail_k[9], old_k) and torch.equal(tail_v[9], old_v)
    assert int((tail_k.abs().sum(dim=(1, 2)) > 0).sum()) == 1
    others = [i for i in range(16) if i != 5]
    assert torch.equal(ring_k[others], ring_k0[others]) and torch.equal(ring_v[others], ring_v0[others])
    # q only (the first decode step)
    before = ring_k.clone()
    q2 = K.decode_store_update(q, k, v, cos, sin, pos + 1, ring_k, ring_v, 6, write_kv=False)
    torch.cuda.synchronize()
    assert torch.equal(ring_k, before)
    assert torch.equal(q2, _apply_rotary(q, cos[pos + 1:pos + 2].to(dtype), sin[pos + 1:pos + 2].to(dtype)))


def test_generator_fused_store_update_matches_step_by_step():
    """codec='sd1' KVRGenerator on the tiny fp16 Llama, 80 steps past a
    prefill (the window stays full, so every step evicts into the tail and a
    full tail is encoded into a tile): the fused kernel and the step-by-step
    path give the same stores and logits (the evicted rows agree exactly or
    to one fp16 ulp: the step-by-step path un-rotates and re-rotates them)."""
    from kvr_b200 import KVRGenerator
    model, prompt, steps = inputs.tiny_llama()
    model = model.cuda()
    gens = []
    for fused in (True, False):
        gen = KVRGenerator(model, window_size=inputs.TINY["window"], top_k=128, device="cuda", codec="sd1",
                           tile=64, transform="dct", fused_store_update=fused)
        gen.prefill(prompt.cuda())
        gens.append(gen)
    rng = np.random.default_rng(0)
    for i in range(80):
        tok = int(rng.integers(0, inputs.TINY["vocab_size"]))
        outs = []
        for gen in gens:
            outs.append(gen.logits_step(tok).float())
            gen.kvr._context_len += 1
            gen._is_first = False
        err = (outs[0] - outs[1]).abs().max().item()
        assert err <= 2e-2 * outs[1].abs().max().item(), (i, err)
    for li in range(inputs.TINY["num_hidden_layers"]):
        w0, w1 = gens[0].kvr.windows[li], gens[1].kvr.windows[li]
        assert (w0.pos, w0.n) == (w1.pos, w1.n)
        assert torch.equal(w0.k, w1.k) and torch.equal(w0.v, w1.v)
        r0, r1 = gens[0].kvr.retrievals[li], gens[1].kvr.retrievals[li]
        assert (r0.n_stored, r0.n_tail) == (r1.n_stored, r1.n_tail)
        a, b = r0.tail_k[0, :r0.n_tail].float(), r1.tail_k[0, :r1.n_tail].float()
        assert torch.all((a - b).abs() <= 2 * torch.finfo(torch.float16).eps * b.abs() + 1e-6)
        assert torch.equal(r0.tail_v[0, :r0.n_tail], r1.tail_v[0, :r1.n_tail])

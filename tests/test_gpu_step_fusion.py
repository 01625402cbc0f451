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


def _sd1_layer(g, nt, n_kv=8, cap=128, tile=64, kind="dct"):
    from kvr_b200 import kernels as K
    st = K.Sd1Store(1, n_kv, nt + 2, tile, kind, "cuda")
    scale = torch.exp(torch.randn(n_kv, 128, device="cuda", generator=g))
    k = torch.randn(1, nt * tile, n_kv, 128, device="cuda", generator=g) * scale
    v = torch.randn(1, nt * tile, n_kv, 128, device="cuda", generator=g)
    K.sd1_encode(st, k.to(torch.bfloat16), v.to(torch.bfloat16))
    win_k = torch.randn(cap, n_kv, 128, device="cuda", generator=g).half()
    win_v = torch.randn(cap, n_kv, 128, device="cuda", generator=g).half()
    tail_k = torch.randn(1, tile, n_kv, 128, device="cuda", generator=g).half()
    tail_v = torch.randn(1, tile, n_kv, 128, device="cuda", generator=g).half()
    return st, win_k, win_v, tail_k, tail_v


@pytest.mark.parametrize("dtype,full,tile,kind", [
    (torch.bfloat16, True, 64, "dct"), (torch.bfloat16, False, 64, "dct"), (torch.float16, True, 64, "dct"),
    (torch.float16, False, 64, "dct"), (torch.float32, True, 64, "dct"), (torch.float32, False, 64, "dct"),
    (torch.bfloat16, True, 32, "hadamard"), (torch.bfloat16, True, 128, "dct")])
def test_fused_step_update_matches_store_update_then_step(dtype, full, tile, kind):
    """kvr_sd1_decode_step_update (one cluster launch) leaves the same window,
    tail and rotated q as kvr_decode_store_update, and gives the same tile
    selection and outputs as kvr_sd1_decode_step after it, bit for bit, over
    three consecutive steps (with and without eviction)."""
    from kvr_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(3)
    cos, sin = inputs.rope_tables(4096, 128, 500000.0)
    cos, sin = cos.cuda(), sin.cuda()
    st, wk, wv, tk, tv = _sd1_layer(g, 40 * 64 // tile, tile=tile, kind=kind)
    wk2, wv2, tk2, tv2 = wk.clone(), wv.clone(), tk.clone(), tv.clone()
    cap, n_kv, k_sel = wk.shape[0], 8, 16 * 64 // tile
    n_win = cap if full else 100
    n_tail = 5
    for step in range(3):
        pos = 3000 + step
        q = (torch.randn(32, 128, device="cuda", generator=g) * 2).to(dtype)
        k = (torch.randn(n_kv, 128, device="cuda", generator=g) * 2).to(dtype)
        v = torch.randn(n_kv, 128, device="cuda", generator=g).to(dtype)
        if full:
            slot, evict = (17 + step) % cap, True
            n_tail += 1
        else:
            slot, evict = n_win, False
            n_win += 1
        q_rot = K.decode_store_update(q, k, v, cos, sin, pos, wk, wv, slot, tk[0] if evict else None,
                                      tv[0] if evict else None, n_tail - 1, True)
        sel1 = torch.empty(1, n_kv, k_sel, dtype=torch.int32, device="cuda")
        out1 = K.sd1_decode_step(st, q_rot, k_sel, wk.unsqueeze(0), wv.unsqueeze(0), n_win, tk, tv, n_tail,
                                 sel_out=sel1)
        sel2 = torch.empty_like(sel1)
        out2, q_out = K.sd1_decode_step_update(st, q, k, v, cos, sin, pos, k_sel, wk2.unsqueeze(0), wv2.unsqueeze(0),
                                               n_win, slot, tk2, tv2, n_tail, evict, sel_out=sel2)
        torch.cuda.synchronize()
        assert torch.equal(q_out, q_rot), step
        assert torch.equal(wk2, wk) and torch.equal(wv2, wv), step
        assert torch.equal(tk2[:, :n_tail], tk[:, :n_tail]) and torch.equal(tv2[:, :n_tail], tv[:, :n_tail]), step
        assert torch.equal(sel2, sel1), step
        assert torch.equal(out2, out1), step


def test_fused_step_update_split_fallback():
    """With the two-kernel step selected, the fused entry point runs the
    store-update kernel and the split step: same stores and selection, outputs
    within fp32 rounding of the cluster kernel's."""
    from kvr_b200 import kernels as K
    from kvr_b200 import _native as N
    g = torch.Generator(device="cuda").manual_seed(4)
    cos, sin = inputs.rope_tables(4096, 128, 500000.0)
    cos, sin = cos.cuda(), sin.cuda()
    st, wk, wv, tk, tv = _sd1_layer(g, 24)
    wk2, wv2, tk2, tv2 = wk.clone(), wv.clone(), tk.clone(), tv.clone()
    q = torch.randn(32, 128, device="cuda", generator=g).to(torch.bfloat16)
    k = torch.randn(8, 128, device="cuda", generator=g).to(torch.bfloat16)
    v = torch.randn(8, 128, device="cuda", generator=g).to(torch.bfloat16)
    sel1 = torch.empty(1, 8, 16, dtype=torch.int32, device="cuda")
    sel2 = torch.empty_like(sel1)
    out1, q1 = K.sd1_decode_step_update(st, q, k, v, cos, sin, 1234, 16, wk.unsqueeze(0), wv.unsqueeze(0), 128, 9,
                                        tk, tv, 3, True, sel_out=sel1)
    lib = N.lib()
    prev = lib.kvr_set_sd1_step_path(1)
    try:
        out2, q2 = K.sd1_decode_step_update(st, q, k, v, cos, sin, 1234, 16, wk2.unsqueeze(0), wv2.unsqueeze(0), 128,
                                            9, tk2, tv2, 3, True, sel_out=sel2)
        torch.cuda.synchronize()
    finally:
        lib.kvr_set_sd1_step_path(prev)
    assert torch.equal(q1, q2) and torch.equal(sel1, sel2)
    assert torch.equal(wk, wk2) and torch.equal(wv, wv2) and torch.equal(tk[:, :3], tk2[:, :3])
    err = (out1.float() - out2.float()).abs().max() / out1.float().abs().max()
    assert err < 1e-2, err  # bf16 outputs: one rounding step apart at most


def test_retrieval_index_decode_step_over_a_tile_period():
    """RetrievalIndex.decode_step against the separate calls (store update
    kernel, tail encode when full, RetrievalIndex.attend) on two copies of one
    index: 70 steps with a full window, so one step fills the tail and encodes
    it; outputs, rotated q, windows, tails and stores bit-identical."""
    from kvr_b200 import RetrievalIndex, WindowBuffer
    from kvr_b200 import kernels as K
    g = torch.Generator(device="cuda").manual_seed(11)
    n_kv, n_q, tile, cap = 8, 32, 64, 128
    cos, sin = inputs.rope_tables(4096, 128, 500000.0)
    cos, sin = cos.cuda(), sin.cuda()
    k0 = torch.randn(40 * tile + 7, n_kv, 128, device="cuda", generator=g) * 3
    v0 = torch.randn(40 * tile + 7, n_kv, 128, device="cuda", generator=g)
    wk0 = torch.randn(cap, n_kv, 128, device="cuda", generator=g).half()
    wv0 = torch.randn(cap, n_kv, 128, device="cuda", generator=g).half()
    pairs = []
    for _ in range(2):
        ri = RetrievalIndex(n_kv, 128, top_k=16 * tile, device="cuda", codec="sd1", tile=tile, transform="dct")
        ri.set_rotary_tables(cos, sin)
        ri.calibrate(k0, v0)
        ri.batch_append(k0, v0)
        wb = WindowBuffer(n_kv, 128, cap, "cuda")
        wb.k.copy_(wk0)
        wb.v.copy_(wv0)
        wb.pos, wb.n = 5, cap
        pairs.append((ri, wb))
    (r1, w1), (r2, w2) = pairs
    assert r1.n_tail == 7
    for step in range(70):
        pos = 3000 + step
        q = torch.randn(n_q, 128, device="cuda", generator=g).to(torch.bfloat16)
        k = torch.randn(n_kv, 128, device="cuda", generator=g).to(torch.bfloat16)
        v = torch.randn(n_kv, 128, device="cuda", generator=g).to(torch.bfloat16)
        # separate calls, as KVRHook.decode_store_update + RetrievalIndex.attend
        slot = w1.pos % w1.cap
        q_rot = K.decode_store_update(q, k, v, cos, sin, pos, w1.k, w1.v, slot, r1.tail_k[0], r1.tail_v[0],
                                      r1.n_tail, True)
        r1.n_tail += 1
        if r1.n_tail == tile:
            K.sd1_encode(r1.store, r1.tail_k, r1.tail_v)
            r1.n_stored += tile
            r1.n_tail = 0
        w1.pos += 1
        out1 = r1.attend(q_rot, w1)
        out2, q2 = r2.decode_step(q, k, v, w2, pos, cos, sin)
        torch.cuda.synchronize()
        assert torch.equal(q2, q_rot), step
        assert torch.equal(out2, out1), step
        assert (r1.n_stored, r1.n_tail, w1.pos, w1.n) == (r2.n_stored, r2.n_tail, w2.pos, w2.n), step
    assert r2.store.n_tiles == r1.store.n_tiles == 41
    assert torch.equal(w1.k, w2.k) and torch.equal(w1.v, w2.v)
    assert torch.equal(r1.tail_k[:, :r1.n_tail], r2.tail_k[:, :r2.n_tail])
    for name in ("kbits", "kscale", "vbits", "vscale"):
        assert torch.equal(getattr(r1.store, name)[:, :, :41], getattr(r2.store, name)[:, :, :41]), name

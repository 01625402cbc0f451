"""Eviction parity (modules/kvr_hook.py:136-148): when the window is full, the
slot about to be overwritten is un-rotated and appended to the index.  The
appended int4 K codes must equal the oracle's quantize_k(reverse_rotary(...))
bit for bit, for both rotation positions: the evicted token's own position
(default) and the reference's ``win.pos`` (reference_eviction_rope=True)."""
import os
import sys

import numpy as np
import pytest
import torch

from oracle import int4w_ref as R

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import inputs  # noqa: E402


@pytest.mark.parametrize("reference_rope", [False, True])
def test_evicted_k_codes_bit_exact(reference_rope):
    from kvr_b200 import KVRHook
    model, prompt, _ = inputs.tiny_llama()
    model = model.to("cuda")
    hook = KVRHook(model, window_size=inputs.TINY["window"], top_k=16, device="cuda", chunk_size=0,
                   reference_eviction_rope=reference_rope)
    hook.prefill(prompt.to("cuda"))
    cos, sin = hook.cos_tbl.cpu().numpy(), hook.sin_tbl.cpu().numpy()
    g = torch.Generator(device="cuda").manual_seed(3)
    for step in range(6):
        for li in range(hook.n_layers):
            win, ret = hook.windows[li], hook.retrievals[li]
            slot = win.pos % win.cap
            old_post = win.k[slot].float().cpu().numpy()
            old_pos = win.pos if reference_rope else win.pos - win.cap
            n0 = ret.n_stored
            k_pre = torch.randn(hook.n_kv, 128, device="cuda", generator=g)
            v = torch.randn(hook.n_kv, 128, device="cuda", generator=g)
            hook._update_stores(li, k_pre, v, k_pre)
            assert ret.n_stored == n0 + 1
            want_pre = R.reverse_rotary(old_post, cos[old_pos][None], sin[old_pos][None]).astype(np.float32)
            want = R.pack_int4(R.quantize_k(want_pre[None], ret.k_scales.cpu().numpy()))[0]
            assert np.array_equal(ret.k_packed[n0].cpu().numpy(), want), (step, li)
        hook._context_len += 1

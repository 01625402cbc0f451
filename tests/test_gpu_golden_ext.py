"""GPU parity against the reference-generated configs[0] and generator
fixtures (tests/golden/make_golden_ext.py); inputs regenerated from the seeds
in tests/golden/inputs.py.  Every kernel call goes through the C ABI."""
import hashlib
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
from test_oracle_golden_ext import residual_boundary_check  # noqa: E402

C = np.load(os.path.join(HERE, "golden", "config0_golden.npz"))
GEN = np.load(os.path.join(HERE, "golden", "generator_golden.npz"))
DEV = "cuda"


def test_config0_encode_on_gpu_vs_reference():
    """GPU calibrate + batch_append (prefill, kvr_hook.py:130-132): k_scales
    and the packed K codes bit-exact; int2 residual codes equal except at
    rounding boundaries of the V prediction (mismatches counted)."""
    from kvr_b200 import RetrievalIndex
    c = inputs.config0_case()
    n_ret = c["n_ret"]
    ri = RetrievalIndex(8, 128, top_k=512, device=DEV, chunk_size=0)
    ri.set_rotary_tables(c["cos"].to(DEV), c["sin"].to(DEV))
    ri.calibrate(c["k_pre"].to(DEV), c["v"].to(DEV))
    ri.batch_append(c["k_pre"][:n_ret].to(DEV), c["v"][:n_ret].to(DEV))
    assert np.array_equal(ri.k_scales.cpu().numpy(), C["k_scales"])
    kp = ri.k_packed[:n_ret].cpu().numpy()
    assert hashlib.sha256(kp.tobytes()).digest() == C["k_packed_sha256"].tobytes()
    got = R.unpack_int2(ri.vr_packed[:n_ret].cpu().numpy())
    want = R.unpack_int2(C["vr_packed"])
    k, v = c["k_pre"].numpy(), c["v"].numpy()
    cal = R.calibrate(k, v)
    vpred = R.predict_v(k[:n_ret].reshape(n_ret, -1), cal["W"], cal["K_mean"], cal["V_mean"]).reshape(n_ret, 8, 128)
    # the V prediction the GPU encoder itself used (same library call as batch_append)
    mine = ri._predict_v(c["k_pre"][:n_ret].to(DEV).reshape(n_ret, -1).float()).reshape(n_ret, 8, 128).cpu().numpy()
    n_bad = residual_boundary_check(v[:n_ret], vpred, cal["vr_scales"], got, want, rel=1e-5, vpred_alt=mine,
                                    vr_scales_alt=ri.vr_scales.cpu().numpy())
    assert n_bad <= 1e-3 * got.size, n_bad


def test_config0_decode_vs_reference():
    """For all 16 queries: the token-branch top-512 (near ties as sets) and
    RetrievalIndex.attend over the window + retrieved rows against the
    reference hook's softmax, 1e-5 of the largest output (fp32)."""
    from kvr_b200 import RetrievalIndex, WindowBuffer
    c = inputs.config0_case()
    n_ret = c["n_ret"]
    k, v = c["k_pre"].numpy(), c["v"].numpy()
    cal = R.calibrate(k, v)      # the reference's calibration (same torch CPU routine)
    ri = RetrievalIndex(8, 128, top_k=512, device=DEV, chunk_size=0)
    ri.set_rotary_tables(c["cos"].to(DEV), c["sin"].to(DEV))
    ri.calibrate(c["k_pre"].to(DEV), c["v"].to(DEV))
    ri.batch_append(c["k_pre"][:n_ret].to(DEV), c["v"][:n_ret].to(DEV))
    for x in ("W", "K_mean", "V_mean", "vr_scales"):
        setattr(ri, x, torch.from_numpy(cal[x]).to(DEV))
    ri.vr_packed[:n_ret] = torch.from_numpy(C["vr_packed"]).to(DEV)
    wb = WindowBuffer(8, 128, window_size=c["window"], device=DEV)
    wb.batch_append(c["k_post"].to(DEV), c["v"].to(DEV))
    assert (wb.pos, wb.n) == (int(C["win_pos"]), int(C["win_n"]))
    st = dict(cal)
    st.update(k_packed=ri.k_packed[:n_ret].cpu().numpy(), n_stored=n_ret)
    cos, sin = c["cos"].numpy(), c["sin"].numpy()
    ex = tuple(int(x) for x in C["ex"])
    win_k, win_v = wb.k.float().cpu().numpy(), wb.v.float().cpu().numpy()
    for qi in range(c["queries"].shape[0]):
        q = c["queries"][qi].to(DEV)
        top = ri.select_indices(q, *ex)
        sc = R.token_scores(c["queries"][qi].numpy(), st["k_packed"], st["k_scales"], cos, sin, n_ret)
        assert R.near_tie_ok(sc, top.cpu().numpy(), C["top"][qi].astype(np.int64)), qi
        out = ri.attend(q, wb, *ex).cpu().numpy()
        rk, rv = ri.retrieve_topk(q, n_q=32, exclude_start=ex[0], exclude_end=ex[1])
        # (a) the attention itself: exact softmax over the rows it was given
        ref = R.softmax_attention(c["queries"][qi].numpy(), np.concatenate([win_k, rk.cpu().numpy()]),
                                  np.concatenate([win_v, rv.float().cpu().numpy()]))
        assert np.abs(out - ref).max() <= 1e-5 * np.abs(ref).max(), qi
        # (b) the retrieved V: within half an fp16 ulp of the exact (float64)
        # value of the reference's arithmetic, as the reference's own fp16 ret_v is
        vex = _v_exact(st, top.cpu().numpy(), cal, C["vr_packed"])
        ulp = np.spacing(np.abs(vex).astype(np.float16)).astype(np.float64)
        assert np.all(np.abs(rv.float().cpu().numpy() - vex) <= 0.5 * ulp + 1e-6 * np.abs(vex).max()), qi
        # (c) against the reference's output: the same up to those last-bit fp16
        # roundings of V (a peaked softmax passes one of them through whole)
        want = C["attn"][qi]
        assert np.abs(out - want).max() <= 1e-3 * np.abs(want).max(), (qi, np.abs(out - want).max())


def _v_exact(st, top, cal, vr_packed):
    n_kv = top.shape[1]
    kpre = R.unpack_int4(st["k_packed"][top]).astype(np.float64) * R.k_step(cal["k_scales"])[None, None]
    W, km, vm = cal["W"].astype(np.float64), cal["K_mean"].astype(np.float64), cal["V_mean"].astype(np.float64)
    vstep = R.vr_step(cal["vr_scales"]).astype(np.float64)
    out = np.empty(top.shape + (128,))
    for h in range(n_kv):
        x = kpre[:, h].reshape(len(top), -1) - km
        vb = (x @ W.T + vm).reshape(len(top), n_kv, 128)[:, h]
        out[:, h] = vb + R.unpack_int2(vr_packed[top[:, h]][:, h]).astype(np.float64) * vstep[h]
    return out


def test_generator_logits_vs_reference():
    """KVRGenerator on the tiny fp16 Llama: prefill 320 tokens (window 96,
    top_k 16), then 12 steps fed with the fixture's token ids; every step
    evicts one token per layer into the index (reference_eviction_rope=True
    reproduces modules/kvr_hook.py:142-144).  Logits within fp16 model
    tolerance of the reference's CPU run; the index grows as the reference's."""
    from kvr_b200 import KVRGenerator
    model, prompt, steps = inputs.tiny_llama()
    model = model.to(DEV)
    gen = KVRGenerator(model, window_size=inputs.TINY["window"], top_k=inputs.TINY["top_k"], device=DEV,
                       chunk_size=0, reference_eviction_rope=True)
    gen.prefill(prompt.to(DEV))
    stored = [gen.kvr.retrievals[0].n_stored]
    want = GEN["logits"]
    for i, tok in enumerate(GEN["tokens"]):
        logits = gen.logits_step(int(tok)).float().cpu().numpy()
        gen.kvr._context_len += 1
        gen._is_first = False
        stored.append(gen.kvr.retrievals[0].n_stored)
        err = np.abs(logits - want[i]).max()
        assert err <= 2e-2 * np.abs(want[i]).max(), (i, err)
        cos = float(logits @ want[i] / (np.linalg.norm(logits) * np.linalg.norm(want[i])))
        assert cos > 0.9999, (i, cos)
    assert stored == GEN["n_stored"].tolist()

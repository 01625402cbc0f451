"""The CPU timing port (oracle/int4w_ref_cpu.py) computes what the pinned
oracle computes (same retrieval + attention) on a small case."""
import numpy as np
import torch

from oracle import int4w_ref as R
from oracle import int4w_ref_cpu as C


def test_cpu_port_matches_oracle():
    c = C.make_case(seed=3, n_stored=600, window=64, n_kv=4, n_q=16, d=128)
    out = C.decode_layer(c, 128, q_index=1).numpy()
    st = {x: c[x].numpy() for x in ("k_packed", "k_scales", "vr_packed", "vr_scales", "W", "K_mean", "V_mean")}
    st["n_stored"] = 600
    q = c["q"][1].numpy()
    rk, rv, top = R.retrieve_token_branch(q, st, c["cos"].numpy(), c["sin"].numpy(), 128)
    want = R.softmax_attention(q, np.concatenate([c["win_k"].float().numpy(), rk]),
                               np.concatenate([c["win_v"].float().numpy(), rv.astype(np.float32)]))
    np.testing.assert_allclose(out, want, rtol=1e-4, atol=1e-4)

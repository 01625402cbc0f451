"""Retired Triton entry points (modules/kvr_triton.py), same names, CUDA kernels.

* ``run_fused_attn(q, k, v)`` (kvr_triton.py:93-104): exact decode attention of
  q (n_q, d) over k, v (n_tok, n_kv, d); output dtype = q's.
* ``run_score_kernel(q_first, k_packed, k_scales, cos_tbl, sin_tbl)``
  (kvr_triton.py:82-90): the reference Triton kernel read the FIRST query head
  of each GQA group and scaled by 2*s/16; its (n_stored, d) cos stride was the
  documented bug #19 (docs, fixed only in the CUDA kernel).  This entry point
  keeps the group-first query but uses the fixed (n_stored, d/2) tables.
"""
from . import kernels as K


def run_fused_attn(q, k, v):
    return K.decode_attn(q, [(k, v)], out_dtype=q.dtype, n_kv=k.shape[1])


def run_score_kernel(q_first, k_packed, k_scales, cos_tbl, sin_tbl):
    n_kv = k_packed.shape[1]
    g = q_first.shape[0] // n_kv
    q_sel = q_first.reshape(n_kv, g, -1)[:, 0, :]
    return K.compute_scores(q_sel, k_packed, k_scales, cos_tbl, sin_tbl)

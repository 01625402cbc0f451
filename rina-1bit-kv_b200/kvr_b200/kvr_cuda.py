"""Drop-in for modules/kvr_cuda.py: the fused score search.

``run_score_kernel_cuda`` keeps the reference signature and semantics
(kvr_cuda.py:20-26, kernel kvr_cuda.cu:9-49: interleaved-pair RoPE with
(n_stored, d/2) tables, dot with the pre-averaged query, / sqrt(d)); it runs
the prebuilt sm_100a kernel instead of JIT-compiling one.
"""
from . import kernels as K


def run_score_kernel_cuda(q_avg, k_packed, k_scales, cos_tbl, sin_tbl):
    """CUDA fused score search. cos_tbl: (n_stored, d//2) — one cos per pair."""
    return K.compute_scores(q_avg, k_packed, k_scales, cos_tbl, sin_tbl)

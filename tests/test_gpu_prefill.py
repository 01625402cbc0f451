"""Prefill-sized tile scoring on tcgen05 tensor cores vs the CPU spec
(oracle/sd1_ref.py prefill_tile_scores): fp16 q' and exact fp16 k_hat, fp32
accumulation -> relative error <= 1e-5 of the largest score."""
import numpy as np
import pytest
import torch

from oracle import sd1_ref as S

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("kind,nq,nt", [("dct", 200, 10), ("hadamard", 128, 4), ("dct", 37, 7), ("hadamard", 300, 13),
                                             ("dct", 1000, 301), ("hadamard", 700, 512)])
@pytest.mark.parametrize("qdtype", [torch.bfloat16])
def test_prefill_scores_vs_spec(kind, nq, nt, qdtype):
    from kvr_b200 import kernels as K
    rng = np.random.default_rng(nq + nt)
    n_kv, n_q, tile = 2, 8, 64
    k = (rng.standard_normal((1, nt * tile, n_kv, 128)) * np.exp(rng.standard_normal((n_kv, 128)))).astype(np.float32)
    v = rng.standard_normal((1, nt * tile, n_kv, 128)).astype(np.float32)
    st = K.Sd1Store(1, n_kv, nt + 2, tile, kind, DEV)
    K.sd1_encode(st, torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV))
    q = torch.from_numpy(rng.standard_normal((nq, n_q, 128)).astype(np.float32)).to(DEV).to(qdtype)
    got = K.sd1_prefill_scores(st, q).cpu().numpy()
    qp16 = S.prefill_qprime_f16(q.float().cpu().numpy(), n_kv, kind)
    for h in range(n_kv):
        want = S.prefill_tile_scores(qp16[:, h], st.kbits[0, h, :nt].cpu().numpy().view(np.uint32),
                                     st.kscale[0, h, :nt].cpu().numpy())
        err = np.abs(got[:, h] - want).max() / np.abs(want).max()
        assert err < 1e-5, (h, err)


@pytest.mark.parametrize("qdtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("kind", ["dct", "hadamard"])
def test_prefill_scores_other_query_dtypes(kind, qdtype):
    test_prefill_scores_vs_spec(kind, 260, 9, qdtype)


def test_prefill_scores_gqa8_and_many_heads():
    """g = 8 query heads per KV head and more (head, token group) items than SMs."""
    from kvr_b200 import kernels as K
    rng = np.random.default_rng(3)
    n_kv, n_q, tile, nt, nq = 4, 32, 64, 160, 130
    k = rng.standard_normal((1, nt * tile, n_kv, 128)).astype(np.float32)
    st = K.Sd1Store(1, n_kv, nt, tile, "dct", DEV)
    K.sd1_encode(st, torch.from_numpy(k).to(DEV), torch.from_numpy(k).to(DEV))
    q = torch.from_numpy(rng.standard_normal((nq, n_q, 128)).astype(np.float32)).to(DEV).bfloat16()
    got = K.sd1_prefill_scores(st, q).cpu().numpy()
    qp16 = S.prefill_qprime_f16(q.float().cpu().numpy(), n_kv, "dct")
    for h in range(n_kv):
        want = S.prefill_tile_scores(qp16[:, h], st.kbits[0, h, :nt].cpu().numpy().view(np.uint32),
                                     st.kscale[0, h, :nt].cpu().numpy())
        assert np.abs(got[:, h] - want).max() / np.abs(want).max() < 1e-5

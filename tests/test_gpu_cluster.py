"""On-device k-means (kvr_kmeans) that replaces the host MiniBatchKMeans of
the int4w attractor branch: labels identical to the specification
(oracle/int4w_ref.py kmeans_lloyd) on separated data, centroids to fp32
accuracy, bit-identical repeat runs; the attractor retrieval path runs on it."""
import numpy as np
import pytest
import torch

from oracle import int4w_ref as R

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _blobs(seed, k_true, per, noise=0.05, ordered=False):
    """k_true separated blobs; ordered=True lays them out blob by blob, so the
    evenly spaced initial centroids fall in distinct blobs (no near-ties
    between two centroids of one blob, where fp32 and float64 may split a
    blob differently)."""
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((k_true, 128)).astype(np.float32) * 4.0
    which = np.repeat(np.arange(k_true), per) if ordered else rng.integers(0, k_true, k_true * per)
    x = centers[which] + noise * rng.standard_normal((k_true * per, 128))
    return x.astype(np.float32)


@pytest.mark.parametrize("k,k_true,per,iters,ordered", [(128, 128, 20, 10, True), (16, 24, 50, 6, False),
                                                        (1, 3, 10, 2, False), (256, 200, 6, 4, False)])
def test_kmeans_matches_spec(k, k_true, per, iters, ordered):
    from kvr_b200 import kernels as K
    x = _blobs(k + k_true, k_true, per, ordered=ordered)
    lab, c = K.kmeans(torch.from_numpy(x).to(DEV), k, iters)
    want_lab, want_c = R.kmeans_lloyd(x, k, iters)
    assert np.array_equal(lab.cpu().numpy(), want_lab)
    np.testing.assert_allclose(c.cpu().numpy(), want_c, rtol=1e-4, atol=1e-4)


def test_kmeans_is_deterministic():
    from kvr_b200 import kernels as K
    x = torch.from_numpy(_blobs(1, 300, 20, noise=1.0)).to(DEV)  # overlapping blobs
    l1, c1 = K.kmeans(x, 128, 8)
    l2, c2 = K.kmeans(x, 128, 8)
    assert torch.equal(l1, l2) and torch.equal(c1, c2)


def test_attractor_branch_on_device_basins():
    from kvr_b200 import RetrievalIndex
    rng = np.random.default_rng(2)
    n_kv, n = 2, 1200
    k_pre = torch.from_numpy(rng.standard_normal((n, n_kv, 128)).astype(np.float32)).to(DEV)
    v = torch.from_numpy(rng.standard_normal((n, n_kv, 128)).astype(np.float32)).to(DEV)
    idx = RetrievalIndex(n_kv, 128, top_k=256, device=DEV, codec="int4w")
    pos = torch.arange(4096, device=DEV, dtype=torch.float32)[:, None]
    inv = 1.0 / (500000.0 ** (torch.arange(0, 128, 2, device=DEV).float() / 128))
    ang = torch.cat([pos * inv, pos * inv], 1)
    idx.set_rotary_tables(ang.cos(), ang.sin())
    idx.calibrate(k_pre, v)
    idx.batch_append(k_pre, v)
    idx.build_attractors()
    assert idx.labels.shape == (n,) and idx.attractors.shape == (128, 128)
    assert int(idx.labels.min()) >= 0 and int(idx.labels.max()) < 128
    q = torch.from_numpy(rng.standard_normal((8, 128)).astype(np.float32)).to(DEV)
    sel = idx.select_indices(q, 100, 300)
    sel2 = idx.select_indices(q, 100, 300)
    assert sel is not None and torch.equal(sel, sel2)
    s = sel.reshape(-1).cpu().numpy()
    s = s[s >= 0]
    assert len(s) > 0 and s.max() < n and not ((s >= 100) & (s < 300)).any()

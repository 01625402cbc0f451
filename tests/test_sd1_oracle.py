"""CPU known-answer tests of the sd1 specification (oracle/sd1_ref.py) and of
the constants the kernels bake in."""
import os
import re

import numpy as np

from oracle import sd1_ref as S

F32 = np.float32
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_transforms_are_orthonormal_and_invert():
    x = np.random.default_rng(0).standard_normal((64, 128)).astype(F32)
    for kind in ("hadamard", "dct"):
        T = S.transform_matrix(kind)
        assert np.abs(T @ T.T - np.eye(128)).max() < 1e-12
        y = S.transform(x, kind)
        assert np.abs(y - x.astype(np.float64) @ T.T).max() < 1e-5 * np.abs(x).max() * 4
        assert np.abs(S.transform(y, kind, inverse=True) - x).max() < 2e-5 * np.abs(x).max()


def test_dct_matches_textbook_dct2():
    x = np.zeros((1, 128), F32)
    x[0, 0] = 1.0
    y = S.dct_fwd(x)[0]
    n = np.arange(128)
    want = np.cos(np.pi * (2 * 0 + 1) * n / 256) * np.sqrt(2 / 128)
    want[0] = np.sqrt(1 / 128)
    assert np.abs(y - want).max() < 1e-6


def test_sigma_delta_hand_case():
    # one channel, tile of 4: x = [1, 1, -1, 3] -> s = fp16(1.5)
    x = np.array([[1.0], [1.0], [-1.0], [3.0]], F32)
    bits, s = S.sigma_delta_tile(x)
    assert float(s[0]) == 1.5
    # u: 1 -> b=1,e=-0.5; u=0.5 -> b=1,e=-1; u=-2 -> b=0,e=-0.5; u=2.5 -> b=1,e=1
    assert bits[:, 0].tolist() == [True, True, False, True]


def test_sigma_delta_tracks_the_tile_mean():
    x = np.random.default_rng(1).standard_normal((512, 64, 128)).astype(F32) * 0.3
    bits, s = S.sigma_delta_tile(x)
    y = np.where(bits, 1.0, -1.0) * s.astype(np.float64)[:, None, :]
    err = np.abs(y.sum(1) - x.sum(1))
    # first-order loop: |sum(x - y)| = |e_t| stays within a few scale steps
    assert (err <= 4 * s.astype(np.float64) + 1e-6).mean() > 0.99


def test_pack_roundtrip():
    b = np.random.default_rng(2).random((3, 7, 128)) > 0.5
    w = S.pack_bits(b)
    assert w.shape == (3, 7, 4) and w.dtype == np.uint32
    assert np.array_equal(S.unpack_bits(w), b)
    one = np.zeros(128, bool)
    one[33] = True
    assert S.pack_bits(one).tolist() == [0, 2, 0, 0]


def test_tile_scores_equal_float_formula():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((6 * 64, 128)).astype(F32)
    enc = S.encode(x, x, 64, "hadamard")
    qp = rng.standard_normal(128).astype(F32)
    got = S.tile_scores(qp, enc["kbits"], enc["kscale"])
    b = S.unpack_bits(enc["kbits"]).astype(np.float64) * 2 - 1
    w = qp[None].astype(np.float64) * enc["kscale"].astype(np.float64)
    exact = (b * w[:, None, :]).sum(-1).max(-1)
    assert np.abs(got - exact).max() < 0.02 * np.abs(exact).max()


def test_select_rule():
    s = np.array([1.0, 5.0, 5.0, np.nan, 3.0, 7.0], F32)
    assert S.select_tiles(s, 3).tolist() == [5, 1, 2]
    assert S.select_tiles(s, 3, 5, 6).tolist() == [1, 2, 4]
    assert S.select_tiles(s, 10).tolist() == [5, 1, 2, 4, 0, 3]


def test_kernel_constants_match_spec():
    """The DCT constants baked into the CUDA sources equal the spec's."""
    src = open(os.path.join(ROOT, "rina-1bit-kv_b200", "csrc", "kvr_lee_table.h")).read()
    words = [int(w, 16) for w in re.findall(r"0x([0-9a-f]{8})u", src)]
    c0, c1, table, table_global = words[0], words[1], words[2:129], words[129:]
    f = S.lee_factors()
    flat = np.zeros(127, F32)
    for M, vals in f.items():
        flat[M // 2 - 1: M - 1] = vals
    assert table == flat.view(np.uint32).tolist() and table_global == table
    cc0, cc1 = S.dct_consts()
    assert c0 == np.array([cc0]).view(np.uint32)[0] and c1 == np.array([cc1]).view(np.uint32)[0]
    tsrc = open(os.path.join(ROOT, "rina-1bit-kv_b200", "csrc", "kvr_transform.cuh")).read()
    inv = int(re.search(r"kInvSqrt128Bits = 0x([0-9a-f]{8})u", tsrc).group(1), 16)
    assert inv == np.array([F32(1.0 / np.sqrt(128))]).view(np.uint32)[0]


def test_exclusion_range_rule():
    # kvr_hook.py:262-267 / kvr_generator.py:439-444
    from kvr_b200.kvr_hook import exclusion_range
    assert exclusion_range(1000, 512, 488) == (0, 0)   # window holds the newest, index the rest
    assert exclusion_range(600, 512, 300) == (88, 300)
    assert exclusion_range(100, 512, 0) == (0, 0)

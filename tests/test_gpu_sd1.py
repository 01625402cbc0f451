"""GPU parity of the sd1 1-bit codec against its CPU specification
(oracle/sd1_ref.py): bits, scales, transforms and tile scores bit-exact;
selection indices bit-exact; attention within the stated tolerance."""
import os

import numpy as np
import pytest
import torch

from oracle import sd1_ref as S
from oracle import int4w_ref as R

pytestmark = pytest.mark.gpu
DEV = "cuda"
F32 = np.float32


def K():
    from kvr_b200 import kernels
    return kernels


def t(x, dtype=None):
    return torch.from_numpy(np.ascontiguousarray(x)).to(DEV, dtype=dtype)


def cfg0(seed, n, n_kv=8, n_q=32, d=128, B=None):
    rng = np.random.default_rng(seed)
    scale = np.exp(rng.standard_normal((n_kv, d))).astype(F32)
    for h in range(n_kv):
        scale[h, rng.permutation(d)[:4]] *= 20
    shape = (n, n_kv, d) if B is None else (B, n, n_kv, d)
    k = (rng.standard_normal(shape) * scale).astype(F32)
    v = rng.standard_normal(shape).astype(F32)
    q = rng.standard_normal((n_q, d) if B is None else (B, n_q, d)).astype(F32)
    return k, v, q


def bits_eq(a, b):
    return np.array_equal(np.asarray(a).view(np.uint32), np.asarray(b).view(np.uint32))


@pytest.mark.parametrize("kind", ["hadamard", "dct"])
def test_transform_bit_exact(kind):
    x = np.random.default_rng(0).standard_normal((777, 128)).astype(F32) * 3
    got = K().transform(t(x), kind).cpu().numpy()
    assert bits_eq(got, S.transform(x, kind))
    inv = K().transform(t(x), kind, inverse=True).cpu().numpy()
    assert bits_eq(inv, S.transform(x, kind, inverse=True))


@pytest.mark.parametrize("tile", [32, 64, 128])
@pytest.mark.parametrize("kind", ["hadamard", "dct"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_encode_bit_exact(tile, kind, dtype):
    n = tile * 5
    k, v, q = cfg0(tile + (kind == "dct"), n, n_kv=4)
    kt, vt = t(k).to(dtype), t(v).to(dtype)
    kf, vf = kt.float().cpu().numpy(), vt.float().cpu().numpy()
    st = K().Sd1Store(1, 4, 8, tile, kind, DEV)
    K().sd1_encode(st, kt, vt)
    assert st.n_tiles == 5
    for h in range(4):
        want = S.encode(kf[:, h], vf[:, h], tile, kind)
        assert np.array_equal(st.kbits[0, h, :5].cpu().numpy().view(np.uint32), want["kbits"])
        assert np.array_equal(st.vbits[0, h, :5].cpu().numpy().view(np.uint32), want["vbits"])
        assert bits_eq(st.kscale[0, h, :5].cpu().numpy().view(np.uint16), want["kscale"].view(np.uint16))
        assert bits_eq(st.vscale[0, h, :5].cpu().numpy().view(np.uint16), want["vscale"].view(np.uint16))


@pytest.mark.parametrize("kind", ["hadamard", "dct"])
def test_encode_with_rope_and_offsets_bit_exact(kind):
    tile, n_kv = 64, 2
    k, v, q = cfg0(7, 3 * tile, n_kv=n_kv)
    cos, sin = R.rope_tables(4096, 128)
    st = K().Sd1Store(1, n_kv, 10, tile, kind, DEV)
    st.n_tiles = 4  # write at tiles 4..6, positions 1000..
    K().sd1_encode(st, t(k), t(v), cos=t(cos), sin=t(sin), pos0=1000)
    assert st.n_tiles == 7
    for h in range(n_kv):
        want = S.encode(k[:, h], v[:, h], tile, kind, cos=cos, sin=sin, pos0=1000)
        assert np.array_equal(st.kbits[0, h, 4:7].cpu().numpy().view(np.uint32), want["kbits"])
        assert np.array_equal(st.vbits[0, h, 4:7].cpu().numpy().view(np.uint32), want["vbits"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_encode_8_byte_aligned_rows_with_rope_bit_exact(dtype):
    """Token rows that start on 8- but not 16-byte boundaries take the 8-byte
    staging copies; the result is the same as for aligned rows."""
    tile, n_kv, n = 64, 2, 2 * 64
    k, v, q = cfg0(11, n, n_kv=n_kv)
    cos, sin = R.rope_tables(1024, 128)

    def skew(x):  # (n, n_kv, d) with token stride n_kv*d + 4, storage offset 4 elements
        buf = torch.zeros(n * (n_kv * 128 + 4) + 8, dtype=dtype, device=DEV)
        y = buf.as_strided((n, n_kv, 128), (n_kv * 128 + 4, 128, 1), 4)
        y.copy_(t(x).to(dtype))
        return y

    ks, vs = skew(k), skew(v)
    st = K().Sd1Store(1, n_kv, 4, tile, "dct", DEV)
    K().sd1_encode(st, ks, vs, cos=t(cos), sin=t(sin), pos0=300)
    kf, vf = ks.float().cpu().numpy(), vs.float().cpu().numpy()
    for h in range(n_kv):
        want = S.encode(kf[:, h], vf[:, h], tile, "dct", cos=cos, sin=sin, pos0=300)
        assert np.array_equal(st.kbits[0, h, :2].cpu().numpy().view(np.uint32), want["kbits"])
        assert np.array_equal(st.vbits[0, h, :2].cpu().numpy().view(np.uint32), want["vbits"])
        assert bits_eq(st.kscale[0, h, :2].cpu().numpy().view(np.uint16), want["kscale"].view(np.uint16))


def _store(seed, n_tiles, tile=64, kind="hadamard", n_kv=8, n_q=32, B=1):
    k, v, q = cfg0(seed, n_tiles * tile, n_kv=n_kv, n_q=n_q, B=B)
    st = K().Sd1Store(B, n_kv, n_tiles + 3, tile, kind, DEV)
    K().sd1_encode(st, t(k), t(v))
    return st, k, v, q


@pytest.mark.parametrize("kind,tile,g", [("hadamard", 64, 4), ("dct", 64, 4), ("dct", 32, 8), ("hadamard", 128, 1)])
def test_tile_scores_and_selection_bit_exact(kind, tile, g):
    n_kv, nt, B = 4, 40, 2
    st, k, v, q = _store(11, nt, tile, kind, n_kv=n_kv, n_q=n_kv * g, B=B)
    qb = t(q).to(torch.bfloat16)
    qf = qb.float().cpu().numpy()
    got = K().sd1_tile_scores(st, qb).cpu().numpy()
    sel, sc, qp = K().sd1_select(st, qb, 7, 3, 9)
    sel = sel.cpu().numpy()
    for b in range(B):
        qa = S.q_group_mean_f32(qf[b], n_kv)
        qprime = S.transform(qa, kind)
        for h in range(n_kv):
            kb = st.kbits[b, h, :nt].cpu().numpy().view(np.uint32)
            ks = st.kscale[b, h, :nt].cpu().numpy()
            want = S.tile_scores(qprime[h], kb, ks)
            assert bits_eq(got[b, h], want)
            assert np.array_equal(sel[b, h], S.select_tiles(want, 7, 3, 9))
        # per-head transformed queries for the attention kernel
        np.testing.assert_allclose(qp[b].cpu().numpy(), S.transform(qf[b], kind), rtol=0, atol=0)


def test_select_large_row_static_plus_dynamic_shared_memory():
    """8192 tiles in a row with k_sel 256: the selection stages the row's
    scores in shared memory and needs more than 48 KB together with the
    kernel's static shared memory; the launcher raises the limit."""
    nt, tile, k_sel = 8192, 32, 256
    rng = np.random.default_rng(9)
    k = rng.standard_normal((1, nt * tile, 1, 128)).astype(F32)
    v = rng.standard_normal(k.shape).astype(F32)
    st = K().Sd1Store(1, 1, nt, tile, "hadamard", DEV)
    K().sd1_encode(st, t(k), t(v))
    q = t(rng.standard_normal((1, 4, 128)).astype(F32))
    scores = K().sd1_tile_scores(st, q).cpu().numpy()
    sel, _, _ = K().sd1_select(st, q, k_sel, 100, 200)
    assert np.array_equal(sel.cpu().numpy()[0, 0], S.select_tiles(scores[0, 0], k_sel, 100, 200))


@pytest.mark.parametrize("kind,tile,g,B,n_kv,nt,k_sel,ex,dtype", [
    ("hadamard", 64, 4, 3, 4, 40, 7, (3, 9), torch.bfloat16),
    ("dct", 64, 4, 2, 8, 100, 16, (0, 0), torch.float32),
    ("dct", 32, 8, 2, 4, 57, 12, (50, 57), torch.float16),
    ("hadamard", 128, 1, 2, 4, 21, 40, (0, 0), torch.float32),  # k_sel > n_tiles
    ("dct", 64, 2, 5, 8, 17, 5, (2, 4), torch.bfloat16),        # ranges start mid-row, odd segments
])
def test_flat_scan_bit_exact(monkeypatch, kind, tile, g, B, n_kv, nt, k_sel, ex, dtype):
    """The flat scan (equal (row, tile) ranges, up to two rows per CTA, the CTA
    completing a row selects it) gives the oracle's selection and the same
    q' and selection as the per-row scan."""
    st, k, v, q = _store(17, nt, tile, kind, n_kv=n_kv, n_q=n_kv * g, B=B)
    qt = t(q).to(dtype)
    qf = qt.float().cpu().numpy()
    res = {}
    for scan in ("flat", "warps"):
        monkeypatch.setenv("KVR_SD1_SCAN", scan)
        res[scan] = [x.cpu().numpy() for x in K().sd1_select(st, qt, k_sel, *ex)]
    monkeypatch.delenv("KVR_SD1_SCAN")
    for a, b_ in zip(res["flat"], res["warps"]):
        assert bits_eq(a, b_) if a.dtype != np.int32 else np.array_equal(a, b_)
    sel, sc, qp = res["flat"]
    for b in range(B):
        qprime = S.transform(S.q_group_mean_f32(qf[b], n_kv), kind)
        for h in range(n_kv):
            want = S.tile_scores(qprime[h], st.kbits[b, h, :nt].cpu().numpy().view(np.uint32),
                                 st.kscale[b, h, :nt].cpu().numpy())
            exp_sel = S.select_tiles(want, k_sel, *ex)
            assert np.array_equal(sel[b, h, :len(exp_sel)], exp_sel) and (sel[b, h, len(exp_sel):] == -1).all()
            assert bits_eq(sc[b, h, :len(exp_sel)], want[exp_sel])
        np.testing.assert_allclose(qp[b], S.transform(qf[b], kind), rtol=0, atol=0)


def test_flat_scan_in_batched_decode_step():
    """At a batched shape the decode step takes the flat scan by itself; its
    selection equals the per-row scan's and the output equals the attention
    over that selection."""
    B, n_kv, g, nt, k_sel = 40, 8, 4, 240, 16  # 76800 row-tiles: 260 tiles per CTA, ranges cross rows
    st, k, v, q = _store(23, nt, 64, "dct", n_kv=n_kv, n_q=n_kv * g, B=B)
    qt = t(q).to(torch.bfloat16)
    rng = np.random.default_rng(5)
    win = t(rng.standard_normal((B, 96, n_kv, 128)).astype(np.float16))
    sel_w, _, qp = K().sd1_select(st, qt, k_sel)
    sel_f = torch.empty_like(sel_w)
    step = K().sd1_decode_step(st, qt, k_sel, win, win, 96, sel_out=sel_f)
    os.environ["KVR_SD1_SCAN"] = "warps"
    try:
        sel_ref, _, qp_ref = K().sd1_select(st, qt, k_sel)
    finally:
        del os.environ["KVR_SD1_SCAN"]
    assert torch.equal(sel_w, sel_ref) and torch.equal(sel_f, sel_ref) and torch.equal(qp, qp_ref)
    want = K().sd1_attend(st, qt, qp_ref, sel_ref, win, win, 96)
    assert torch.equal(step, want)


def test_select_more_than_available_and_empty():
    st, k, v, q = _store(3, 5)
    sel, sc, _ = K().sd1_select(st, t(q), 8)
    s = sel.cpu().numpy()
    assert (s[..., 5:] == -1).all() and (np.sort(s[..., :5], -1) == np.arange(5)).all()
    st.n_tiles = 0
    sel, _, qp = K().sd1_select(st, t(q), 4)
    assert (sel.cpu().numpy() == -1).all()


@pytest.mark.parametrize("nt,k_sel,ex", [(24, 9, (5, 11)), (7, 12, (0, 0)), (300, 16, (250, 300)), (40, 16, (0, 40))])
def test_decode_step_in_unit_selection_matches_select(nt, k_sel, ex):
    """The decode step picks tiles inside the attention units (one order
    statistic per unit); with duplicated tiles (exact score ties, broken by
    index), an exclusion range and fewer tiles than k_sel it must select
    exactly what the selection kernel selects, and attend the same."""
    tile, n_kv, g, B = 64, 4, 4, 2
    rng = np.random.default_rng(nt)
    base = rng.standard_normal((B, 4 * tile, n_kv, 128)).astype(F32)
    reps = (nt + 3) // 4
    k = np.concatenate([base] * reps, 1)[:, :nt * tile]  # tile i == tile i % 4
    v = rng.standard_normal(k.shape).astype(F32)
    st = K().Sd1Store(B, n_kv, nt + 2, tile, "dct", DEV)
    K().sd1_encode(st, t(k), t(v))
    q = t(rng.standard_normal((B, n_kv * g, 128)).astype(F32))
    win = t(rng.standard_normal((B, 70, n_kv, 128)).astype(np.float16))
    sel, _, qp = K().sd1_select(st, q, k_sel, ex_t0=ex[0], ex_t1=ex[1])
    want = K().sd1_attend(st, q, qp, sel, win, win, 70)
    for path in ("split", "cluster"):
        sel_f = torch.full_like(sel, -7)
        with K().sd1_step_path(path):
            step = K().sd1_decode_step(st, q, k_sel, win, win, 70, ex_t0=ex[0], ex_t1=ex[1], sel_out=sel_f)
        assert torch.equal(sel_f, sel), path
        if path == "split":
            assert torch.equal(step, want)
        else:  # same rows, partials merged in another order
            err = (step.float() - want.float()).abs().max() / want.float().abs().max()
            assert err < 1e-5, err


def _oracle_attend(q, st, b, h, sel_row, win_k, win_v, nw, tail_k, tail_v, ntl, kind, g):
    rows_k = [win_k[b, :nw, h].astype(np.float64), tail_k[b, :ntl, h].astype(np.float64)]
    rows_v = [win_v[b, :nw, h].astype(np.float64), tail_v[b, :ntl, h].astype(np.float64)]
    good = [s for s in sel_row if s >= 0]
    if good:
        dk = S.decode_tiles(st.kbits[b, h].cpu().numpy().view(np.uint32)[good], st.kscale[b, h].cpu().numpy()[good], kind)
        dv = S.decode_tiles(st.vbits[b, h].cpu().numpy().view(np.uint32)[good], st.vscale[b, h].cpu().numpy()[good], kind)
        rows_k.append(dk.reshape(-1, 128))
        rows_v.append(dv.reshape(-1, 128))
    return S.decode_attention(q[b, h * g:(h + 1) * g], np.concatenate(rows_k), np.concatenate(rows_v),
                              np.empty((0, 128)), np.empty((0, 128)))


@pytest.mark.parametrize("kind,tile,nw,ntl,g,B", [
    ("hadamard", 64, 512, 17, 4, 1), ("dct", 64, 256, 0, 4, 2), ("dct", 32, 100, 31, 8, 1),
    ("hadamard", 128, 0, 5, 4, 1), ("dct", 64, 1024, 63, 8, 1)])
def test_attend_vs_oracle(kind, tile, nw, ntl, g, B):
    n_kv, nt, k_sel = 4, 24, 6
    st, k, v, q = _store(21, nt, tile, kind, n_kv=n_kv, n_q=n_kv * g, B=B)
    rng = np.random.default_rng(1)
    cap = max(nw, 1) + 3
    win_k = rng.standard_normal((B, cap, n_kv, 128)).astype(np.float16)
    win_v = rng.standard_normal((B, cap, n_kv, 128)).astype(np.float16)
    tail_k = rng.standard_normal((B, tile, n_kv, 128)).astype(np.float16)
    tail_v = rng.standard_normal((B, tile, n_kv, 128)).astype(np.float16)
    qt = t(q)
    sel, _, qp = K().sd1_select(st, qt, k_sel)
    out = K().sd1_attend(st, qt, qp, sel, t(win_k), t(win_v), nw, t(tail_k), t(tail_v), ntl,
                         out_dtype=torch.float32).cpu().numpy()
    # decode_step selects the same tiles as select, on both of its paths; the
    # split path is the select + attend kernels, bit for bit
    steps = {}
    for path in ("split", "cluster", "cluster8"):
        sel_f = torch.empty_like(sel)
        with K().sd1_step_path(path):
            steps[path] = K().sd1_decode_step(st, qt, k_sel, t(win_k), t(win_v), nw, t(tail_k), t(tail_v), ntl,
                                              sel_out=sel_f).cpu().numpy()
        assert torch.equal(sel_f, sel), path
    assert np.array_equal(steps["split"], out)
    s = sel.cpu().numpy()
    for b in range(B):
        for h in range(n_kv):
            want = _oracle_attend(q, st, b, h, s[b, h], win_k, win_v, nw, tail_k, tail_v, ntl, kind, g)
            for got in (out[b, h * g:(h + 1) * g], steps["cluster"][b, h * g:(h + 1) * g],
                        steps["cluster8"][b, h * g:(h + 1) * g]):
                err = np.abs(got - want).max() / np.abs(want).max()
                assert err < 1e-5, (b, h, err)


def _batched_path_taken(B, n_kv, nw, ntl, k_sel):
    """The attention host picks the batched-rows kernel when the rows x units
    of the step exceed two CTAs per SM (296 on B200)."""
    units = -(-nw // 64) + -(-ntl // 64) + k_sel
    return B * n_kv * units > 296


@pytest.mark.parametrize("kind,tile,nw,ntl,g,B,n_kv,nt,k_sel,q_dtype", [
    ("dct", 64, 256, 17, 4, 16, 8, 24, 16, torch.bfloat16),
    ("hadamard", 32, 100, 0, 8, 12, 4, 30, 12, torch.float32),
    ("dct", 128, 200, 63, 4, 8, 8, 12, 8, torch.float16),
    ("hadamard", 64, 0, 5, 2, 32, 4, 10, 16, torch.float32),  # no window, 6 of 16 slots empty
    ("dct", 64, 512, 0, 8, 6, 8, 20, 16, torch.float32),
    ("dct", 64, 300, 1, 1, 24, 8, 20, 4, torch.float32),       # g = 1 (MHA)
])
def test_attend_batched_rows_vs_oracle(kind, tile, nw, ntl, g, B, n_kv, nt, k_sel, q_dtype):
    """Batched decode (many (b, h) rows): every lane-owned channel quad, the
    reduce-scatter of the scores, the per-warp online softmax, the parked
    exact sums and the cross-warp fold against the float64 oracle."""
    assert _batched_path_taken(B, n_kv, nw, ntl, k_sel)
    st, k, v, q = _store(31, nt, tile, kind, n_kv=n_kv, n_q=n_kv * g, B=B)
    rng = np.random.default_rng(3)
    cap = max(nw, 1) + 5
    win_k = rng.standard_normal((B, cap, n_kv, 128)).astype(np.float16)
    win_v = rng.standard_normal((B, cap, n_kv, 128)).astype(np.float16)
    tail_k = rng.standard_normal((B, tile, n_kv, 128)).astype(np.float16)
    tail_v = rng.standard_normal((B, tile, n_kv, 128)).astype(np.float16)
    qt = t(q).to(q_dtype)
    qn = qt.float().cpu().numpy()
    sel, _, qp = K().sd1_select(st, qt, k_sel)
    out = K().sd1_attend(st, qt, qp, sel, t(win_k), t(win_v), nw, t(tail_k), t(tail_v), ntl,
                         out_dtype=torch.float32).cpu().numpy()
    sel_f = torch.empty_like(sel)
    step = K().sd1_decode_step(st, qt, k_sel, t(win_k), t(win_v), nw, t(tail_k), t(tail_v), ntl,
                               sel_out=sel_f, out=torch.empty(B, n_kv * g, 128, device=DEV)).cpu().numpy()
    assert torch.equal(sel_f, sel)
    assert np.array_equal(step, out)
    s = sel.cpu().numpy()
    assert (s < 0).any() == (nt < k_sel)
    worst = 0.0
    for b in range(B):
        for h in range(n_kv):
            want = _oracle_attend(qn, st, b, h, s[b, h], win_k, win_v, nw, tail_k, tail_v, ntl, kind, g)
            got = out[b, h * g:(h + 1) * g]
            worst = max(worst, np.abs(got - want).max() / np.abs(want).max())
    assert worst < 1e-5, worst


@pytest.mark.parametrize("kind,tile,g,out_dtype", [("dct", 64, 4, torch.bfloat16), ("hadamard", 32, 8, torch.float16)])
def test_attend_batched_rows_16bit_output_vs_oracle(kind, tile, g, out_dtype):
    """16-bit outputs on the batched path (for bf16 the P.V products take only
    the fp16 high part of P: the output's own rounding is far coarser):
    relative error (norm of the group's rows) within 2e-3 of the float64
    oracle, and elementwise the fp32-output result rounded to the output type,
    up to half an ulp of that type plus 5e-4 of the row maximum."""
    B, n_kv, nt, k_sel, nw, ntl = 16, 8, 24, 16, 256, 9
    assert _batched_path_taken(B, n_kv, nw, ntl, k_sel)
    st, k, v, q = _store(41, nt, tile, kind, n_kv=n_kv, n_q=n_kv * g, B=B)
    rng = np.random.default_rng(8)
    win_k = rng.standard_normal((B, nw + 4, n_kv, 128)).astype(np.float16)
    win_v = rng.standard_normal((B, nw + 4, n_kv, 128)).astype(np.float16)
    tail_k = rng.standard_normal((B, tile, n_kv, 128)).astype(np.float16)
    tail_v = rng.standard_normal((B, tile, n_kv, 128)).astype(np.float16)
    qt = t(q).to(torch.bfloat16)
    qn = qt.float().cpu().numpy()
    sel, _, qp = K().sd1_select(st, qt, k_sel)
    args = (st, qt, qp, sel, t(win_k), t(win_v), nw, t(tail_k), t(tail_v), ntl)
    out = K().sd1_attend(*args, out_dtype=out_dtype).float().cpu().numpy()
    full = K().sd1_attend(*args, out_dtype=torch.float32).cpu().numpy()
    half_ulp = np.abs(full) * (2.0 ** -8 if out_dtype == torch.bfloat16 else 2.0 ** -11)
    assert (np.abs(out - full) <= half_ulp + 5e-4 * np.abs(full).max(-1, keepdims=True)).all()
    s = sel.cpu().numpy()
    worst = 0.0
    for b in range(B):
        for h in range(n_kv):
            want = _oracle_attend(qn, st, b, h, s[b, h], win_k, win_v, nw, tail_k, tail_v, ntl, kind, g)
            got = out[b, h * g:(h + 1) * g]
            worst = max(worst, np.linalg.norm(got - want) / np.linalg.norm(want))
    assert worst < 2e-3, worst


def test_attend_batched_rows_partial_merge_like_whole():
    """Sequence split on the batched path: two halves of the selection as
    partial rows, merged by kvr_lse_merge, equal the whole attention."""
    B, n_kv, g = 16, 8, 4
    st, k, v, q = _store(7, 30, n_kv=n_kv, n_q=n_kv * g, B=B)
    assert _batched_path_taken(B, n_kv, 0, 0, 16)
    qt = t(q)
    sel, _, qp = K().sd1_select(st, qt, 16)
    whole = K().sd1_attend(st, qt, qp, sel, out_dtype=torch.float32)
    a, b = sel.clone(), sel.clone()
    a[..., 8:] = -1
    b[..., :8] = -1
    pa = K().sd1_attend(st, qt, qp, a, partial=True)
    pb = K().sd1_attend(st, qt, qp, b, partial=True)
    for bi in range(B):
        merged = K().lse_merge(torch.stack([pa[bi], pb[bi]]))
        np.testing.assert_allclose(merged.cpu().numpy(), whole[bi].cpu().numpy(), rtol=1e-5, atol=1e-6)


def test_partial_rows_merge_like_whole():
    """Sequence split: two halves of the selection -> partials -> kvr_lse_merge."""
    st, k, v, q = _store(5, 30, n_kv=8, n_q=32)
    qt = t(q)
    sel, _, qp = K().sd1_select(st, qt, 8)
    whole = K().sd1_attend(st, qt, qp, sel, out_dtype=torch.float32)
    a, b = sel.clone(), sel.clone()
    a[..., 4:] = -1
    b[..., :4] = -1
    pa = K().sd1_attend(st, qt, qp, a, partial=True)
    pb = K().sd1_attend(st, qt, qp, b, partial=True)
    merged = K().lse_merge(torch.stack([pa[0], pb[0]]))
    np.testing.assert_allclose(merged.cpu().numpy(), whole[0].cpu().numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("kind", ["hadamard", "dct"])
def test_decode_tiles_vs_oracle(kind):
    st, k, v, q = _store(9, 12, kind=kind, n_kv=2, n_q=8)
    sel = torch.tensor([[[3, 0, 11], [5, -1, 2]]], device=DEV)
    dk, dv = K().sd1_decode_tiles(st, sel)
    dk, dv = dk.cpu().numpy(), dv.float().cpu().numpy()
    for h in range(2):
        for j, s in enumerate(sel[0, h].tolist()):
            rows = slice(j * 64, (j + 1) * 64)
            if s < 0:
                assert (dk[0, rows, h] == 0).all()
                continue
            wk = S.decode_tiles(st.kbits[0, h, [s]].cpu().numpy().view(np.uint32), st.kscale[0, h, [s]].cpu().numpy(), kind)[0]
            np.testing.assert_allclose(dk[0, rows, h], wk, rtol=1e-5, atol=1e-5 * np.abs(wk).max())


def test_full_size_config1_layer_sampled_parity():
    """Config-1 shape (T = 32768 - 512 stored tokens, 8 heads, tile 64, DCT):
    encode on the GPU, check 16 random tiles bit-exactly against the oracle and
    the selection of every head against the oracle's scores."""
    n_kv, tile, T = 8, 64, 32256
    k, v, q = cfg0(1234, T, n_kv=n_kv)
    kb16, vb16 = t(k).to(torch.bfloat16), t(v).to(torch.bfloat16)
    st = K().Sd1Store(1, n_kv, T // tile, tile, "dct", DEV)
    K().sd1_encode(st, kb16, vb16)
    kf = kb16.float().cpu().numpy()
    vf = vb16.float().cpu().numpy()
    rng = np.random.default_rng(0)
    for ti in rng.choice(T // tile, 16, replace=False):
        h = int(rng.integers(n_kv))
        rows = slice(ti * tile, (ti + 1) * tile)
        want = S.encode(kf[rows, h], vf[rows, h], tile, "dct")
        assert np.array_equal(st.kbits[0, h, ti].cpu().numpy().view(np.uint32), want["kbits"][0])
        assert np.array_equal(st.vscale[0, h, ti].cpu().numpy().view(np.uint16), want["vscale"][0].view(np.uint16))
    qb = t(q).to(torch.bfloat16)
    sel, _, _ = K().sd1_select(st, qb, 16)
    qa = S.q_group_mean_f32(qb.float().cpu().numpy(), n_kv)
    qp = S.transform(qa, "dct")
    for h in range(n_kv):
        want = S.tile_scores(qp[h], st.kbits[0, h].cpu().numpy().view(np.uint32), st.kscale[0, h].cpu().numpy())
        assert np.array_equal(sel[0, h].cpu().numpy(), S.select_tiles(want, 16))


@pytest.mark.parametrize("g,k_sel,nw,ntl,ex", [(4, 16, 512, 0, (0, 0)), (4, 32, 512, 40, (500, 504)),
                                               (8, 16, 1024, 63, (0, 3)), (2, 8, 256, 1, (0, 0)),
                                               (1, 1, 96, 0, (0, 0))])
def test_cluster_step_config1_layer(g, k_sel, nw, ntl, ex):
    """Config-1 layer (504 tiles of 64 per head, 8 KV heads, DCT, bf16 q):
    the one-kernel cluster step selects exactly the oracle's tiles and its
    output matches the split path (select + attend kernels) and the exact
    softmax over the same rows."""
    n_kv, tile, T = 8, 64, 504 * 64
    k, v, q = cfg0(77 + g, T, n_kv=n_kv, n_q=n_kv * g)
    st = K().Sd1Store(1, n_kv, T // tile, tile, "dct", DEV)
    K().sd1_encode(st, t(k).to(torch.bfloat16), t(v).to(torch.bfloat16))
    rng = np.random.default_rng(g)
    win_k = rng.standard_normal((1, nw, n_kv, 128)).astype(np.float16)
    win_v = rng.standard_normal((1, nw, n_kv, 128)).astype(np.float16)
    tail_k = rng.standard_normal((1, tile, n_kv, 128)).astype(np.float16)
    tail_v = rng.standard_normal((1, tile, n_kv, 128)).astype(np.float16)
    qb = t(q[None]).to(torch.bfloat16)
    outs, sels = {}, {}
    for path in ("split", "cluster", "cluster8"):
        sels[path] = torch.full((1, n_kv, k_sel), -7, dtype=torch.int32, device=DEV)
        with K().sd1_step_path(path):
            outs[path] = K().sd1_decode_step(st, qb, k_sel, t(win_k), t(win_v), nw, t(tail_k), t(tail_v), ntl,
                                             ex_t0=ex[0], ex_t1=ex[1], sel_out=sels[path]).float().cpu().numpy()
    assert torch.equal(sels["split"], sels["cluster"]) and torch.equal(sels["split"], sels["cluster8"])
    qa = S.q_group_mean_f32(qb.float().cpu().numpy()[0], n_kv)
    qp = S.transform(qa, "dct")
    s = sels["cluster"].cpu().numpy()
    for h in range(n_kv):
        sc = S.tile_scores(qp[h], st.kbits[0, h].cpu().numpy().view(np.uint32), st.kscale[0, h].cpu().numpy())
        sc[ex[0]:ex[1]] = -np.inf
        assert np.array_equal(s[0, h], S.select_tiles(sc, k_sel)), h
    qf = qb.float().cpu().numpy()
    for h in range(n_kv):
        want = _oracle_attend(qf, st, 0, h, s[0, h], win_k, win_v, nw, tail_k, tail_v, ntl, "dct", g)
        for path in ("split", "cluster", "cluster8"):
            got = outs[path][0, h * g:(h + 1) * g]
            err = np.linalg.norm(got - want) / np.linalg.norm(want)
            assert err < 2e-3, (path, h, err)  # bf16 output: norm-relative, as the batched 16-bit test


def test_retrieval_index_sd1_api():
    from kvr_b200 import RetrievalIndex, WindowBuffer
    n_kv, tile = 2, 64
    k, v, q = cfg0(4, 1000, n_kv=n_kv, n_q=8)
    cos, sin = R.rope_tables(2048, 128)
    ri = RetrievalIndex(n_kv, 128, top_k=256, device=DEV, codec="sd1", tile=tile, transform="dct")
    ri.set_rotary_tables(t(cos), t(sin))
    ri.calibrate(t(k[:900]), t(v[:900]))
    ri.batch_append(t(k[:900]), t(v[:900]))
    assert (ri.n_stored, ri.n_tail) == (896, 4)
    for i in range(900, 1000):
        ri.append(t(k[i]), t(v[i]))
    assert ri.n_tokens == 1000 and ri.n_stored == 960 and ri.n_tail == 40
    # encoded tiles equal the oracle's encoding of the RoPE'd stream
    for h in range(n_kv):
        want = S.encode(k[:960, h], v[:960, h], tile, "dct", cos=cos, sin=sin, pos0=0)
        got = ri.store.kbits[0, h, :15].cpu().numpy().view(np.uint32)
        # tiles that passed through the fp16 tail were rounded to fp16 first
        assert np.array_equal(got[:14], want["kbits"][:14])
    rk, rv = ri.retrieve_topk(t(q), n_q=8)
    assert rk.shape == (4 * tile + 40, n_kv, 128) and rv.dtype == torch.float16
    wb = WindowBuffer(n_kv, 128, 128, DEV)
    wb.batch_append(t(k[:128]), t(v[:128]))
    out = ri.attend(t(q), wb)
    want = K().decode_attn(t(q), [(wb.k, wb.v), (rk, rv)], out_dtype=torch.float32)
    # the API returns V in fp16 (reference format), the fused path keeps it exact
    np.testing.assert_allclose(out.cpu().numpy(), want.cpu().numpy(), rtol=3e-3, atol=3e-3)


def test_bounded_wait_runs_out_and_is_reported():
    """The kernels' bounded mbarrier wait, made to run out on purpose (a
    phase that never completes, a short poll limit): the kernel returns,
    kvr_workspace_status reports KVR_ETIMEOUT once and clears it, and the
    same context keeps working."""
    from kvr_b200 import _native as N
    ws = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    N.call("kvr_selftest_bounded_wait", N.ptr(ws), 256, N.stream())
    with pytest.raises(N.KvrError, match="KVR_ETIMEOUT"):
        N.call("kvr_workspace_status", N.ptr(ws), N.stream())
    N.call("kvr_workspace_status", N.ptr(ws), N.stream())  # cleared: no error now
    q = torch.randn(8, 128, device="cuda")
    k = torch.randn(100, 2, 128, device="cuda").half()
    out = K().decode_attn(q, [(k, k)], out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()

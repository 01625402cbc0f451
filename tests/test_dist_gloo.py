"""Sequence-split orchestration on CPU with two gloo ranks: candidate
all-gather + global top-k (kvr_b200.sharding.global_selection) and the
log-sum-exp merge of partial attention rows reproduce the single-process
result exactly; a rank that fails before a collective is detected by the
other through a short process-group timeout (no GPU involved)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import sd1_ref as S

TILE, NT, K_SEL, G = 64, 37, 6, 4


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _problem():
    rng = np.random.default_rng(5)
    k = rng.standard_normal((NT * TILE, 128)).astype(np.float32)
    v = rng.standard_normal((NT * TILE, 128)).astype(np.float32)
    q = rng.standard_normal((G, 128)).astype(np.float32)
    win = rng.standard_normal((50, 128)).astype(np.float32)
    enc = S.encode(k, v, TILE, "hadamard")
    qp = S.transform(S.q_group_mean_f32(q, 1), "hadamard")[0]
    scores = S.tile_scores(qp, enc["kbits"], enc["kscale"])
    return enc, q, win, scores


def _partial(q, kk, vv):
    """Unnormalised (m, l, o) rows of q over rows kk/vv (float64)."""
    if len(kk) == 0:
        return np.concatenate([np.full((len(q), 1), -np.inf), np.zeros((len(q), 129))], 1)
    s = q.astype(np.float64) @ kk.T / np.sqrt(128)
    m = s.max(1, keepdims=True)
    p = np.exp(s - m)
    return np.concatenate([m, p.sum(1, keepdims=True), p @ vv], 1)


def _merge(parts):
    m = parts[:, :, 0].max(0)
    w = np.where(np.isinf(parts[:, :, 0]), 0.0, np.exp(parts[:, :, 0] - m))
    return (w[..., None] * parts[:, :, 2:]).sum(0) / (w * parts[:, :, 1]).sum(0)[:, None]


def _worker(rank, world, port, mode, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from kvr_b200.sharding import TorchDistComm, global_selection, tile_ranges

    comm = TorchDistComm()
    try:
        if mode == "fail" and rank == 1:
            raise RuntimeError("rank 1 failed before the collective")
        enc, q, win, scores = _problem()
        base, n = tile_ranges(NT, world)[rank]
        loc = S.select_tiles(scores[base:base + n], K_SEL)
        sc = torch.full((1, 1, K_SEL), float("-inf"))
        ix = torch.full((1, 1, K_SEL), -1, dtype=torch.int64)
        sc[0, 0, :len(loc)] = torch.from_numpy(scores[base + loc].astype(np.float32))
        ix[0, 0, :len(loc)] = torch.from_numpy(base + loc)
        gsel = global_selection(torch.stack(comm.all_gather(sc)), torch.stack(comm.all_gather(ix)), K_SEL)[0, 0]
        owned = [int(t) for t in gsel if base <= t < base + n]
        dk = S.decode_tiles(enc["kbits"][owned], enc["kscale"][owned], "hadamard").reshape(-1, 128)
        dv = S.decode_tiles(enc["vbits"][owned], enc["vscale"][owned], "hadamard").reshape(-1, 128)
        if rank == world - 1:
            dk, dv = np.concatenate([win, dk]), np.concatenate([win, dv])
        part = torch.from_numpy(_partial(q, dk, dv))
        merged = _merge(torch.stack(comm.all_gather(part)).numpy())
        results[rank] = (gsel.numpy(), merged)
    except Exception as e:  # noqa: BLE001 - reported to the parent
        results[rank] = ("error", repr(e))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(mode, world=2):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        res = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, world, port, mode, res)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(60)
            if p.is_alive():
                p.kill()
                pytest.fail("gloo rank hung")
        return dict(res)


def test_seq_split_matches_single_process():
    res = _run("ok")
    enc, q, win, scores = _problem()
    want_sel = S.select_tiles(scores, K_SEL)
    dk = S.decode_tiles(enc["kbits"][want_sel], enc["kscale"][want_sel], "hadamard").reshape(-1, 128)
    dv = S.decode_tiles(enc["vbits"][want_sel], enc["vscale"][want_sel], "hadamard").reshape(-1, 128)
    want = S.decode_attention(q, win, win, dk, dv)
    for r in range(2):
        assert not isinstance(res[r][0], str), res[r]
        assert np.array_equal(res[r][0], want_sel)
        np.testing.assert_allclose(res[r][1], want, rtol=1e-9, atol=1e-9)


def test_failed_rank_is_detected_by_the_other():
    res = _run("fail")
    assert res[1][0] == "error" and "rank 1 failed" in res[1][1]
    assert res[0][0] == "error"  # the surviving rank's collective ends with an error, it does not hang


def test_global_selection_tie_rule():
    from kvr_b200.sharding import global_selection
    sc = torch.tensor([[[[5.0, 3.0, float("-inf")]]], [[[5.0, 4.0, 3.0]]]])
    ix = torch.tensor([[[[9, 2, -1]]], [[[4, 7, 1]]]])
    assert global_selection(sc, ix, 4)[0, 0].tolist() == [4, 9, 7, 1]
    assert global_selection(sc, ix, 6)[0, 0].tolist() == [4, 9, 7, 1, 2, -1]


def test_tile_ranges_and_head_shard():
    from kvr_b200.sharding import head_shard, tile_ranges
    assert tile_ranges(10, 3) == [(0, 4), (4, 3), (7, 3)]
    assert head_shard(8, 32, 1, 4) == (slice(2, 4), slice(8, 16))
    with pytest.raises(ValueError):
        head_shard(8, 32, 0, 3)


# ---- SeqSplitDecoder.step itself, with the per-rank GPU work done by the oracle


class _OracleSplit:
    """Stands in for the GPU parts of SeqSplitDecoder (local selection,
    partial attention, merge) with the sd1 oracle, so that the class's own
    exchange logic runs on gloo ranks."""

    @staticmethod
    def make(rank, world, nt, k_sel, comm):
        from kvr_b200.sharding import SeqSplitDecoder, tile_ranges

        rng = np.random.default_rng(11)
        k = rng.standard_normal((nt * TILE, 128)).astype(np.float32)
        v = rng.standard_normal((nt * TILE, 128)).astype(np.float32)
        enc = S.encode(k, v, TILE, "hadamard")
        base, n = tile_ranges(nt, world)[rank]

        class Dec(SeqSplitDecoder):
            def local_candidates(self, q, kk):
                qp = S.transform(S.q_group_mean_f32(q[0].numpy(), 1), "hadamard")[0]
                scores = S.tile_scores(qp, enc["kbits"][base:base + n], enc["kscale"][base:base + n]) if n else []
                loc = S.select_tiles(np.asarray(scores, np.float32), min(kk, n)) if n else np.zeros(0, np.int64)
                sc = torch.full((1, 1, kk), float("-inf"))
                ix = torch.full((1, 1, kk), -1, dtype=torch.int32)
                sc[0, 0, :len(loc)] = torch.from_numpy(np.asarray(scores, np.float32)[loc])
                ix[0, 0, :len(loc)] = torch.from_numpy((base + loc).astype(np.int32))
                return ix, sc, None

            def n_local_tiles(self):
                return n

            def local_partial(self, q, qp, local_sel):
                owned = [base + int(t) for t in local_sel[0, 0] if t >= 0]
                dk = S.decode_tiles(enc["kbits"][owned], enc["kscale"][owned], "hadamard").reshape(-1, 128)
                dv = S.decode_tiles(enc["vbits"][owned], enc["vscale"][owned], "hadamard").reshape(-1, 128)
                return torch.from_numpy(_partial(q[0].numpy(), dk, dv)).unsqueeze(0)

            def merge(self, parts, out_dtype):
                return torch.from_numpy(_merge(parts.numpy()))

            def select_global(self, all_sc, all_idx, kk):
                from kvr_b200.sharding import global_selection
                g = global_selection(all_sc, all_idx.long(), kk)
                loc = g - base
                mine = (g >= 0) & (loc >= 0) & (loc < n)
                return torch.where(mine, loc, torch.full_like(loc, -1)), g

        return Dec(None, base, comm), enc


def _split_worker(rank, world, port, nt, k_sel, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    from kvr_b200.sharding import TorchDistComm

    try:
        dec, _ = _OracleSplit.make(rank, world, nt, k_sel, TorchDistComm())
        q = torch.from_numpy(np.random.default_rng(3).standard_normal((1, G, 128)).astype(np.float32))
        out, gsel = dec.step(q, k_sel)
        results[rank] = (gsel[0, 0].numpy(), out[0].numpy())
    except Exception as e:  # noqa: BLE001 - reported to the parent
        results[rank] = ("error", repr(e))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("nt,world", [(9, 2), (5, 3), (2, 3)])
def test_seq_split_decoder_with_fewer_tiles_than_k(nt, world):
    """Ranks owning fewer than k_sel tiles (uneven, or none at all) still pass
    equal shapes to the all-gathers, and the result equals the one-process
    selection and attention."""
    k_sel = 6
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        res = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_split_worker, args=(r, world, port, nt, k_sel, res)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(90)
            if p.is_alive():
                p.kill()
                pytest.fail("gloo rank hung")
        res = dict(res)
    rng = np.random.default_rng(11)
    k = rng.standard_normal((nt * TILE, 128)).astype(np.float32)
    v = rng.standard_normal((nt * TILE, 128)).astype(np.float32)
    enc = S.encode(k, v, TILE, "hadamard")
    q = np.random.default_rng(3).standard_normal((G, 128)).astype(np.float32)
    qp = S.transform(S.q_group_mean_f32(q, 1), "hadamard")[0]
    want_sel = S.select_tiles(S.tile_scores(qp, enc["kbits"], enc["kscale"]), min(k_sel, nt))
    dk = S.decode_tiles(enc["kbits"][want_sel], enc["kscale"][want_sel], "hadamard").reshape(-1, 128)
    dv = S.decode_tiles(enc["vbits"][want_sel], enc["vscale"][want_sel], "hadamard").reshape(-1, 128)
    want = _merge(_partial(q, dk, dv)[None])
    for r in range(world):
        assert not isinstance(res[r][0], str), res[r]
        got_sel = res[r][0]
        assert np.array_equal(got_sel[:len(want_sel)], want_sel)
        assert np.all(got_sel[len(want_sel):] == -1)
        np.testing.assert_allclose(res[r][1], want, rtol=1e-9, atol=1e-9)

"""Sequence split of the sd1 decode step on the GPU: two ranks' stores, the
candidate exchange, partial attention on owned tiles and the log-sum-exp merge
reproduce the single-store step (selection bit-exact, output within 1e-5).
On one GPU the two ranks run in two threads over a barrier-based exchange;
with two or more GPUs the same code runs as two processes over NCCL."""
import datetime
import os
import socket
import threading

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NT, TILE, K_SEL, NKV, NQ = 61, 64, 12, 4, 16


class ThreadComm:
    """all_gather between threads of one process (test double of TorchDistComm)."""

    def __init__(self, world):
        self.world = world
        self.slots = [None] * world
        self.bar = threading.Barrier(world)

    def view(self, rank):
        comm = self

        class V:
            def all_gather(self, t):
                torch.cuda.synchronize()
                comm.slots[rank] = t.clone()
                comm.bar.wait()
                out = [s.clone() for s in comm.slots]
                comm.bar.wait()
                return out

        return V()


def _setup(dev, seed=3):
    from kvr_b200 import kernels as K
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(1, NT * TILE, NKV, 128, device=dev, generator=g)
    v = torch.randn(1, NT * TILE, NKV, 128, device=dev, generator=g)
    q = torch.randn(1, NQ, 128, device=dev, generator=g)
    win = torch.randn(1, 200, NKV, 128, device=dev, generator=g).half()
    full = K.Sd1Store(1, NKV, NT, TILE, "dct", dev)
    K.sd1_encode(full, k, v)
    return k, v, q, win, full


def _ref(full, q, win):
    from kvr_b200 import kernels as K
    sel, _, qp = K.sd1_select(full, q, K_SEL)
    out = K.sd1_attend(full, q, qp, sel, win, win, 200, out_dtype=torch.float32)
    return sel, out


def _rank_store(k, v, rank, world, dev):
    from kvr_b200 import kernels as K
    from kvr_b200.sharding import tile_ranges
    base, n = tile_ranges(NT, world)[rank]
    st = K.Sd1Store(1, NKV, n, TILE, "dct", dev)
    K.sd1_encode(st, k[:, base * TILE:(base + n) * TILE].contiguous(), v[:, base * TILE:(base + n) * TILE].contiguous())
    return st, base


def test_seq_split_two_ranks_one_gpu():
    from kvr_b200.sharding import SeqSplitDecoder
    k, v, q, win, full = _setup("cuda")
    want_sel, want = _ref(full, q, win)
    comm = ThreadComm(2)
    decs = []
    for r in range(2):
        st, base = _rank_store(k, v, r, 2, "cuda")
        decs.append(SeqSplitDecoder(st, base, comm.view(r), window=(win, win) if r == 1 else None,
                                    n_win=200 if r == 1 else 0))
    res = [None, None]

    def run(r):
        res[r] = decs[r].step(q, K_SEL, out_dtype=torch.float32)

    th = [threading.Thread(target=run, args=(r,)) for r in range(2)]
    for t in th:
        t.start()
    for t in th:
        t.join(120)
    for r in range(2):
        out, gsel = res[r]
        assert torch.equal(gsel.to(torch.int32), want_sel)
        err = (out - want).abs().max() / want.abs().max()
        assert err < 1e-5, err
    # and both against the CPU specification (selection exact, attention 1e-5)
    from oracle import sd1_ref as S
    kc, vc, qc, wc = k[0].cpu().numpy(), v[0].cpu().numpy(), q[0].cpu().numpy(), win[0].float().cpu().numpy()
    qp = S.transform(S.q_group_mean_f32(qc, NKV), "dct")
    g = NQ // NKV
    for h in range(NKV):
        enc = S.encode(kc[:, h], vc[:, h], TILE, "dct")
        sel_h = S.select_tiles(S.tile_scores(qp[h], enc["kbits"], enc["kscale"]), K_SEL)
        assert np.array_equal(res[0][1][0, h].cpu().numpy(), sel_h)
        dk = S.decode_tiles(enc["kbits"][sel_h], enc["kscale"][sel_h], "dct").reshape(-1, 128)
        dv = S.decode_tiles(enc["vbits"][sel_h], enc["vscale"][sel_h], "dct").reshape(-1, 128)
        ref_h = S.decode_attention(qc[h * g:(h + 1) * g], wc[:, h], wc[:, h], dk, dv)
        got_h = res[0][0][0, h * g:(h + 1) * g].cpu().numpy()
        assert np.abs(got_h - ref_h).max() <= 1e-5 * np.abs(ref_h).max()


def test_merge_candidates_matches_global_selection():
    """kvr_merge_candidates against the torch restatement of the rule (score
    desc, index asc; -1 / -inf / NaN are not candidates), with ties, empty
    slots and uneven ownership."""
    from kvr_b200 import kernels as K
    from kvr_b200.sharding import global_selection
    g = torch.Generator().manual_seed(0)
    for N_, B, H, kl, k_sel in [(2, 1, 8, 16, 16), (4, 2, 8, 32, 32), (8, 1, 8, 32, 32), (3, 3, 2, 5, 9)]:
        sc = torch.randint(-4, 5, (N_, B, H, kl), generator=g).float() / 4  # many ties
        ix = torch.randperm(N_ * kl * 4, generator=g)[:N_ * kl].view(N_, 1, 1, kl).expand(N_, B, H, kl).clone()
        drop = torch.rand(N_, B, H, kl, generator=g) < 0.2
        ix[drop] = -1
        sc[torch.rand(N_, B, H, kl, generator=g) < 0.05] = float("nan")
        sc[torch.rand(N_, B, H, kl, generator=g) < 0.05] = float("-inf")
        want = global_selection(sc, ix, k_sel).to(torch.int32)
        base, n_loc = 7, 40
        gsel, lsel = K.merge_candidates(sc.cuda(), ix.to(torch.int32).cuda(), k_sel, base, n_loc)
        assert torch.equal(gsel.cpu(), want)
        loc = want - base
        want_l = torch.where((want >= 0) & (loc >= 0) & (loc < n_loc), loc, torch.full_like(loc, -1))
        assert torch.equal(lsel.cpu(), want_l)


def test_peer_exchange_single_rank_and_graph_replay():
    """PeerComm on one rank (the exchange kernels store into and read from
    this GPU's buffer): the split decoder equals the single-store step, over
    repeated exchanges (epochs advance) and from a replayed CUDA graph."""
    from kvr_b200.sharding import PeerComm, SeqSplitDecoder
    k, v, q, win, full = _setup("cuda")
    want_sel, want = _ref(full, q, win)
    comm = PeerComm.local()
    try:
        dec = SeqSplitDecoder(full, 0, comm, window=(win, win), n_win=200)
        for _ in range(3):
            out, gsel = dec.step(q, K_SEL, out_dtype=torch.float32)
            torch.cuda.synchronize()
            assert torch.equal(gsel, want_sel)
            assert float((out - want).abs().max() / want.abs().max()) < 1e-5
        res = {}
        st = torch.cuda.Stream()
        with torch.cuda.stream(st):
            dec.step(q, K_SEL, out_dtype=torch.float32)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            res["out"], res["sel"] = dec.step(q, K_SEL, out_dtype=torch.float32)
        for _ in range(3):
            gr.replay()
            torch.cuda.synchronize()
            assert torch.equal(res["sel"], want_sel)
            assert float((res["out"] - want).abs().max() / want.abs().max()) < 1e-5
        comm.status()
    finally:
        comm.close()


def _nccl_worker(rank, world, port, q_path, use_peer=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from kvr_b200.sharding import PeerComm, SeqSplitDecoder, TorchDistComm
    dev = f"cuda:{rank}"
    k, v, q, win, full = _setup(dev)
    st, base = _rank_store(k, v, rank, world, dev)
    comm = PeerComm() if use_peer else TorchDistComm()
    dec = SeqSplitDecoder(st, base, comm, window=(win, win) if rank == world - 1 else None,
                          n_win=200 if rank == world - 1 else 0)
    want_sel, want = _ref(full, q, win)
    ok = True
    for _ in range(3 if use_peer else 1):
        out, gsel = dec.step(q, K_SEL, out_dtype=torch.float32)
        torch.cuda.synchronize()
        ok = ok and torch.equal(gsel.to(torch.int32), want_sel)
        ok = ok and float((out - want).abs().max() / want.abs().max()) < 1e-5
    if use_peer:
        comm.status()
    if rank == 0:
        torch.save({"ok": ok}, q_path)
    dist.barrier()
    if use_peer:
        comm.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_seq_split_nccl_two_gpus(tmp_path):
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    path = str(tmp_path / "r.pt")
    mp.spawn(_nccl_worker, args=(2, port, path), nprocs=2, join=True)
    assert torch.load(path)["ok"]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_seq_split_peer_exchange_two_gpus(tmp_path):
    """The NVLink peer-memory exchanges (PeerComm) across two GPUs, three steps."""
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    path = str(tmp_path / "r.pt")
    mp.spawn(_nccl_worker, args=(2, port, path, True), nprocs=2, join=True)
    assert torch.load(path)["ok"]

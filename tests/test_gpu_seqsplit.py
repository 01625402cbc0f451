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


def _nccl_worker(rank, world, port, q_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from kvr_b200.sharding import SeqSplitDecoder, TorchDistComm
    dev = f"cuda:{rank}"
    k, v, q, win, full = _setup(dev)
    st, base = _rank_store(k, v, rank, world, dev)
    dec = SeqSplitDecoder(st, base, TorchDistComm(), window=(win, win) if rank == world - 1 else None,
                          n_win=200 if rank == world - 1 else 0)
    out, gsel = dec.step(q, K_SEL, out_dtype=torch.float32)
    if rank == 0:
        want_sel, want = _ref(full, q, win)
        ok = torch.equal(gsel.to(torch.int32), want_sel) and float((out - want).abs().max() / want.abs().max()) < 1e-5
        torch.save({"ok": ok}, q_path)
    dist.barrier()
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

"""Multi-GPU partitioning of the sd1 decode path (one process per GPU).

Head sharding (``head_shard``): the KV heads are independent in sd1, so rank r
owns heads [r*H/N, (r+1)*H/N) with their query groups and runs the one-GPU
decode step on them; there is no collective on the data path.

Sequence split (``SeqSplitDecoder``) for very long contexts: rank r owns the
tiles [tile_base_r, tile_base_r + n_r) of every head, the last rank also owns
the window and the pending tail.  One decode step is
  1. local selection: each rank scores its tiles and keeps its local top k
     (score, global tile index) per (b, h);
  2. all-gather of the candidates (N*B*H*k pairs — a few KB); every rank
     derives the same global top k, which is exact because the global top k
     is contained in the union of the local ones (ties: score desc, tile asc);
  3. each rank attends the selected tiles it owns (+ the window on the last
     rank) and emits log-sum-exp partial rows (m, l, o);
  4. all-gather of the partial rows and a local merge (kvr_lse_merge).
The global top k of step 2 is one kernel (kvr_merge_candidates) that also
writes the rank's own slice of the selection as local tile indices.
The exchanges use either a communicator with ``all_gather(tensor) -> list``
(``TorchDistComm``: torch.distributed, NCCL on the GPU box, gloo in the CPU
tests) or ``PeerComm``: one kernel per exchange that stores this rank's rows
into every rank's buffer over NVLink and merges locally (kvr_peer_*).  Either
way remote data lands in local memory before any kernel reads it; no kernel
loads from a peer's memory.
"""
from __future__ import annotations

import torch

from . import kernels as K


def head_shard(n_kv: int, n_q: int, rank: int, world: int):
    """(kv_head_slice, q_head_slice) owned by `rank`."""
    if n_kv % world:
        raise ValueError(f"{n_kv} KV heads do not split over {world} ranks")
    hk = n_kv // world
    g = n_q // n_kv
    return slice(rank * hk, (rank + 1) * hk), slice(rank * hk * g, (rank + 1) * hk * g)


def tile_ranges(n_tiles: int, world: int):
    """Contiguous, balanced tile ranges [(base, count)] per rank."""
    per, extra = divmod(n_tiles, world)
    out, base = [], 0
    for r in range(world):
        n = per + (1 if r < extra else 0)
        out.append((base, n))
        base += n
    return out


def global_selection(scores: torch.Tensor, idx: torch.Tensor, k: int):
    """scores, idx: (N, B, H, k_local) candidates of N ranks (idx < 0 = none).
    Returns (B, H, k) global tile indices ordered by (score desc, index asc),
    -1 where fewer than k candidates exist."""
    N, B, H, kl = scores.shape
    s = scores.permute(1, 2, 0, 3).reshape(B, H, N * kl).float()
    i = idx.permute(1, 2, 0, 3).reshape(B, H, N * kl).long()
    s = torch.where(i < 0, torch.full_like(s, float("-inf")), s)
    s = torch.where(torch.isnan(s), torch.full_like(s, float("-inf")), s)
    big = torch.iinfo(torch.int64).max
    i_key = torch.where(i < 0, torch.full_like(i, big), i)
    o1 = torch.argsort(i_key, dim=-1, stable=True)           # index ascending
    s1 = torch.gather(s, -1, o1)
    o2 = torch.argsort(-s1, dim=-1, stable=True)              # then score descending
    order = torch.gather(o1, -1, o2)[..., :k]
    sel = torch.gather(i, -1, order)
    ok = torch.gather(s, -1, order) > float("-inf")
    return torch.where(ok, sel, torch.full_like(sel, -1))


class TorchDistComm:
    """all_gather over torch.distributed (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather(self, t: torch.Tensor):
        out = [torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t.contiguous(), group=self.group)
        return out

    def all_gather_stacked(self, t: torch.Tensor):
        """(N, *t.shape): rank r's tensor at [r] (one all_gather_into_tensor
        on NCCL; a list all-gather elsewhere)."""
        t = t.contiguous()
        if t.is_cuda:
            out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            self.dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        return torch.stack(self.all_gather(t))


class PeerComm:
    """The sequence-split exchanges over NVLink peer memory (kvr_peer_*): each
    rank allocates one exchange buffer, the CUDA IPC handles travel once over
    torch.distributed, and every later exchange is a single kernel per rank
    that stores its rows into all ranks' buffers and merges locally — no NCCL
    on the data path.  Build it collectively on every rank (after
    torch.cuda.set_device), or with ``PeerComm.local()`` for one rank."""

    def __init__(self, group=None, _local=False):
        import ctypes

        from . import _native as N

        self.N = N
        buf = ctypes.c_void_p()
        N.call("kvr_peer_alloc", ctypes.byref(buf))
        self.own = buf.value
        self.opened = []
        if _local:
            self.world, self.rank, ptrs = 1, 0, [self.own]
        else:
            import torch.distributed as dist

            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
            hb = N.call("kvr_peer_handle_bytes")
            h = (ctypes.c_char * hb)()
            N.call("kvr_peer_handle", self.own, h)
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(h), group=group)
            ptrs = []
            for r, hr in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.own)
                    continue
                p = ctypes.c_void_p()
                N.call("kvr_peer_open", (ctypes.c_char * hb).from_buffer_copy(hr), ctypes.byref(p))
                self.opened.append(p.value)
                ptrs.append(p.value)
            dist.barrier(group=group)
        self.ptrs = (ctypes.c_void_p * self.world)(*ptrs)

    @classmethod
    def local(cls):
        return cls(_local=True)

    def merge_candidates(self, sc, sel, k_sel, tile_base, n_local):
        """Local candidates (B, H, k_local) -> (global sel, local sel), both
        (B, H, k_sel) int32, identical on every rank."""
        B, H, kl = sel.shape
        sc, sel = sc.float().contiguous(), sel.to(torch.int32).contiguous()
        lsel = torch.empty(B, H, k_sel, dtype=torch.int32, device=sel.device)
        gsel = torch.empty_like(lsel)
        self.N.call("kvr_peer_merge_candidates", self.ptrs, self.world, self.rank, self.N.ptr(sc), self.N.ptr(sel),
                    B * H, kl, k_sel, tile_base, n_local, self.N.ptr(gsel), self.N.ptr(lsel), self.N.stream())
        return gsel, lsel

    def merge_partials(self, part, out_dtype):
        """This rank's partial rows (rows, d+2) -> the merged output (rows, d)."""
        part = part.float().contiguous()
        rows = part.shape[0]
        out = torch.empty(rows, part.shape[1] - 2, dtype=out_dtype, device=part.device)
        self.N.call("kvr_peer_lse_merge", self.ptrs, self.world, self.rank, self.N.ptr(part), rows,
                    part.shape[1] - 2, self.N.ptr(out), self.N.dtype_code(out), self.N.stream())
        return out

    def status(self):
        """Raises KvrError(KVR_ETIMEOUT) if an exchange wait gave up."""
        import ctypes
        self.N.call("kvr_workspace_status", ctypes.c_void_p(self.own), self.N.stream())

    def close(self):
        for p in self.opened:
            self.N.call("kvr_peer_close", p)
        self.opened = []
        if self.own:
            self.N.call("kvr_peer_free", self.own)
            self.own = None


class SeqSplitDecoder:
    """Per-rank state of a sequence-split layer: the local sd1 store (global
    tile indices [tile_base, tile_base + store.n_tiles)) and, on the last
    rank, the window (B, cap, n_kv, d) fp16 with n_win valid rows."""

    def __init__(self, store: K.Sd1Store, tile_base: int, comm, window=None, n_win=0):
        self.store = store
        self.tile_base = tile_base
        self.comm = comm
        self.window = window
        self.n_win = n_win

    def local_candidates(self, q, k_sel):
        """Local top `k_sel` of this rank's tiles: (sel (B, H, k_sel) int32
        global tile indices, scores fp32, q').  A rank that owns fewer than
        k_sel tiles (or none) pads its list with index -1 / score -inf, so
        every rank passes tensors of the same shape to the all-gather."""
        return K.sd1_select(self.store, q, k_sel, tile_base=self.tile_base)

    def local_partial(self, q, qp, local_sel):
        """Log-sum-exp partial rows (B, n_q, d+2) over the selected tiles this
        rank owns (local indices, -1 = not here) plus, on the window rank, the
        window."""
        wk = wv = None
        if self.window is not None and self.n_win:
            wk, wv = self.window
        return K.sd1_attend(self.store, q, qp, local_sel, wk, wv, self.n_win if wk is not None else 0, partial=True)

    def n_local_tiles(self):
        return self.store.n_tiles

    def select_global(self, all_sc, all_idx, k_sel):
        """Gathered candidates (N, B, H, k) -> this rank's local selection
        (B, H, k_sel) int32 (-1 = tile not owned here) and the global
        selection (B, H, k_sel) (kvr_merge_candidates)."""
        gsel, lsel = K.merge_candidates(all_sc, all_idx, k_sel, self.tile_base, self.n_local_tiles())
        return lsel, gsel

    def step(self, q, k_sel, out_dtype=None, marks=None):
        """q (B, n_q, d) on this rank's GPU (same on every rank) -> (out
        (B, n_q, d), global selection (B, H, k_sel)).  `marks`, if given, is
        called between the phases with the phase name just finished (the
        bench records CUDA events there)."""
        q = q if q.dim() == 3 else q.unsqueeze(0)
        B, n_q, d = q.shape
        mark = marks or (lambda name: None)
        sel, sc, qp = self.local_candidates(q, k_sel)
        mark("local_select")
        if hasattr(self.comm, "merge_candidates"):
            # NVLink peer-memory exchanges: one kernel each, no NCCL
            gsel, local = self.comm.merge_candidates(sc, sel, k_sel, self.tile_base, self.n_local_tiles())
            mark("candidate_exchange")
            part = self.local_partial(q, qp, local)
            mark("local_attend")
            out = self.comm.merge_partials(part.reshape(B * n_q, d + 2), out_dtype or q.dtype)
            mark("partial_exchange")
            return out.view(B, n_q, d), gsel
        gather = getattr(self.comm, "all_gather_stacked", None) or (lambda t: torch.stack(self.comm.all_gather(t)))
        all_sc = gather(sc)
        all_idx = gather(sel.to(torch.int32))
        mark("candidate_allgather")
        local, gsel = self.select_global(all_sc, all_idx, k_sel)
        part = self.local_partial(q, qp, local)
        mark("local_attend")
        parts = gather(part)       # (N, B, n_q, d+2)
        mark("partial_allgather")
        merged = self.merge(parts.reshape(parts.shape[0], B * n_q, d + 2), out_dtype or q.dtype)
        mark("merge")
        return merged.view(B, n_q, d), gsel

    def merge(self, parts, out_dtype):
        """(N, rows, d+2) gathered partial rows -> (rows, d) (kvr_lse_merge)."""
        return K.lse_merge(parts, out_dtype)

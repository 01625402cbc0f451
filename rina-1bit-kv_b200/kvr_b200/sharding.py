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
Both exchanges use a communicator with ``all_gather(tensor) -> list``;
``TorchDistComm`` wraps torch.distributed (NCCL over NVLink on the GPU box,
gloo in the CPU tests); remote data lands in local memory before any kernel
reads it.
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

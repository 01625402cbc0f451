"""RetrievalIndex — compressed store of evicted tokens, drop-in for
modules/kvr_retrieval.py.

``codec='int4w'`` (default) keeps the reference's format and semantics: int4
K_pre codes with a per-(head, channel) absmax scale, V = W-predict(K) + int2
per-head residual, both bit-packed (kvr_retrieval.py:2-4, 69-91, 95-207).
Encode, scoring, top-k (token, chunk and attractor branches), gather, the
V-predict contraction (tensor cores, straight from the packed codes) and the
residual dequantisation run as sm_100a kernels; the one dense one-off —
``torch.linalg.pinv`` in ``calibrate`` — stays a library call, as in the
reference.  ``attend`` runs a whole layer's retrieval + attention with no host
synchronisation.

``codec='sd1'`` stores post-RoPE K and V as 1-bit sigma-delta codes in the
Hadamard/DCT domain with per-tile fp16 scales (no reference counterpart; spec
in oracle/sd1_ref.py).  Tokens that do not yet fill a tile wait, exact and
post-RoPE in fp16, in a tail buffer.

Selection order is deterministic: score descending, then index ascending
(torch.topk's tie order is unspecified, kvr_retrieval.py:392).
"""
import math

import numpy as np
import torch
import torch.nn.functional as F

from . import kernels as K


def _rotate_half(x):
    d2 = x.shape[-1] // 2
    return torch.cat([-x[..., d2:], x[..., :d2]], dim=-1)


def _apply_rotary(x, cos, sin):
    """kvr_retrieval.py:32-33."""
    return x * cos[:x.shape[0]] + _rotate_half(x) * sin[:x.shape[0]]


def _reverse_rotary(x, cos, sin):
    """kvr_retrieval.py:36-37."""
    return x * cos[:x.shape[0]] - _rotate_half(x) * sin[:x.shape[0]]


class RetrievalIndex:
    def __init__(self, n_kv, d_head, top_k=128, device="cuda", chunk_size=8, codec="int4w", tile=64,
                 transform="hadamard"):
        if codec not in ("int4w", "sd1"):
            raise ValueError(f"unknown codec {codec!r}")
        self.n_kv = n_kv
        self.d_head = d_head
        self.kv_dim = n_kv * d_head
        self.top_k = top_k
        self.chunk_size = chunk_size
        self.top_per_basin = 16
        self.device = device
        self.codec = codec
        self.k_scales = None
        self.k_packed = None
        self.vr_scales = None
        self.vr_packed = None
        self.n_stored = 0
        self.W = None
        self.K_mean = None
        self.V_mean = None
        self.cos = None
        self.sin = None
        self._halves_equal = False
        self.n_attractors = 128
        self.attractors = None
        self.labels = None
        self._vp = None          # (key, prepared V-predict weights)
        self._lab = None         # [int32 label buffer, labels view, labelled count]
        # sd1 state
        self.tile = tile
        self.transform = transform
        self.store = None
        self.tail_k = None
        self.tail_v = None
        self.n_tail = 0
        self._sd1_call = None    # cached pointer arguments of attend()
        self._sd1_upd_call = None  # cached pointer arguments of decode_step()

    # ------------------------------------------------------------ tables --
    def set_rotary_tables(self, cos, sin):
        """kvr_retrieval.py:63-65.  Also records whether the halves of each row
        are duplicated (true for HF tables), which lets kernels read half rows."""
        self.cos = cos
        self.sin = sin
        d2 = cos.shape[-1] // 2
        self._halves_equal = bool(torch.equal(cos[..., :d2], cos[..., d2:]) and torch.equal(sin[..., :d2], sin[..., d2:]))

    def _tables(self, n):
        if self.cos is None:
            z = torch.zeros(max(n, 1), self.d_head, device=self.device)
            return z + 1.0, z, False
        return self.cos, self.sin, self._halves_equal

    # ----------------------------------------------------- pack / unpack --
    def _pack_int4(self, x):
        u = (x.to(torch.uint8) + 8)
        return (u[..., 0::2] << 4) | u[..., 1::2]

    def _unpack_int4(self, p):
        hi = ((p >> 4).to(torch.int8) - 8)
        lo = ((p & 0x0F).to(torch.int8) - 8)
        return torch.stack([hi, lo], dim=-1).reshape(*p.shape[:-1], p.shape[-1] * 2)

    def _pack_int2(self, x):
        u = (x.to(torch.uint8) + 2)
        return (u[..., 0::4] << 6) | (u[..., 1::4] << 4) | (u[..., 2::4] << 2) | u[..., 3::4]

    def _unpack_int2(self, p):
        v = [((p >> s) & 0x03).to(torch.int8) - 2 for s in (6, 4, 2, 0)]
        return torch.stack(v, dim=-1).reshape(*p.shape[:-1], p.shape[-1] * 4)

    # -------------------------------------------------------------- core --
    @torch.no_grad()
    def calibrate(self, k_pre_sample, v_sample=None):
        """kvr_retrieval.py:95-122 (int4w).  For sd1 this only resets the store."""
        n = k_pre_sample.shape[0]
        self.n_stored = 0
        self.attractors = self.labels = None
        if self.codec == "sd1":
            self.k_scales = torch.ones(self.n_kv, self.d_head, device=self.device)  # marks "calibrated"
            self._sd1_reset()
            return
        k = k_pre_sample.to(self.device)
        self.k_scales = K.absmax_scales(k.float().reshape(n, self.n_kv, self.d_head))
        self.k_packed = torch.zeros(0, self.n_kv, self.d_head // 2, device=self.device, dtype=torch.uint8)
        self.vr_packed = torch.zeros(0, self.n_kv, self.d_head // 4, device=self.device, dtype=torch.uint8)
        self.k_codes = None
        self.vr_codes = None
        if v_sample is not None and n > 10:
            k2 = k.reshape(n, self.kv_dim).float()
            v2 = v_sample.to(self.device).reshape(n, self.kv_dim).float()
            half = n // 2
            k_tr, v_tr = k2[:half], v2[:half]
            self.K_mean = k_tr.mean(0, keepdim=True)
            self.V_mean = v_tr.mean(0, keepdim=True)
            kc = k_tr - self.K_mean
            vc = v_tr - self.V_mean
            self.W = (kc.T @ vc).T @ torch.linalg.pinv(kc.T @ kc)
            v_res = v2 - ((k2 - self.K_mean) @ self.W.T + self.V_mean)
            self.vr_scales = v_res.view(-1, self.n_kv, self.d_head).abs().amax(dim=(0, 2)).unsqueeze(1).clamp(min=1e-8)
        else:
            self.W = torch.eye(self.kv_dim, device=self.device)
            self.K_mean = torch.zeros(1, self.kv_dim, device=self.device)
            self.V_mean = torch.zeros(1, self.kv_dim, device=self.device)
            self.vr_scales = torch.ones(self.n_kv, 1, device=self.device)

    def _deq_k(self, kvh):
        """kvr_retrieval.py:124-129."""
        step = 2 * self.k_scales / 16
        packed = self.k_packed[:self.n_stored, kvh, :]
        return self._unpack_int4(packed).float() * step[kvh].float()

    def _predict_v(self, k_pre_flat):
        """kvr_retrieval.py:131-134 (a library GEMM)."""
        if self.W is None:
            return torch.zeros_like(k_pre_flat)
        return (k_pre_flat - self.K_mean) @ self.W.T + self.V_mean

    def _rotary(self, k_pre_2d, indices):
        if self.cos is None:
            return k_pre_2d
        c = self.cos[indices].squeeze(1).to(k_pre_2d.dtype)
        s = self.sin[indices].squeeze(1).to(k_pre_2d.dtype)
        return _apply_rotary(k_pre_2d, c, s)

    def _reconstruct_v(self, k_pre_top, top_idx):
        kv_flat = k_pre_top.reshape(-1, self.kv_dim)
        v_base = self._predict_v(kv_flat).reshape(-1, self.n_kv, self.d_head)
        vr_step = 2 * self.vr_scales / 4
        vr_dq = self._unpack_int2(self.vr_packed[top_idx]).float() * vr_step.unsqueeze(0)
        return (v_base + vr_dq).float()

    @torch.no_grad()
    def _ensure_capacity(self, needed):
        """kvr_retrieval.py:150-160: grow x2."""
        if needed <= self.k_packed.shape[0]:
            return
        new_cap = max(needed, self.k_packed.shape[0] * 2)
        k_ext = torch.zeros(new_cap - self.k_packed.shape[0], self.n_kv, self.d_head // 2, device=self.device,
                            dtype=torch.uint8)
        self.k_packed = torch.cat([self.k_packed, k_ext], dim=0)
        vr_ext = torch.zeros(new_cap - self.vr_packed.shape[0], self.n_kv, self.d_head // 4, device=self.device,
                             dtype=torch.uint8)
        self.vr_packed = torch.cat([self.vr_packed, vr_ext], dim=0)

    @torch.no_grad()
    def append(self, k_pre_rope, v=None):
        """kvr_retrieval.py:162-185."""
        if self.k_scales is None:
            raise RuntimeError("Call calibrate() first")
        if self.codec == "sd1":
            return self._sd1_append(k_pre_rope.reshape(1, self.n_kv, self.d_head),
                                    None if v is None else v.reshape(1, self.n_kv, self.d_head))
        self._ensure_capacity(self.n_stored + 1)
        k1 = k_pre_rope.to(self.device).reshape(1, self.n_kv, self.d_head)
        K.int4w_encode_k(k1, self.k_scales, out=self.k_packed[self.n_stored:self.n_stored + 1])
        if v is not None and self.W is not None:
            vp = self._predict_v(k1.float().reshape(1, -1)).reshape(1, self.n_kv, self.d_head)
            K.int4w_encode_vres(v.to(self.device).reshape(1, self.n_kv, self.d_head), vp, self.vr_scales,
                                out=self.vr_packed[self.n_stored:self.n_stored + 1])
        else:
            self.vr_packed[self.n_stored] = 0
        self.n_stored += 1

    @torch.no_grad()
    def batch_append(self, k_pre_all, v_all):
        """kvr_retrieval.py:187-207: REPLACES the store, pads max(1024, n//2) zero rows."""
        if self.codec == "sd1":
            self._sd1_reset()
            return self._sd1_append(k_pre_all, v_all)
        n = k_pre_all.shape[0]
        extra = max(1024, n // 2)
        k = k_pre_all.to(self.device)
        self.k_packed = torch.zeros(n + extra, self.n_kv, self.d_head // 2, device=self.device, dtype=torch.uint8)
        K.int4w_encode_k(k, self.k_scales, out=self.k_packed[:n])
        self.vr_packed = torch.zeros(n + extra, self.n_kv, self.d_head // 4, device=self.device, dtype=torch.uint8)
        if self.W is not None and n > 0:
            v_pred = self._predict_v(k.reshape(n, -1).float()).reshape(n, self.n_kv, self.d_head)
            K.int4w_encode_vres(v_all.to(self.device), v_pred, self.vr_scales, out=self.vr_packed[:n])
        self.n_stored = n

    # ----------------------------------------------------------- scoring --
    @torch.no_grad()
    def compute_all_scores(self, q_post_rope):
        """kvr_retrieval.py:265-289 -> (n_stored, n_kv) (a transposed view of
        the kernel's head-major buffer)."""
        self._require_int4w("compute_all_scores")
        cos, sin, he = self._tables(self.n_stored)
        return K.int4w_token_scores(q_post_rope, self.k_packed, self.k_scales, cos, sin, self.n_stored, he).t()

    @torch.no_grad()
    def compute_chunk_scores(self, q_post_rope):
        """kvr_retrieval.py:291-315 -> (n_chunks, n_kv)."""
        self._require_int4w("compute_chunk_scores")
        cs = self.chunk_size
        if cs <= 0 or self.n_stored // cs < 1:
            return self.compute_all_scores(q_post_rope)
        cos, sin, he = self._tables(self.n_stored)
        return K.int4w_chunk_scores(q_post_rope, self.k_packed, self.k_scales, cos, sin, self.n_stored, cs, he).t()

    @torch.no_grad()
    def build_attractors(self, iters=10):
        """kvr_retrieval.py:234-246: 128 basins of head-0 K_pre.  The reference
        clusters on the host with sklearn's MiniBatchKMeans (seed 42); here the
        clustering is a deterministic Lloyd k-means on the device
        (kernels.kmeans, kvr_cluster.cu) — same role and output shapes, not
        the same basins (sklearn's mini-batch result is version-dependent, so
        the branch was never pinned)."""
        if self.codec != "int4w":
            return
        nr = self.n_stored
        if nr < self.n_attractors * 2:
            return
        self.labels, self.attractors = K.kmeans(self._deq_k(0).float(), self.n_attractors, iters)
        self._lab = None

    @torch.no_grad()
    def compute_attractor_scores(self, q_post_rope):
        """kvr_retrieval.py:248-263: cosine of the head-0 group-mean query
        against every basin centroid, in column 0 of an (n_attractors, n_kv)
        tensor (the reference scores head 0 only and leaves the other columns
        unset; here they are zero)."""
        if self.attractors is None:
            return self.compute_all_scores(q_post_rope)
        g = q_post_rope.shape[0] // self.n_kv
        qa = q_post_rope[:g].float().mean(0)
        cen = self.attractors.float()
        out = torch.zeros(cen.shape[0], self.n_kv, device=cen.device)
        out[:, 0] = (cen @ qa) / ((cen.norm(dim=1) + 1e-8) * (qa.norm() + 1e-8))
        return out

    # --------------------------------------------------------- retrieval --
    def _empty(self):
        z = torch.zeros(0, self.n_kv, self.d_head, device=self.device, dtype=torch.float16)
        return z, z

    def _labels_device(self):
        """(int32 label buffer, labelled count): the clustering's basin labels,
        and every token appended after it assigned to its nearest basin on the
        device (kvr_int4w_assign_basins), so the attractor branch can return
        it.  ``self.labels`` stays a view of the labelled prefix; a caller that
        replaces it (or sets it to None) is followed."""
        lab = self.labels
        if self._lab is None or self._lab[1] is not lab:
            n0 = lab.numel()
            buf = torch.empty(max(n0, self.n_stored, 1), dtype=torch.int32, device=self.device)
            buf[:n0] = lab.to(device=self.device, dtype=torch.int32)
            self._lab = [buf, buf[:n0], n0]
            self.labels = self._lab[1]
        buf, view, n0 = self._lab
        nr = self.n_stored
        if nr > n0:
            if nr > buf.numel():
                grown = torch.empty(max(nr, 2 * buf.numel()), dtype=torch.int32, device=self.device)
                grown[:n0] = buf[:n0]
                buf = grown
            K.int4w_assign_basins(self.k_packed, self.k_scales, n0, nr, self.attractors, buf)
            self._lab = [buf, buf[:nr], nr]
            self.labels = self._lab[1]
        return self._lab[0], self._lab[2]

    def _vpredict_weights(self):
        """W' = W * diag(step) split for the tensor-core V-predict, prepared
        once per calibration (re-prepared if W, the means or the scales are
        replaced or modified in place)."""
        parts = (self.W, self.K_mean, self.V_mean, self.k_scales)
        key = tuple((t.data_ptr(), t._version) for t in parts)
        if self._vp is None or self._vp[0] != key:
            self._vp = (key, K.int4w_vpredict_prepare(self.W, self.K_mean, self.V_mean, self.k_scales, self.n_kv))
        return self._vp[1]

    @torch.no_grad()
    def select_device(self, q_post_rope, exclude_start=0, exclude_end=0):
        """The token indices retrieve_topk gathers, on the device: (top
        (rows, n_kv) int64, count) where count is None (all rows valid) or a
        device int32 (attractor branch, whose size is data-dependent); None
        when the reference would return nothing.  No host synchronisation."""
        nr = self.n_stored
        if nr == 0 or exclude_start >= nr or (exclude_start <= 0 and exclude_end >= nr):
            return None
        top_k = min(self.top_k, nr)
        if self.attractors is not None and self.labels is not None:
            # kvr_retrieval.py:332-367: top 48 basins x top 16 tokens, same list for every head
            lab, n_lab = self._labels_device()
            cos, sin, _ = self._tables(nr)
            top_a = min(48, self.attractors.shape[0])
            return K.int4w_attractor_select(q_post_rope, self.n_kv, self.k_packed, self.k_scales, cos, sin,
                                            self.attractors, lab, n_lab, top_a, exclude_start, exclude_end)
        cs = self.chunk_size
        if cs > 0 and nr >= cs * 2:
            # intended chunk branch (kvr_retrieval.py:370-388; the reference body is unreachable)
            sc = self.compute_chunk_scores(q_post_rope).t().contiguous()  # (n_kv, n_chunks)
            n_chunks = sc.shape[1]
            ec0 = exclude_start // cs
            ec1 = min((exclude_end + cs - 1) // cs, n_chunks)
            if ec0 >= ec1:
                ec0 = ec1 = 0
            top_chunks = min(max(1, top_k // cs), n_chunks)
            cidx, _ = K.topk_rows(sc, top_chunks, ec0, ec1, transpose_out=True)  # (top_chunks, n_kv)
            tok = cidx.unsqueeze(1) * cs + torch.arange(cs, device=self.device).view(1, cs, 1)
            return tok.reshape(top_chunks * cs, self.n_kv), None
        cos, sin, he = self._tables(nr)
        idx = K.int4w_token_topk(q_post_rope, self.k_packed, self.k_scales, cos, sin, nr, top_k, he, exclude_start,
                                 exclude_end)
        return idx, None

    @torch.no_grad()
    def select_indices(self, q_post_rope, exclude_start=0, exclude_end=0):
        """Token indices (rows, n_kv) the int4w retrieve_topk gathers, or None
        when it would return nothing (reads the attractor branch's row count
        back to the host)."""
        sel = self.select_device(q_post_rope, exclude_start, exclude_end)
        if sel is None:
            return None
        top, count = sel
        if count is not None:
            n = int(count.item())
            if n == 0:
                return None
            top = top[:n]
        return top

    def _gather_kv(self, top, count=None):
        cos, sin, _ = self._tables(self.n_stored)
        ret_k, _ = K.int4w_gather(self.k_packed, self.k_scales, top, cos, sin, want_x=False, count=count)
        ret_v = K.int4w_vpredict(self.k_packed, top, self._vpredict_weights(), self.vr_packed, self.vr_scales,
                                 count=count)
        return ret_k, ret_v

    @torch.no_grad()
    def retrieve_topk(self, q_post_rope, n_q=None, exclude_start=0, exclude_end=0):
        """kvr_retrieval.py:317-412 -> (ret_k fp32 post-RoPE, ret_v fp16), each
        (rows, n_kv, d).  For sd1: the decoded selected tiles followed by the
        exact pending tail."""
        if self.codec == "sd1":
            return self._sd1_retrieve(q_post_rope, exclude_start, exclude_end)
        top = self.select_indices(q_post_rope, exclude_start, exclude_end)
        if top is None:
            return self._empty()
        return self._gather_kv(top)

    @torch.no_grad()
    def retrieve(self, q_post_rope, n_q=None):
        """Legacy per-Q-head path (kvr_retrieval.py:209-232): every query head
        scores all stored tokens of its KV head by dot / sqrt(d) (post-RoPE),
        keeps its own top_k and attends only those.  Kernel pieces: the
        dequantised, re-rotated keys of all tokens (kvr_int4w_gather over
        every index), per-head score rows, kvr_topk_rows, the V-predict
        kernel, and one decode attention per query head."""
        self._require_int4w("retrieve")
        n_q = n_q or q_post_rope.shape[0]
        g = n_q // self.n_kv
        d = self.d_head
        out = torch.zeros(n_q, d, device=q_post_rope.device, dtype=torch.float32)
        nr = self.n_stored
        if nr == 0:
            return out
        top_k = min(self.top_k, nr)
        every = torch.arange(nr, device=self.device).view(nr, 1).expand(nr, self.n_kv).contiguous()
        cos, sin, _ = self._tables(nr)
        k_post, _ = K.int4w_gather(self.k_packed, self.k_scales, every, cos, sin, want_x=False)  # (nr, n_kv, d)
        q = q_post_rope[:n_q].float().view(self.n_kv, g, d)
        # (n_kv, g, nr) dot products, one row per query head
        sc = torch.einsum("hgd,thd->hgt", q, k_post).reshape(n_q, nr).div_(math.sqrt(d)).contiguous()
        idx, _ = K.topk_rows(sc, top_k)                                    # (n_q, top_k)
        for hi in range(n_q):
            kvh = hi // g
            top = idx[hi].view(top_k, 1).expand(top_k, self.n_kv).contiguous()
            rk, rv = self._gather_kv(top)
            out[hi] = K.decode_attn(q_post_rope[hi:hi + 1].float(), [(rk[:, kvh:kvh + 1], rv[:, kvh:kvh + 1])],
                                    out_dtype=torch.float32, n_kv=1)[0]
        return out

    def _require_int4w(self, what):
        if self.codec != "int4w":
            raise NotImplementedError(f"{what} is defined for codec='int4w' only")

    # ------------------------------------------------------- save / load --
    _INT4W_TENSORS = ("k_scales", "vr_scales", "W", "K_mean", "V_mean", "attractors", "labels")

    def state_dict(self, prefix=""):
        """(meta, tensors) for kvr_b200.cache_io: the packed store and its
        counters.  RoPE tables are not part of it (set_rotary_tables again
        after loading; KVRHook does)."""
        meta = {"codec": self.codec, "n_kv": self.n_kv, "d_head": self.d_head, "top_k": self.top_k,
                "chunk_size": self.chunk_size, "tile": self.tile, "transform": self.transform,
                "n_stored": self.n_stored, "n_tail": self.n_tail, "calibrated": self.k_scales is not None}
        t = {}
        if self.codec == "int4w":
            for name in self._INT4W_TENSORS:
                v = getattr(self, name)
                if v is not None:
                    t[prefix + name] = v
            if self.k_packed is not None:
                t[prefix + "k_packed"] = self.k_packed[:self.n_stored]
            if self.vr_packed is not None:
                t[prefix + "vr_packed"] = self.vr_packed[:self.n_stored]
        elif self.store is not None:
            nt = self.store.n_tiles
            meta["n_tiles"] = nt
            for name in ("kbits", "kscale", "vbits", "vscale"):
                t[prefix + name] = getattr(self.store, name)[:, :, :nt]
            t[prefix + "tail_k"] = self.tail_k[:, :self.n_tail]
            t[prefix + "tail_v"] = self.tail_v[:, :self.n_tail]
        return meta, t

    def load_state_dict(self, meta, tensors, prefix=""):
        for key in ("codec", "n_kv", "d_head", "tile", "transform"):
            if meta[key] != getattr(self, key):
                raise ValueError(f"cache {key}={meta[key]!r} does not match this index ({getattr(self, key)!r})")
        self.top_k, self.chunk_size = meta["top_k"], meta["chunk_size"]
        dev = self.device
        if self.codec == "sd1":
            self._sd1_reset()  # fresh buffers (clears the counters), filled below
            self.attractors = self.labels = None
            self.k_scales = (torch.ones(self.n_kv, self.d_head, device=dev)  # marks "calibrated"
                             if meta.get("calibrated", self.n_stored > 0) else None)
        self.n_stored, self.n_tail = int(meta["n_stored"]), int(meta["n_tail"])
        if self.codec == "int4w":
            for name in self._INT4W_TENSORS:
                setattr(self, name, tensors[prefix + name].to(dev) if prefix + name in tensors else None)
            n = self.n_stored
            for name in ("k_packed", "vr_packed"):
                if prefix + name in tensors:
                    src = tensors[prefix + name].to(dev)
                    buf = torch.zeros(n + max(1024, n // 2), *src.shape[1:], dtype=src.dtype, device=dev)
                    buf[:n] = src
                    setattr(self, name, buf)
                else:
                    setattr(self, name, None)
            return
        if "n_tiles" in meta:
            nt = int(meta["n_tiles"])
            self.store.grow(max(64, 2 * nt))
            for name in ("kbits", "kscale", "vbits", "vscale"):
                getattr(self.store, name)[:, :, :nt] = tensors[prefix + name].to(dev)
            self.store.n_tiles = nt
            self.tail_k[:, :self.n_tail] = tensors[prefix + "tail_k"].to(dev)
            self.tail_v[:, :self.n_tail] = tensors[prefix + "tail_v"].to(dev)

    # --------------------------------------------------------------- sd1 --
    def _sd1_reset(self):
        self.store = K.Sd1Store(1, self.n_kv, 64, self.tile, self.transform, self.device)
        self.tail_k = torch.zeros(1, self.tile, self.n_kv, self.d_head, dtype=torch.float16, device=self.device)
        self.tail_v = torch.zeros_like(self.tail_k)
        self.n_tail = 0
        self.n_stored = 0

    def _rope_post(self, k_pre, pos0):
        if self.cos is None:
            return k_pre.float()
        n = k_pre.shape[0]
        c = self.cos[pos0:pos0 + n].to(self.device).float().unsqueeze(1)
        s = self.sin[pos0:pos0 + n].to(self.device).float().unsqueeze(1)
        return k_pre.float() * c + _rotate_half(k_pre.float()) * s

    def _sd1_append(self, k_pre, v):
        """Encode whole tiles straight from K_pre (RoPE at positions n_stored+i
        inside the encoder); keep the remainder exact in the tail."""
        if self.store is None:
            self._sd1_reset()
        k_pre = k_pre.to(self.device)
        v = torch.zeros_like(k_pre) if v is None else v.to(self.device)
        n = k_pre.shape[0]
        t = self.tile
        i = 0
        # fill a partial tail first
        if self.n_tail:
            take = min(t - self.n_tail, n)
            self._tail_put(k_pre[:take], v[:take], self.n_stored)
            i = take
        n_full = (n - i) // t
        if n_full:
            need = self.store.n_tiles + n_full
            if need > self.store.nt_cap:
                self.store.grow(max(need, 2 * self.store.nt_cap))
            cos = self.cos.to(self.device) if self.cos is not None else None
            sin = self.sin.to(self.device) if self.sin is not None else None
            K.sd1_encode(self.store, k_pre[i:i + n_full * t], v[i:i + n_full * t], cos=cos, sin=sin,
                         pos0=self.n_stored)
            self.n_stored += n_full * t
            i += n_full * t
        if i < n:
            self._tail_put(k_pre[i:], v[i:], self.n_stored)

    def _tail_put(self, k_pre, v, pos0):
        m = k_pre.shape[0]
        self.tail_k[0, self.n_tail:self.n_tail + m] = self._rope_post(k_pre.float(), pos0 + self.n_tail).half()
        self.tail_v[0, self.n_tail:self.n_tail + m] = v.float().half()
        self.n_tail += m
        if self.n_tail == self.tile:
            if self.store.n_tiles + 1 > self.store.nt_cap:
                self.store.grow(2 * self.store.nt_cap)
            K.sd1_encode(self.store, self.tail_k, self.tail_v)
            self.n_stored += self.tile
            self.n_tail = 0

    @torch.no_grad()
    def prefill_tile_scores(self, q_block):
        """sd1: tile scores of a block of prefill-position queries against the
        encoded tiles on the tensor cores (kvr_sd1_prefill_scores, tcgen05):
        q_block (nq, n_q, d) post-RoPE -> (nq, n_kv, n_tiles) fp32, the max over
        each tile of q'.k-hat.  No reference counterpart (the reference only
        retrieves at decode); for prefill-time retrieval over a long prompt."""
        if self.codec != "sd1" or self.store is None:
            raise NotImplementedError("prefill_tile_scores needs codec='sd1' with encoded tiles")
        return K.sd1_prefill_scores(self.store, q_block)

    @property
    def n_tokens(self):
        """Tokens held: encoded + pending tail (sd1); n_stored (int4w)."""
        return self.n_stored + (self.n_tail if self.codec == "sd1" else 0)

    def _sd1_select(self, q_post_rope, exclude_start=0, exclude_end=0):
        t = self.tile
        k_sel = max(1, self.top_k // t)
        ex0, ex1 = exclude_start // t, min((exclude_end + t - 1) // t, self.store.n_tiles)
        if ex0 >= ex1:
            ex0 = ex1 = 0
        return K.sd1_select(self.store, q_post_rope.unsqueeze(0), k_sel, ex0, ex1)

    def _sd1_retrieve(self, q_post_rope, exclude_start, exclude_end):
        if self.store is None or self.n_tokens == 0:
            return self._empty()
        parts_k, parts_v = [], []
        if self.store.n_tiles:
            sel, _, _ = self._sd1_select(q_post_rope, exclude_start, exclude_end)
            rk, rv = K.sd1_decode_tiles(self.store, sel.long())
            keep = (sel[0] >= 0).repeat_interleave(self.tile, dim=1).all(0)  # drop empty slots
            parts_k.append(rk[0][keep])
            parts_v.append(rv[0][keep])
        if self.n_tail:
            parts_k.append(self.tail_k[0, :self.n_tail].float())
            parts_v.append(self.tail_v[0, :self.n_tail])
        return torch.cat(parts_k, 0).contiguous(), torch.cat(parts_v, 0).contiguous()

    @torch.no_grad()
    def decode_step(self, q_pre, k_pre, v, window, pos, cos, sin, exclude_start=0, exclude_end=0, out=None):
        """sd1, batch 1: one layer's decode step with its store update fused in
        (kvr_generator.py:78-98, kvr_hook.py:136-148 and :274-282 in one
        call).  q_pre (n_q, d), k_pre and v (n_kv, d): the new token's
        pre-RoPE rows in the model dtype; RoPE at `pos` from the (max_pos, d)
        tables cos/sin.  The new K/V take the window's next ring slot; when the
        window is full the slot's old row first moves to the pending tail.
        Then window + tail + selected tiles are attended (exclusion range in
        tokens, as for ``attend``).  One cluster launch; when the eviction
        fills the tail, the store update, the tile encode and the step run as
        separate launches so the new tile is in the store before the step, as
        in the step-by-step path.  Returns (out (n_q, d) of q's dtype, RoPE(q));
        the RoPE(q) buffer belongs to the index and the next call overwrites it."""
        if self.codec != "sd1":
            raise NotImplementedError("decode_step is the sd1 codec's fused path")
        if self.store is None:
            self._sd1_reset()
        slot = window.pos % window.cap
        evict = window.n >= window.cap
        if evict and self.n_tail + 1 == self.tile:
            q_rot = K.decode_store_update(q_pre, k_pre, v, cos, sin, pos, window.k, window.v, slot, self.tail_k[0],
                                          self.tail_v[0], self.n_tail, True)
            self.n_tail += 1
            st = self.store
            if st.n_tiles + 1 > st.nt_cap:
                st.grow(2 * st.nt_cap)
            K.sd1_encode(st, self.tail_k, self.tail_v)
            self.n_stored += self.tile
            self.n_tail = 0
            window.pos += 1
            window.n = min(window.n + 1, window.cap)
            return self.attend(q_rot, window, exclude_start, exclude_end, out=out), q_rot
        if evict:
            self.n_tail += 1
        window.pos += 1
        window.n = min(window.n + 1, window.cap)
        st = self.store
        t = self.tile
        k_sel = max(1, self.top_k // t) if st.n_tiles else 0
        ex0, ex1 = exclude_start // t, min((exclude_end + t - 1) // t, st.n_tiles)
        if ex0 >= ex1:
            ex0 = ex1 = 0
        for x in (q_pre, k_pre, v):
            if not x.is_cuda or not x.is_contiguous() or x.dtype != q_pre.dtype:
                raise ValueError("q, k and v must be contiguous CUDA tensors of one dtype")
        N = K.N
        n_q = q_pre.shape[0]
        # pointer arguments of the tables, window, tail and store are cached
        # (they change only when a buffer is reallocated): one ctypes call
        key = (st.kbits.data_ptr(), st.nt_cap, id(window), window.k.data_ptr(), self.tail_k.data_ptr(),
               cos.data_ptr(), sin.data_ptr(), q_pre.dtype, n_q)
        c = self._sd1_upd_call
        if c is None or c[0] != key:
            cos_c, sin_c, rs = K._rope_args(cos.float(), sin.float())
            c = self._sd1_upd_call = (
                key, (cos_c.data_ptr(), sin_c.data_ptr(), rs),
                (window.k.data_ptr(), window.v.data_ptr(), window.cap), (self.tail_k.data_ptr(), self.tail_v.data_ptr()),
                (st.kbits.data_ptr(), st.kscale.data_ptr(), st.vbits.data_ptr(), st.vscale.data_ptr(), st.nt_cap),
                torch.empty_like(q_pre), N.dtype_code(q_pre), N.TRANSFORMS[st.kind], (cos_c, sin_c))
        _, tb, wk, tl, sp, q_rot, dt, kind, _ = c
        if out is None:
            res = None
            out = torch.empty(n_q, self.d_head, dtype=q_pre.dtype, device=q_pre.device)
        else:
            if out.dtype != q_pre.dtype or not out.is_contiguous() or out.numel() != n_q * self.d_head:
                raise ValueError("out must be a contiguous (n_q, d) tensor of q's dtype")
            res = out
        wkey = (1, n_q, self.n_kv, st.n_tiles, t, k_sel, window.n, self.n_tail)
        need = K._STEP_WS.get(wkey)
        if need is None:
            need = K._STEP_WS[wkey] = N.call("kvr_sd1_workspace_bytes", *wkey)
        ws = N.workspace("sd1_step", need, q_pre.device)
        N.call("kvr_sd1_decode_step_update", q_pre.data_ptr(), k_pre.data_ptr(), v.data_ptr(), dt, n_q, self.n_kv,
               tb[0], tb[1], tb[2], pos, q_rot.data_ptr(), wk[0], wk[1], wk[2], window.n, slot, tl[0], tl[1],
               self.n_tail, int(evict), sp[0], sp[1], sp[2], sp[3], sp[4], st.n_tiles, t, kind, k_sel, ex0, ex1, 0.0,
               out.data_ptr(), dt, None, ws.data_ptr(), ws.numel(), N.stream())
        return (out if res is None else res), q_rot

    def attend(self, q_post_rope, window=None, exclude_start=0, exclude_end=0, out_dtype=None, out=None):
        """One layer's retrieval + attention for the current step, q (n_q, d)
        -> (n_q, d): exact softmax over the window buffer (if given) and the
        retrieved rows — the hook's einsum over cat(window, retrieved)
        (kvr_hook.py:274-282) without materialising the concatenation and with
        no host synchronisation.  int4w: selection (token, chunk or attractor
        branch) -> gather -> tensor-core V-predict -> decode attention (the
        attractor branch's row count stays on the device).  sd1: one fused
        decode step over the window, the pending tail and the selected tiles.
        ``out`` (sd1, optional): an (n_q, d) tensor of q's dtype to write the
        result into instead of a new tensor."""
        if self.codec == "int4w":
            nw = window.n if window is not None else 0
            out_dtype = out_dtype or torch.float32
            sel = self.select_device(q_post_rope.float(), exclude_start, exclude_end) if self.n_stored else None
            if sel is None and not nw:
                return torch.zeros(q_post_rope.shape[0], self.d_head, dtype=out_dtype, device=q_post_rope.device)
            if nw:
                win = (window.k[:nw], window.v[:nw])
            else:
                z = torch.zeros(0, self.n_kv, self.d_head, dtype=torch.float16, device=q_post_rope.device)
                win = (z, z)
            if sel is None:
                return K.decode_attn(q_post_rope, [win], out_dtype=out_dtype, n_kv=self.n_kv)
            top, count = sel
            rk, rv = self._gather_kv(top, count)
            return K.decode_attn(q_post_rope, [win, (rk, rv)], out_dtype=out_dtype, n_kv=self.n_kv, n1_count=count)
        if self.store is None:
            self._sd1_reset()
        st = self.store
        t = self.tile
        k_sel = max(1, self.top_k // t) if st.n_tiles else 0
        ex0, ex1 = exclude_start // t, min((exclude_end + t - 1) // t, st.n_tiles)
        if ex0 >= ex1:
            ex0 = ex1 = 0
        q = q_post_rope if q_post_rope.is_contiguous() else q_post_rope.contiguous()
        if not q.is_cuda:
            raise ValueError("kvr_b200 operators need CUDA tensors (this build has no CPU path)")
        n_q = q.shape[0]
        nw = window.n if window is not None else 0
        # the pointer arguments of this store / window / tail are cached (they
        # change only when a buffer is reallocated); one ctypes call per layer
        key = (st.kbits.data_ptr(), st.nt_cap, id(window), window.k.data_ptr() if window is not None else 0,
               self.tail_k.data_ptr())
        c = self._sd1_call
        if c is None or c[0] != key:
            P = K.ptr
            wk = (P(window.k), P(window.v), window.cap) if window is not None else (None, None, 1)
            c = self._sd1_call = (key, wk, (P(self.tail_k), P(self.tail_v)),
                                  (P(st.kbits), P(st.kscale), P(st.vbits), P(st.vscale), st.nt_cap))
        _, wk, tl, sp = c
        N = K.N
        if out is not None and (out.dtype != q.dtype or not out.is_contiguous() or out.numel() != n_q * self.d_head):
            raise ValueError("out must be a contiguous (n_q, d) tensor of q's dtype")
        res = out
        out = torch.empty(1, n_q, self.d_head, dtype=q.dtype, device=q.device) if out is None else out
        wkey = (1, n_q, self.n_kv, st.n_tiles, t, k_sel, nw, self.n_tail)
        need = K._STEP_WS.get(wkey)
        if need is None:
            need = K._STEP_WS[wkey] = N.call("kvr_sd1_workspace_bytes", *wkey)
        ws = N.workspace("sd1_step", need, q.device)
        N.call("kvr_sd1_decode_step", q.data_ptr(), N.dtype_code(q), 1, n_q, self.n_kv, wk[0] if nw else None,
               wk[1] if nw else None, wk[2], nw, tl[0] if self.n_tail else None, tl[1] if self.n_tail else None,
               self.n_tail, sp[0], sp[1], sp[2], sp[3], sp[4], st.n_tiles, t, N.TRANSFORMS[st.kind], k_sel, ex0,
               ex1, 0.0, out.data_ptr(), N.dtype_code(out), None, ws.data_ptr(), ws.numel(), N.stream())
        if res is not None:
            return res
        return out[0] if out_dtype is None or out_dtype == q.dtype else out[0].to(out_dtype)

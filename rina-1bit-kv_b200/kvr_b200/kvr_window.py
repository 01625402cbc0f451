"""WindowBuffer — fp16 ring of the last N tokens' post-RoPE K/V.

Drop-in for modules/kvr_window.py (same constructor, attributes ``k, v, pos,
n, cap`` and methods).  Ring writes run in one kernel (kvr_window_write) and
``attention`` runs the split-K decode-attention kernel (kvr_decode_attn)
instead of the reference's per-head Python loop (kvr_window.py:64-68).
"""
import torch

from . import kernels as K


class WindowBuffer:
    def __init__(self, n_kv, d_head, window_size=2048, device="cuda"):
        self.n_kv = n_kv
        self.d_head = d_head
        self.cap = window_size
        self.k = torch.zeros(window_size, n_kv, d_head, device=device, dtype=torch.float16)
        self.v = torch.zeros(window_size, n_kv, d_head, device=device, dtype=torch.float16)
        self.pos = 0
        self.n = 0

    @torch.no_grad()
    def append(self, k_post_rope, v):
        """kvr_window.py:19-25."""
        K.window_write(k_post_rope.reshape(1, self.n_kv, self.d_head), v.reshape(1, self.n_kv, self.d_head),
                       self.k, self.v, self.pos)
        self.pos += 1
        self.n = min(self.n + 1, self.cap)

    # ------------------------------------------------------- save / load --
    def state_dict(self, prefix=""):
        """(meta, tensors) for kvr_b200.cache_io: the fp16 rings and counters."""
        return ({"cap": self.cap, "pos": self.pos, "n": self.n, "n_kv": self.n_kv, "d_head": self.d_head},
                {prefix + "k": self.k, prefix + "v": self.v})

    def load_state_dict(self, meta, tensors, prefix=""):
        if (meta["cap"], meta["n_kv"], meta["d_head"]) != (self.cap, self.n_kv, self.d_head):
            raise ValueError(f"window shape {(meta['cap'], meta['n_kv'], meta['d_head'])} does not match "
                             f"{(self.cap, self.n_kv, self.d_head)}")
        self.k.copy_(tensors[prefix + "k"])
        self.v.copy_(tensors[prefix + "v"])
        self.pos, self.n = int(meta["pos"]), int(meta["n"])

    @torch.no_grad()
    def batch_append(self, k_all, v_all):
        """kvr_window.py:27-41: token i lands in slot (pos + i) % cap."""
        n = k_all.shape[0]
        if n == 0:
            return
        K.window_write(k_all, v_all, self.k, self.v, self.pos)
        self.pos += n
        self.n = min(self.n + n, self.cap)

    @torch.no_grad()
    def attention(self, q_post_rope, n_q=None, scale=None):
        """kvr_window.py:43-69: exact softmax over the window, GQA kvh = hi // g.
        Returns (n_q, d_head) fp32."""
        n_q = n_q or q_post_rope.shape[0]
        q = q_post_rope[:n_q].float()
        return K.decode_attn(q, [(self.k[:self.n], self.v[:self.n])], scale=scale, out_dtype=torch.float32,
                             n_kv=self.n_kv)

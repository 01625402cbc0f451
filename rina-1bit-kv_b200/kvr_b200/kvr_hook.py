"""KVRHook — window + compressed-retrieval attention injected into a HF
decoder through forward hooks.  Drop-in for modules/kvr_hook.py: same
constructor keywords, ``prefill/register/remove/reset``, the ``_step`` and
``_context_len`` counters callers bump by hand, per-layer ``windows`` and
``retrievals``.

Differences, all deliberate:
* attention runs on the B200 kernels through ``RetrievalIndex.attend``
  (selection, gather, tensor-core V-predict and the window + retrieved
  attention for int4w; the fused 1-bit step for ``codec='sd1'``), with no
  host synchronisation, instead of the reference's einsum
  (modules/kvr_hook.py:274-282);
* RoPE tables come from ``model.model.rotary_emb`` when the attention module
  has none (transformers >= 5 removed ``self_attn.rotary_emb``, which
  modules/kvr_hook.py:50-53 uses);
* eviction un-rotates the evicted key at its own position ``pos - cap``; the
  reference un-rotates at ``pos`` (modules/kvr_hook.py:142-144) —
  ``reference_eviction_rope=True`` reproduces that for parity studies;
* the k-means the reference runs on the host after prefill
  (modules/kvr_hook.py:133, sklearn) is a device Lloyd k-means here, and the
  attractor branch it enables runs on kernels; ``attractors=False`` skips it
  (token branch).
The quality experiments of the reference (calibration s/b, MLP adapters,
denoise steps, warm-up capture; modules/kvr_hook.py:157-214, 286-307) are kept
as plain torch code — they are not part of the compressed-KV hot path.
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import kernels as K
from .kvr_retrieval import RetrievalIndex, _apply_rotary, _reverse_rotary
from .kvr_window import WindowBuffer


def rope_tables(model, max_pos, device):
    """(max_pos, d) cos/sin tables from the model's rotary module."""
    layer0 = model.model.layers[0].self_attn
    rot = getattr(layer0, "rotary_emb", None) or getattr(model.model, "rotary_emb", None)
    if rot is None:
        raise RuntimeError("model has no rotary embedding module")
    cfg = model.config
    n_q = cfg.num_attention_heads
    d = getattr(cfg, "head_dim", None) or cfg.hidden_size // n_q
    dummy = torch.empty(1, max_pos, n_q, d, device=device, dtype=torch.float32)
    pos = torch.arange(max_pos, device=device).unsqueeze(0)
    cos, sin = rot(dummy, position_ids=pos)
    return cos[0].float(), sin[0].float()


def exclusion_range(context_len, n_window, n_stored):
    """Token range of the index that is also in the window (kvr_hook.py:262-267,
    kvr_generator.py:439-444): [max(0, ctx - nw), min(n_stored, ctx)), empty
    if inverted."""
    s, e = max(0, context_len - n_window), min(n_stored, context_len)
    return (0, 0) if s >= e else (s, e)


class KVRHook:
    def __init__(self, model, window_size=2048, top_k=128, ret_weight=1.0, device=None, **kwargs):
        self.model = model
        self.device = device or model.device
        cfg = model.config
        self.n_layers = cfg.num_hidden_layers
        self.n_kv = cfg.num_key_value_heads
        self.n_q = cfg.num_attention_heads
        self.d_head = getattr(cfg, "head_dim", None) or (cfg.hidden_size // self.n_q)
        self.g = self.n_q // self.n_kv
        self.window_size = window_size
        self.top_k = top_k
        self._ret_weight = ret_weight
        self.num_denoise_steps = kwargs.get("num_denoise_steps", 3)
        self.chunk_size = kwargs.get("chunk_size", 0)
        self.warmup_mode = kwargs.get("warmup_mode", False)
        self.codec = kwargs.get("codec", "int4w")
        self.tile = kwargs.get("tile", 64)
        self.transform = kwargs.get("transform", "hadamard")
        self.use_attractors = kwargs.get("attractors", True)
        self.reference_eviction_rope = kwargs.get("reference_eviction_rope", False)
        # sd1: encode each layer's evicted prefix inside its projection hook
        # during the prefill forward (no fp32 K/V capture of the prompt)
        self.fused_prefill = kwargs.get("fused_prefill", True)
        self._context_len = 0
        self._prefill_done = False
        self._hooks = []
        self._step = 0
        self._retrieval_built = False
        self.calib_native = [[] for _ in range(self.n_layers)]
        self.calib_kvr = [[] for _ in range(self.n_layers)]
        self.calib_s = None
        self.calib_b = None
        self.mlp_adapter_data = [[] for _ in range(self.n_layers)]
        self.adapters = [None] * self.n_layers
        self._new_stores()
        max_pos = cfg.max_position_embeddings
        self.cos_tbl, self.sin_tbl = rope_tables(model, max_pos, self.device)

    def _new_stores(self):
        self.windows = [WindowBuffer(self.n_kv, self.d_head, self.window_size, self.device)
                        for _ in range(self.n_layers)]
        self.retrievals = [RetrievalIndex(self.n_kv, self.d_head, self.top_k, device=self.device,
                                          chunk_size=self.chunk_size, codec=self.codec, tile=self.tile,
                                          transform=self.transform)
                           for _ in range(self.n_layers)]

    # ------------------------------------------------------------ stores --
    def _rotate(self, x, pos0, reverse=False):
        n = x.shape[0]
        c = self.cos_tbl[pos0:pos0 + n].unsqueeze(1).to(x.dtype)
        s = self.sin_tbl[pos0:pos0 + n].unsqueeze(1).to(x.dtype)
        fn = _reverse_rotary if reverse else _apply_rotary
        return fn(x.reshape(n, -1, self.d_head), c, s).view(n, -1, self.d_head)

    def _ensure_retrieval_built(self, li):
        """kvr_hook.py:57-76: build the index from a full window (lazy path)."""
        if self._retrieval_built and self.retrievals[li].n_stored > 0:
            return
        win = self.windows[li]
        if win.n < win.cap:
            return
        k_post = win.k[:win.n].float()
        k_pre = self._rotate(k_post, 0, reverse=True)
        ret = self.retrievals[li]
        ret.set_rotary_tables(self.cos_tbl, self.sin_tbl)
        ret.calibrate(k_pre, win.v[:win.n].float())
        ret.batch_append(k_pre, win.v[:win.n].float())

    def _build_all_retrievals(self):
        if self._retrieval_built:
            return
        for li in range(self.n_layers):
            self._ensure_retrieval_built(li)
        self._retrieval_built = True

    @torch.no_grad()
    def prefill(self, input_ids):
        """kvr_hook.py:85-134: one HF forward with capture hooks on k/v
        projections; the window keeps the last `window` tokens, the index the
        evicted prefix (calibrated on the whole prompt)."""
        if self.codec == "sd1" and self.fused_prefill:
            return self._prefill_sd1_fused(input_ids)
        n_prompt = input_ids.shape[1]
        cap_k, cap_v, hooks = {}, {}, []
        for li in range(self.n_layers):
            attn = self.model.model.layers[li].self_attn

            def hook_fn(mod, args, kwargs, output, li=li):
                hidden = kwargs["hidden_states"] if "hidden_states" in kwargs else args[0]
                cap_k[li] = mod.k_proj(hidden).float().view(-1, self.n_kv, self.d_head)
                cap_v[li] = mod.v_proj(hidden).float().view(-1, self.n_kv, self.d_head)

            hooks.append(attn.register_forward_hook(hook_fn, with_kwargs=True))
        try:
            self.model(input_ids, logits_to_keep=1)
        finally:
            for h in hooks:
                h.remove()
        for li in range(self.n_layers):
            k_post = self._rotate(cap_k[li], 0)
            self.retrievals[li].set_rotary_tables(self.cos_tbl, self.sin_tbl)
            self.windows[li].batch_append(k_post, cap_v[li])
        self._context_len = n_prompt
        self._prefill_done = True
        if n_prompt > self.window_size:
            n_ret = n_prompt - self.window_size
            for li in range(self.n_layers):
                ret = self.retrievals[li]
                ret.calibrate(cap_k[li], cap_v[li])
                ret.batch_append(cap_k[li][:n_ret], cap_v[li][:n_ret])
                if self.use_attractors:
                    ret.build_attractors()
            self._retrieval_built = True

    def _prefill_sd1_fused(self, input_ids):
        """prefill for codec='sd1' with the stores built inside the forward:
        each layer's k/v projection hook writes the last `window` tokens
        (post-RoPE) into the window ring and encodes the evicted prefix into
        the 1-bit store straight from the projection output (RoPE applied in
        the encoder).  Same stores as the capture path of `prefill` (the sd1
        index needs no whole-prompt calibration), without holding fp32 copies
        of every layer's K/V for the whole prompt."""
        n = input_ids.shape[1]
        hooks = []
        for li in range(self.n_layers):
            attn = self.model.model.layers[li].self_attn

            def hook_fn(mod, args, kwargs, output, li=li):
                hidden = kwargs["hidden_states"] if "hidden_states" in kwargs else args[0]
                k = mod.k_proj(hidden).view(-1, self.n_kv, self.d_head)
                v = mod.v_proj(hidden).view(-1, self.n_kv, self.d_head)
                win = self.windows[li]
                m = min(n, win.cap)
                win.pos = n - m  # the ring holds the last m tokens in the slots a full write leaves them in
                win.batch_append(self._rotate(k[n - m:].float(), n - m), v[n - m:].float())
                ret = self.retrievals[li]
                ret.set_rotary_tables(self.cos_tbl, self.sin_tbl)
                if n > self.window_size:
                    n_ret = n - self.window_size
                    ret.calibrate(k)
                    ret.batch_append(k[:n_ret], v[:n_ret])

            hooks.append(attn.register_forward_hook(hook_fn, with_kwargs=True))
        try:
            self.model(input_ids, logits_to_keep=1)
        finally:
            for h in hooks:
                h.remove()
        self._context_len = n
        self._prefill_done = True
        if n > self.window_size:
            self._retrieval_built = True

    # ------------------------------------------------------- save / load --
    def save_cache(self, path, extra=None):
        """Writes every layer's window and packed index plus the decode
        counters to `path` (kvr_b200.cache_io container); `extra` (a JSON
        value) is stored alongside and returned by load_cache."""
        from .cache_io import write_cache

        meta = {"n_layers": self.n_layers, "n_kv": self.n_kv, "d_head": self.d_head,
                "window_size": self.window_size, "codec": self.codec, "tile": self.tile,
                "transform": self.transform, "context_len": self._context_len, "step": self._step,
                "retrieval_built": self._retrieval_built, "prefill_done": self._prefill_done, "layers": [],
                "extra": extra}
        tensors = {}
        for li in range(self.n_layers):
            wm, wt = self.windows[li].state_dict(f"L{li}.win.")
            rm, rt = self.retrievals[li].state_dict(f"L{li}.ret.")
            meta["layers"].append({"window": wm, "index": rm})
            tensors.update(wt)
            tensors.update(rt)
        write_cache(path, meta, tensors)

    def load_cache(self, path):
        """Restores a cache written by save_cache for the same model shape,
        window size and codec; decoding continues where it stopped."""
        from .cache_io import read_cache

        meta, tensors = read_cache(path)
        for key, mine in (("n_layers", self.n_layers), ("n_kv", self.n_kv), ("d_head", self.d_head),
                          ("window_size", self.window_size), ("codec", self.codec)):
            if meta[key] != mine:
                raise ValueError(f"cache {key}={meta[key]!r} does not match this hook ({mine!r})")
        for li in range(self.n_layers):
            self.windows[li].load_state_dict(meta["layers"][li]["window"], tensors, f"L{li}.win.")
            self.retrievals[li].load_state_dict(meta["layers"][li]["index"], tensors, f"L{li}.ret.")
            self.retrievals[li].set_rotary_tables(self.cos_tbl, self.sin_tbl)
        self._context_len, self._step = int(meta["context_len"]), int(meta["step"])
        self._retrieval_built, self._prefill_done = bool(meta["retrieval_built"]), bool(meta["prefill_done"])
        return meta.get("extra")

    def _update_stores(self, li, k_pre, v_val, k_post):
        """kvr_hook.py:136-148: on a full window, move the slot about to be
        overwritten into the index, then append the new token."""
        win = self.windows[li]
        if self._retrieval_built and win.n >= win.cap:
            slot = win.pos % win.cap
            old_pos = win.pos if self.reference_eviction_rope else win.pos - win.cap
            old_k_pre = self._rotate(win.k[slot].float().unsqueeze(0), old_pos, reverse=True)[0]
            self.retrievals[li].append(old_k_pre, win.v[slot].float())
        elif not self._retrieval_built and self._context_len >= self.window_size - 1 and li == 0:
            self._build_all_retrievals()
        win.append(k_post, v_val)

    def fused_store_update_ok(self, li):
        """True when decode_store_update can stand for RoPE + _update_stores:
        the 1-bit codec with eviction at the evicted token's own position, and
        no lazy index build due at this step."""
        if self.codec != "sd1" or self.reference_eviction_rope:
            return False
        win = self.windows[li]
        if not self._retrieval_built:
            return not (self._context_len >= self.window_size - 1 and li == 0) and win.n < win.cap
        return self.retrievals[li].store is not None

    def decode_store_update(self, li, q, k_pre, v, pos, write_kv=True):
        """One launch (kvr_decode_store_update) for what a decode step does
        between the projections and the attention (kvr_generator.py:91-98):
        RoPE of q and k at `pos`, eviction of the window slot about to be
        overwritten into the 1-bit index (its post-RoPE row goes to the pending
        tail as it is; a full tail is encoded into a tile), and the window
        write.  Returns the rotated q (model dtype)."""
        win, ret = self.windows[li], self.retrievals[li]
        evict = write_kv and self._retrieval_built and win.n >= win.cap
        slot = win.pos % win.cap
        tk = tv = None
        if evict:
            tk, tv = ret.tail_k[0], ret.tail_v[0]
        q_rot = K.decode_store_update(q, k_pre, v, self.cos_tbl, self.sin_tbl, pos, win.k, win.v, slot, tk, tv,
                                      ret.n_tail if evict else 0, write_kv)
        if evict:
            ret.n_tail += 1
            if ret.n_tail == ret.tile:
                st = ret.store
                if st.n_tiles + 1 > st.nt_cap:
                    st.grow(2 * st.nt_cap)
                K.sd1_encode(st, ret.tail_k, ret.tail_v)
                ret.n_stored += ret.tile
                ret.n_tail = 0
        if write_kv:
            win.pos += 1
            win.n = min(win.n + 1, win.cap)
        return q_rot

    def decode_step_fused(self, li, q, k_pre, v, pos):
        """The whole decode step of layer li after the projections in one
        launch where that applies (sd1 index built and active, eviction at
        the evicted token's own position): RoPE, eviction into the tail,
        window write, selection and attention
        (RetrievalIndex.decode_step).  Returns the (n_q, d) output in q's
        dtype, or None when the step must take the separate calls."""
        win, ret = self.windows[li], self.retrievals[li]
        if (self.codec != "sd1" or self.reference_eviction_rope or not self._retrieval_built or ret.store is None
                or self._ret_weight <= 0 or ret.n_tokens == 0):
            return None
        fills = win.n >= win.cap and ret.n_tail + 1 == ret.tile
        ex = exclusion_range(self._context_len, min(win.n + 1, win.cap), ret.n_stored + (ret.tile if fills else 0))
        out, _ = ret.decode_step(q, k_pre, v, win, pos, self.cos_tbl, self.sin_tbl, ex[0], ex[1])
        return out

    # ------------------------------------------------------- attention --
    def attend(self, li, q_post, out_dtype=torch.float32):
        """Window + retrieval attention of one layer for the current step:
        q_post (n_q, d) -> (n_q, d)."""
        win = self.windows[li]
        ret = self.retrievals[li]
        active = self._ret_weight > 0 and self._retrieval_built and ret.n_tokens > 0
        if active:
            ex = exclusion_range(self._context_len, win.n, ret.n_stored)
            return ret.attend(q_post, win, ex[0], ex[1], out_dtype=out_dtype)
        return K.decode_attn(q_post, [(win.k[:win.n], win.v[:win.n])], out_dtype=out_dtype, n_kv=self.n_kv)

    def register(self):
        for li in range(self.n_layers):
            attn = self.model.model.layers[li].self_attn
            self._hooks.append(attn.register_forward_hook(self._make_hook(li), with_kwargs=True))

    def _make_hook(self, li):
        def hook(mod, args, kwargs, output):
            hidden = kwargs["hidden_states"] if "hidden_states" in kwargs else args[0]
            T = hidden.shape[1]
            last = hidden[:, -1:, :]
            q = mod.q_proj(last).float().view(self.n_q, self.d_head)
            k_pre = mod.k_proj(last).float().view(self.n_kv, self.d_head)
            v = mod.v_proj(last).float().view(self.n_kv, self.d_head)
            pos = self._context_len if T == 1 else self._context_len - 1
            pe = kwargs.get("position_embeddings")
            if pe is not None:
                c, s = pe[0][0, -1:].float(), pe[1][0, -1:].float()
            else:
                c, s = self.cos_tbl[pos:pos + 1], self.sin_tbl[pos:pos + 1]
            q_rot = _apply_rotary(q, c, s)
            k_post = _apply_rotary(k_pre, c, s)
            if self._step > 0:
                self._update_stores(li, k_pre, v, k_post)
            out = self.attend(li, q_rot)
            fwr_proj = mod.o_proj(out.to(hidden.dtype).reshape(1, -1))
            layer = self.model.model.layers[li]
            if self.num_denoise_steps > 0 and not self.warmup_mode:
                h_in = last.reshape(1, -1)
                h = h_in + fwr_proj
                for _ in range(self.num_denoise_steps):
                    h = h + layer.mlp(layer.post_attention_layernorm(h))
                fwr_proj = h - h_in
            if self.warmup_mode:
                h_in = last.reshape(1, -1)
                native = layer.post_attention_layernorm(h_in + output[0][:, -1, :])
                mine = layer.post_attention_layernorm(h_in + fwr_proj)
                self.mlp_adapter_data[li].append((mine.detach().cpu(), native.detach().cpu()))
                return output
            if self.calib_s is not None:
                fwr_proj = fwr_proj * self.calib_s[li].to(fwr_proj.device) + self.calib_b[li].to(fwr_proj.device)
            new_attn = output[0].clone()
            new_attn[:, -1, :] = fwr_proj
            return (new_attn,) + tuple(output[1:])

        return hook

    def remove(self):
        for h in self._hooks:
            h.remove()
        self._hooks = []
        for h in getattr(self, "_mlp_hooks", []):
            h.remove()
        self._mlp_hooks = []

    def reset(self):
        self._context_len = 0
        self._prefill_done = False
        self._step = 0
        self._retrieval_built = False
        self.remove()
        self._new_stores()

    # ---------------------------------------- quality experiments (torch) --
    def fit_calibration(self):
        """Per-layer, per-dimension least squares native ~ s*kvr + b
        (kvr_hook.py:157-172)."""
        self.calib_s, self.calib_b = [None] * self.n_layers, [None] * self.n_layers
        for li in range(self.n_layers):
            x = torch.stack(self.calib_kvr[li]).float()
            y = torch.stack(self.calib_native[li]).float()
            xc, yc = x - x.mean(0), y - y.mean(0)
            s = (xc * yc).sum(0) / ((xc ** 2).sum(0) + 1e-8)
            self.calib_s[li], self.calib_b[li] = s, y.mean(0) - s * x.mean(0)

    def fit_mlp_adapters(self, lr=0.01, epochs=200):
        """Tiny per-layer MLP mapping the KVR MLP input toward native
        (kvr_hook.py:174-193)."""
        self.adapters = [None] * self.n_layers
        for li in range(self.n_layers):
            data = self.mlp_adapter_data[li]
            if len(data) < 3:
                continue
            x = torch.stack([p[0] for p in data]).float()
            y = torch.stack([p[1] for p in data]).float()
            net = nn.Sequential(nn.Linear(x.shape[-1], 16), nn.ReLU(), nn.Linear(16, x.shape[-1]))
            opt = torch.optim.Adam(net.parameters(), lr=lr)
            for _ in range(epochs):
                loss = F.mse_loss(net(x), y)
                opt.zero_grad()
                loss.backward()
                opt.step()
            self.adapters[li] = net

    def register_mlp_hooks(self):
        """Apply the adapters to each MLP input (kvr_hook.py:195-214)."""
        self._mlp_hooks = []
        for li in range(self.n_layers):
            net = self.adapters[li]
            if net is None:
                continue
            net = net.to(self.device)
            mlp = self.model.model.layers[li].mlp
            busy = [False]

            def hook(mod, args, output, net=net, busy=busy):
                if busy[0]:
                    return output
                busy[0] = True
                try:
                    return mod.__class__.forward(mod, net(args[0].float()).to(args[0].dtype))
                finally:
                    busy[0] = False

            self._mlp_hooks.append(mlp.register_forward_hook(hook))

    def __repr__(self):
        state = "ready" if self._retrieval_built else "lazy"
        return (f"KVRHook(layers={self.n_layers}, window={self.window_size}, top_k={self.top_k}, "
                f"ctx={self._context_len}, ret={state}, codec={self.codec})")

"""KVRGenerator — hand-rolled incremental decoding with window + retrieval
attention.  Drop-in for modules/kvr_generator.py (same constructor, prefill,
step, generate).

Per step and layer (modules/kvr_generator.py:78-126): input norm, q/k/v
projections, RoPE at the step position, store update (eviction into the
index), then attention over the window and the retrieved tokens — here one
call into the B200 kernels (RetrievalIndex.attend) instead of ``torch.cat``
+ the Triton kernel — then o_proj, residual and MLP.  With ``codec='sd1'``,
once the 1-bit index is active, RoPE, eviction, window write, selection and
attention are one kernel per layer (RetrievalIndex.decode_step); before that
the RoPE, the eviction and the window write are one kernel
(kvr_decode_store_update).  Sampling uses the HF logits processors, as the reference
does (modules/kvr_generator.py:129-154).
"""
import torch
import torch.nn.functional as F
from transformers import LogitsProcessorList, RepetitionPenaltyLogitsProcessor
from transformers import TemperatureLogitsWarper, TopKLogitsWarper, TopPLogitsWarper

from .kvr_hook import KVRHook
from .kvr_retrieval import _apply_rotary


class KVRGenerator:
    def __init__(self, model, window_size=2048, top_k=128, device=None, **kwargs):
        self.model = model
        self.device = device or model.device
        cfg = model.config
        self.n_layers = cfg.num_hidden_layers
        self.n_kv = cfg.num_key_value_heads
        self.n_q = cfg.num_attention_heads
        self.d_head = getattr(cfg, "head_dim", None) or (cfg.hidden_size // self.n_q)
        self.hidden_size = cfg.hidden_size
        self.g = self.n_q // self.n_kv
        self.vocab_size = cfg.vocab_size
        self._step_count = 0
        self._generated_ids = []
        self._is_first = True
        # codec='sd1': one fused kernel per layer for RoPE + store update
        # (fused_store_update=False keeps the step-by-step torch path)
        self.fused_store_update = kwargs.pop("fused_store_update", True)
        self.kvr = KVRHook(model, window_size=window_size, top_k=top_k, device=device, **kwargs)
        self.window_size = window_size
        self.top_k = top_k
        self.embed = model.model.embed_tokens
        self.final_norm = model.model.norm
        self.lm_head = model.lm_head
        self.layers = model.model.layers

    @torch.no_grad()
    def prefill(self, input_ids):
        """kvr_generator.py:41-47."""
        self.kvr.prefill(input_ids)
        self._generated_ids = []
        self._step_count = 0
        self._is_first = True

    def save_cache(self, path):
        """Saves the compressed KV state (KVRHook.save_cache) and this
        generator's step counters, so that decoding can resume later."""
        self.kvr.save_cache(path, extra={"is_first": self._is_first, "step_count": self._step_count,
                                         "generated_ids": [int(i) for i in self._generated_ids]})

    def load_cache(self, path):
        extra = self.kvr.load_cache(path) or {}
        self._is_first = bool(extra.get("is_first", False))
        self._step_count = int(extra.get("step_count", 0))
        self._generated_ids = list(extra.get("generated_ids", []))

    @torch.no_grad()
    def logits_step(self, token_id):
        """One incremental forward pass; returns the (vocab,) fp32 logits."""
        if isinstance(token_id, int):
            token_id = torch.tensor([[token_id]], device=self.device)
        elif token_id.dim() == 0:
            token_id = token_id.view(1, 1)
        elif token_id.dim() == 1:
            token_id = token_id.view(1, -1)
        h = self.embed(token_id)[0, 0]
        pos = self.kvr._context_len
        c = self.kvr.cos_tbl[pos:pos + 1].to(h.dtype)
        s = self.kvr.sin_tbl[pos:pos + 1].to(h.dtype)
        for li, layer in enumerate(self.layers):
            attn = layer.self_attn
            hn = layer.input_layernorm(h)
            q = attn.q_proj(hn).view(self.n_q, self.d_head)
            k_pre = attn.k_proj(hn).view(self.n_kv, self.d_head)
            v = attn.v_proj(hn).view(self.n_kv, self.d_head)
            out = None
            if self.fused_store_update and not self._is_first:
                # store update + selection + attention in one kernel
                out = self.kvr.decode_step_fused(li, q, k_pre, v, pos)
            if out is None:
                if self.fused_store_update and self.kvr.fused_store_update_ok(li):
                    # RoPE + eviction + window write in one kernel (kvr_decode_store_update)
                    q_rot = self.kvr.decode_store_update(li, q, k_pre, v, pos, write_kv=not self._is_first)
                else:
                    q_rot = _apply_rotary(q, c, s)
                    k_rot = _apply_rotary(k_pre, c, s)
                    if not self._is_first:
                        self.kvr._update_stores(li, k_pre.to(torch.float16), v.to(torch.float16),
                                                k_rot.to(torch.float16))
                out = self.kvr.attend(li, q_rot, out_dtype=q_rot.dtype)
            h = h + attn.o_proj(out.reshape(-1).to(h.dtype))
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        return self.lm_head(self.final_norm(h)).float()

    @torch.no_grad()
    def step(self, token_id=None, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0):
        """kvr_generator.py:49-161: returns the sampled next id, shape (1,)."""
        if token_id is None:
            if not self._generated_ids:
                raise ValueError("First step requires token_id")
            token_id = self._generated_ids[-1]
        logits = self.logits_step(token_id)
        procs = LogitsProcessorList()
        if repetition_penalty != 1.0:
            procs.append(RepetitionPenaltyLogitsProcessor(repetition_penalty))
        if temperature != 1.0:
            procs.append(TemperatureLogitsWarper(temperature))
        if top_k > 0:
            procs.append(TopKLogitsWarper(top_k))
        if top_p < 1.0:
            procs.append(TopPLogitsWarper(top_p))
        if self._generated_ids:
            ids = torch.tensor(self._generated_ids, device=self.device).unsqueeze(0)
        else:
            ids = torch.as_tensor(token_id, device=self.device).view(1, -1)
        for proc in procs:
            logits = proc(ids, logits.unsqueeze(0))[0]
        next_id = torch.multinomial(F.softmax(logits, dim=-1), 1)
        self._generated_ids.append(next_id.item())
        self._step_count += 1
        self.kvr._context_len += 1
        self._is_first = False
        return next_id

    @torch.no_grad()
    def generate(self, max_new_tokens=100, temperature=1.0, top_k=0, top_p=1.0, repetition_penalty=1.0):
        """kvr_generator.py:163-173."""
        out = [self.step(temperature=temperature, top_k=top_k, top_p=top_p, repetition_penalty=repetition_penalty)
               for _ in range(max_new_tokens)]
        return torch.cat(out)

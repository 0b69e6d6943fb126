"""Qwen3-VL-MoE text stack (REF cuda_qwen3_vl/models/moe.py:18-100).

``CudaQwen3VLMoeModel(cfg).forward(input_ids, pixel_values, vision_position_ids,
image_token_mask, position_ids, past_key_values, return_kv)`` returns
``(logits, router_logits_list[, new_kvs])`` like the reference.  With
``pixel_values`` and ``image_token_mask`` the vision tower (``vision.py``; its
grid (t, h, w) per image passed as ``vision_position_ids``, as in the
reference) replaces the embeddings of the image tokens with its merged
features.  ``vision=False`` builds a text-only model (``visual`` is None).
"""
from __future__ import annotations

import torch
from torch import nn

from .configs import MoETextConfig, Qwen3VLConfig
from .kv_cache import KVCache
from .modules import CudaEmbedding, CudaLinear, CudaRMSNorm, CudaTextDecoderLayer, TextMRoPE


def _layer_uses_moe(cfg: MoETextConfig, layer_idx: int) -> bool:
    """MoE on layers with (i+1) % decoder_sparse_step == 0 outside mlp_only_layers
    (REF models/moe.py:18-23)."""
    if cfg.num_experts <= 0:
        return False
    if layer_idx in cfg.mlp_only_layers:
        return False
    return ((layer_idx + 1) % cfg.decoder_sparse_step) == 0


class CudaQwen3VLMoeModel(nn.Module):
    def __init__(self, cfg: Qwen3VLConfig, expert_group=None, vision: bool = True) -> None:
        """``expert_group`` shards every MoE layer's experts over that process
        group (expert parallelism); attention and the rest stay replicated.
        ``vision=False`` leaves the vision tower out (text-only use)."""
        super().__init__()
        if cfg.family != "moe" or not isinstance(cfg.text, MoETextConfig):
            raise ValueError(f"expected an MoE config, got {cfg.family}")
        self.cfg = cfg
        t = cfg.text
        if vision:
            from .vision import CudaVisionTower
            self.visual = CudaVisionTower(cfg.vision)
        else:
            self.visual = None
        self.embed_tokens = CudaEmbedding(t.vocab_size, t.hidden_size)
        self.rotary = TextMRoPE(t.head_dim, theta=t.rope_theta, mrope_section=t.mrope_section)
        self.layers = nn.ModuleList([
            CudaTextDecoderLayer(
                hidden_size=t.hidden_size, num_heads=t.num_heads, num_kv_heads=t.num_kv_heads,
                head_dim=t.head_dim, intermediate_size=t.intermediate_size,
                rms_norm_eps=t.rms_norm_eps, use_moe=_layer_uses_moe(t, i),
                num_experts=t.num_experts, top_k=t.num_experts_per_tok,
                moe_intermediate_size=t.moe_intermediate_size, attention_bias=t.attention_bias,
                expert_group=expert_group)
            for i in range(t.num_layers)
        ])
        self.norm = CudaRMSNorm(t.hidden_size, eps=t.rms_norm_eps)
        self.lm_head = CudaLinear(t.hidden_size, t.vocab_size, bias=False)
        if t.tie_word_embeddings:
            self.lm_head.weight = self.embed_tokens.weight

    def _text_forward(self, input_embeds: torch.Tensor, position_ids: torch.Tensor,
                      past_key_values=None):
        x = input_embeds
        mrope_fn = self.rotary.bind(position_ids)
        router_logits_all: list[torch.Tensor] = []
        new_kvs: list[tuple[torch.Tensor, torch.Tensor]] = []
        for i, layer in enumerate(self.layers):
            layer_past = past_key_values[i] if past_key_values is not None else None
            x, rl, new_kv = layer(x, mrope_fn, past_kv=layer_past)
            if rl is not None:
                router_logits_all.append(rl)
            new_kvs.append(new_kv)
        return self.norm(x), router_logits_all, new_kvs

    def forward(self, input_ids: torch.Tensor | None = None, pixel_values=None,
                vision_position_ids=None, image_token_mask=None, position_ids=None,
                past_key_values=None, return_kv: bool = False, inputs_embeds=None):
        if inputs_embeds is None:
            if input_ids is None:
                raise ValueError("input_ids or inputs_embeds is required")
            inputs_embeds = self.embed_tokens(input_ids)
        if pixel_values is not None and image_token_mask is not None:
            # REF models/moe.py:87-90 (the reference unpacks two of the tower's
            # three outputs there; the merged features are its first)
            if self.visual is None:
                raise RuntimeError("this model was built with vision=False")
            feats = self.visual(pixel_values, vision_position_ids)[0]
            inputs_embeds = inputs_embeds.clone()
            inputs_embeds[image_token_mask] = feats.to(inputs_embeds.dtype)
        B, S = inputs_embeds.shape[:2]
        if position_ids is None:
            past_len = past_key_values[0][0].shape[2] if past_key_values else 0
            pos = torch.arange(past_len, past_len + S, device=inputs_embeds.device)
            pos = pos.unsqueeze(0).expand(B, S)
            position_ids = torch.stack([pos, pos, pos], dim=0)
        hidden, router_logits, new_kvs = self._text_forward(inputs_embeds, position_ids,
                                                            past_key_values=past_key_values)
        logits = self.lm_head(hidden)
        if return_kv:
            return logits, router_logits, new_kvs
        return logits, router_logits

    def make_kv_cache(self, batch: int, capacity: int, device=None) -> KVCache:
        """A zeroed ``KVCache`` for every layer of this model (bf16)."""
        t = self.cfg.text
        device = device or self.embed_tokens.weight.device
        return KVCache(len(self.layers), batch, t.num_kv_heads, capacity, t.head_dim, device)

    def _last_logits(self, input_ids: torch.Tensor, cache) -> torch.Tensor:
        """Logits of the last position only (B, vocab): the forward of
        ``forward(input_ids, past_key_values=cache)`` with the lm_head applied to
        the last hidden row instead of all of them."""
        B, S = input_ids.shape
        emb = self.embed_tokens(input_ids)
        past_len = cache.length if cache is not None else 0
        pos = torch.arange(past_len, past_len + S, device=emb.device).unsqueeze(0).expand(B, S)
        hidden, _, _ = self._text_forward(emb, torch.stack([pos, pos, pos], dim=0),
                                          past_key_values=cache)
        return self.lm_head(hidden[:, -1:].contiguous())[:, 0]

    @torch.no_grad()
    def generate(self, input_ids: torch.Tensor, max_new_tokens: int, eos_token_id: int | None = None,
                 kv_cache: KVCache | None = None) -> torch.Tensor:
        """Greedy decoding: one prefill over ``input_ids`` (B, S), then one token
        per step with the K/V history kept in a preallocated ``KVCache``
        (capacity S + max_new_tokens unless ``kv_cache`` is given).  Returns
        (B, S + n) token ids; stops early once every sequence has produced
        ``eos_token_id``.  The reference generates only with its dense model
        (REF models/dense.py:123-162); this is the same greedy loop for the MoE
        model."""
        B, S = input_ids.shape
        if max_new_tokens < 1:
            return input_ids
        cache = kv_cache if kv_cache is not None else self.make_kv_cache(B, S + max_new_tokens,
                                                                         input_ids.device)
        if cache.length + S + max_new_tokens - 1 > cache[0].capacity:
            raise RuntimeError("generate: the KV cache is too small for the requested tokens")
        nxt = self._last_logits(input_ids, cache).argmax(dim=-1)
        out = [nxt]
        done = (nxt == eos_token_id) if eos_token_id is not None else None
        for _ in range(max_new_tokens - 1):
            if done is not None and bool(done.all()):
                break
            nxt = self._last_logits(nxt[:, None], cache).argmax(dim=-1)
            if done is not None:
                nxt = torch.where(done, torch.full_like(nxt, eos_token_id), nxt)
                done = done | (nxt == eos_token_id)
            out.append(nxt)
        return torch.cat([input_ids, torch.stack(out, dim=1).to(input_ids.dtype)], dim=1)

"""nn.Module drop-ins for the Qwen3-VL-MoE text decoder layer.

Class names, constructor arguments, parameter names/shapes and forward
signatures follow the reference (REF cuda_qwen3_vl/modules/{norms,linear,
embedding,rotary,attention,moe,mlp,text_decoder}.py), so ``load_state_dict``
of a reference (or HF-remapped) state dict works unchanged.  The compute runs
in libq35b200 kernels; there is no torch fallback.

Deliberate differences from the reference, all documented on the class:
  * activations and weights must be bf16 CUDA tensors (``module.to("cuda",
    torch.bfloat16)``); the MoE router weight stays fp32 and router_logits are
    returned in fp32;
  * chunked prefill with a cache (S_q > 1 and a past) uses a bottom-right
    aligned causal mask; the reference turns such a call fully non-causal
    (REF modules/attention.py:95).  ``CudaFullAttention.reference_chunk_mask``
    restores the reference's behaviour.
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import kernels as K
from .kv_cache import LayerKVCache


# ------------------------------------------------------------------ norms
class CudaRMSNorm(nn.Module):
    """y = x * rsqrt(mean(x^2) + eps) * weight (REF modules/norms.py:9-22)."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.dim = dim
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return K.rmsnorm(x, self.weight, self.eps)

    def extra_repr(self) -> str:
        return f"{self.dim}, eps={self.eps}"


# ------------------------------------------------------------------ linear
class CudaLinear(nn.Module):
    """nn.Linear layout (weight (out, in), optional bias), tcgen05 GEMM
    (REF modules/linear.py:11-39)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features))
        else:
            self.register_parameter("bias", None)
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in = self.weight.shape[1]
            bound = 1.0 / math.sqrt(fan_in) if fan_in > 0 else 0.0
            nn.init.uniform_(self.bias, -bound, bound)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None,
                out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        return K.matmul(x, self.weight, self.bias, residual=residual, out_dtype=out_dtype)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, bias={self.bias is not None}"


class CudaEmbedding(nn.Module):
    """Token embedding gather (REF modules/embedding.py:9-30); the gather runs in
    the row-gather kernel."""

    def __init__(self, num_embeddings: int, embedding_dim: int, padding_idx: int | None = None) -> None:
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.padding_idx = padding_idx
        self.weight = nn.Parameter(torch.empty(num_embeddings, embedding_dim))
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.normal_(self.weight)
        if self.padding_idx is not None:
            with torch.no_grad():
                self.weight[self.padding_idx].zero_()

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """Row gather with the id range checked on the device (no host
        synchronisation): an id outside [0, num_embeddings) yields a zero row and
        is reported through the device error word (``kernels.device_error_check``)."""
        out = K.embedding(ids, self.weight)
        return out


# ------------------------------------------------------------------ rotary
class BoundMRoPE:
    """The ``mrope_apply(q, k)`` callable of one forward, bound to its position
    ids.  CudaFullAttention recognises it and fuses the rotation into its
    QK-norm kernel; calling it directly applies the rotation like
    ``TextMRoPE.apply``."""

    __slots__ = ("rotary", "position_ids")

    def __init__(self, rotary: "TextMRoPE", position_ids: torch.Tensor) -> None:
        self.rotary = rotary
        self.position_ids = position_ids

    def __call__(self, q: torch.Tensor, k: torch.Tensor):
        return self.rotary.apply(q, k, self.position_ids)


class TextMRoPE(nn.Module):
    """Text mRoPE over (3, B, S) positions (REF modules/rotary.py:34-59).

    ``interleaved=False`` (default) is the reference's chunked section layout
    (REF kernels/mrope.py:19-35); ``interleaved=True`` is HF Qwen3-VL's T/H/W
    interleave.  The two agree whenever t == h == w.
    """

    def __init__(self, dim: int, theta: float = 500000.0, mrope_section: list[int] | None = None,
                 interleaved: bool = False) -> None:
        super().__init__()
        self.dim = dim
        self.theta = theta
        self.mrope_section = list(mrope_section or [24, 20, 20])
        self.interleaved = interleaved
        inv_freq = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    def _apply(self, fn, recurse=True):
        inv = self.inv_freq
        out = super()._apply(fn, recurse)
        # inv_freq is part of the rotary math: keep it fp32 whatever the module dtype.
        if self.inv_freq.dtype != torch.float32:
            self.inv_freq = inv.to(device=self.inv_freq.device, dtype=torch.float32)
        return out

    def compute_cos_sin(self, position_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """(3,B,S) positions -> cos, sin of shape (3,B,S,dim), fp32 (API parity
        with REF modules/rotary.py:46-55; the kernels compute these on the fly)."""
        freqs = position_ids.float().unsqueeze(-1) * self.inv_freq.to(position_ids.device)
        emb = torch.cat([freqs, freqs], dim=-1)
        return emb.cos(), emb.sin()

    def apply(self, q: torch.Tensor, k: torch.Tensor, position_ids: torch.Tensor):
        return (K.mrope(q, position_ids, self.inv_freq, self.mrope_section, self.interleaved),
                K.mrope(k, position_ids, self.inv_freq, self.mrope_section, self.interleaved))

    def bind(self, position_ids: torch.Tensor) -> BoundMRoPE:
        return BoundMRoPE(self, position_ids)


# ------------------------------------------------------------------ MLPs
class CudaSwiGLUMLP(nn.Module):
    """Dense SwiGLU MLP of non-MoE layers (REF modules/mlp.py:10-22)."""

    def __init__(self, hidden_size: int, intermediate_size: int, bias: bool = False) -> None:
        super().__init__()
        self.gate_proj = CudaLinear(hidden_size, intermediate_size, bias=bias)
        self.up_proj = CudaLinear(hidden_size, intermediate_size, bias=bias)
        self.down_proj = CudaLinear(intermediate_size, hidden_size, bias=bias)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        act = K.swiglu(self.gate_proj(x), self.up_proj(x))
        return self.down_proj(act, residual=residual)


# ------------------------------------------------------------------ attention
def _params_key(*ps: torch.Tensor) -> tuple:
    return tuple((p.data_ptr(), p._version, p.dtype, p.device) for p in ps)


class CudaFullAttention(nn.Module):
    """Causal GQA text attention with per-head QK RMSNorm and mRoPE
    (REF modules/attention.py:45-98).

    ``forward(x, mrope_apply, past_kv=None) -> (o_proj(out), (k, v))`` with
    k, v of shape (B, Hkv, S_past + S, D).  When ``mrope_apply`` is a
    ``BoundMRoPE`` (what CudaQwen3VLMoeModel passes) the q/k/v projections run
    as one GEMM and QK-norm + mRoPE + the head-major split run in one kernel;
    any other callable gets the unfused path: separate projections, QK-norm,
    then ``mrope_apply(q, k)`` on (B, H, S, D) tensors.
    """

    reference_chunk_mask = False

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int | None = None,
                 rms_norm_eps: float = 1e-6, attention_bias: bool = False) -> None:
        super().__init__()
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.num_kv_groups = num_heads // num_kv_heads
        self.head_dim = head_dim or (hidden_size // num_heads)
        self.scale = self.head_dim ** -0.5
        self.q_proj = CudaLinear(hidden_size, num_heads * self.head_dim, bias=attention_bias)
        self.k_proj = CudaLinear(hidden_size, num_kv_heads * self.head_dim, bias=attention_bias)
        self.v_proj = CudaLinear(hidden_size, num_kv_heads * self.head_dim, bias=attention_bias)
        self.o_proj = CudaLinear(num_heads * self.head_dim, hidden_size, bias=attention_bias)
        self.q_norm = CudaRMSNorm(self.head_dim, eps=rms_norm_eps)
        self.k_norm = CudaRMSNorm(self.head_dim, eps=rms_norm_eps)
        self._qkv_cache: tuple | None = None

    # prefill (>= 256 tokens, head_dim 128): QK-norm + mRoPE in the projection
    # GEMM's epilogue instead of a separate pass over the bf16 projection
    fuse_qkv_epilogue = True

    def _qkv_weight(self) -> tuple[torch.Tensor, torch.Tensor | None]:
        """Concatenated (q; k; v) projection weight (and bias), rebuilt whenever a
        source parameter is replaced or modified in place."""
        ps = [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight]
        bs = [self.q_proj.bias, self.k_proj.bias, self.v_proj.bias]
        key = _params_key(*ps, *[b for b in bs if b is not None])
        if self._qkv_cache is None or self._qkv_cache[0] != key:
            with torch.no_grad():
                w = torch.cat([p.detach() for p in ps], dim=0).contiguous()
                b = None if bs[0] is None else torch.cat([t.detach() for t in bs]).contiguous()
            self._qkv_cache = (key, w, b)
        return self._qkv_cache[1], self._qkv_cache[2]

    def _project(self, x: torch.Tensor, mrope_apply):
        B, S, _ = x.shape
        Hq, Hkv, D = self.num_heads, self.num_kv_heads, self.head_dim
        if isinstance(mrope_apply, BoundMRoPE):
            w, b = self._qkv_weight()
            rot = mrope_apply.rotary
            pos = mrope_apply.position_ids
            if pos.shape != (3, B, S):
                raise RuntimeError(f"position_ids must be (3, {B}, {S}), got {tuple(pos.shape)}")
            if (self.fuse_qkv_epilogue and D == 128 and b is None and (Hq + 2 * Hkv) % 2 == 0
                    and B * S >= 256 and x.shape[-1] % 8 == 0):
                return K.qkv_proj_norm_rope(x, w, self.q_norm.weight, self.k_norm.weight, pos,
                                            rot.inv_freq, rot.mrope_section, Hq, Hkv,
                                            self.q_norm.eps, rot.interleaved)
            qkv = K.matmul(x, w, b)
            return K.qknorm_mrope(qkv, self.q_norm.weight, self.k_norm.weight, pos, rot.inv_freq,
                                  rot.mrope_section, B, S, Hq, Hkv, D, self.q_norm.eps,
                                  rot.interleaved)
        q = self.q_proj(x).reshape(B, S, Hq, D)
        k = self.k_proj(x).reshape(B, S, Hkv, D)
        v = self.v_proj(x).reshape(B, S, Hkv, D)
        q = self.q_norm(q).transpose(1, 2)
        k = self.k_norm(k).transpose(1, 2)
        q, k = mrope_apply(q.contiguous(), k.contiguous())
        return q.contiguous(), k.contiguous(), v.transpose(1, 2).contiguous()

    def forward(self, x: torch.Tensor, mrope_apply, past_kv: tuple[torch.Tensor, torch.Tensor] | None = None,
                residual: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16):
        """``residual`` (optional, same shape as x) is added in the o_proj
        epilogue and ``out_dtype`` may be fp32: the decoder layer uses both to
        fuse its residual add and keep the post-attention residual in fp32."""
        B, S, _ = x.shape
        q, k, v = self._project(x, mrope_apply)
        if isinstance(past_kv, LayerKVCache):
            # preallocated cache: append in place, attend over the buffers
            cache = past_kv
            Sk = cache.length + S
            if Sk > cache.capacity:
                raise RuntimeError(f"KV cache full: {cache.length} + {S} > {cache.capacity}")
            K.kv_append(k, v, cache.k, cache.v, cache.length)
            causal = (S == Sk) if self.reference_chunk_mask else S > 1
            out = K.attention_cache(q, cache.k, cache.v, Sk, self.scale, causal)
            cache.length = Sk
            return self.o_proj(out, residual=residual, out_dtype=out_dtype), cache
        if past_kv is not None:
            past_k, past_v = past_kv
            k = torch.cat([past_k, k], dim=2)
            v = torch.cat([past_v, v], dim=2)
        new_kv = (k, v)
        Sk = k.shape[2]
        if self.reference_chunk_mask:
            causal = S == Sk
        else:
            causal = S > 1
        out = K.attention_tokens(q, k, v, self.scale, causal)
        return self.o_proj(out, residual=residual, out_dtype=out_dtype), new_kv


# ------------------------------------------------------------------ MoE
class CudaSparseMoE(nn.Module):
    """Top-k routed experts with SwiGLU (REF modules/moe.py:26-85).

    Parameters: ``gate_weight`` (E, H) -- kept fp32 even after
    ``.to(torch.bfloat16)``, the router is an fp32 GEMV; ``gate_up_proj``
    (E, 2I, H) and ``down_proj`` (E, H, I), bf16 for the kernels.
    ``forward(x (B,S,H)) -> (out (B,S,H), router_logits (B*S, E) fp32)``.

    Pipeline (no host synchronisation): fused router (logits, softmax, top-k,
    renormalise) -> (expert, token) permutation -> row gather -> grouped
    gate_up GEMM with SwiGLU epilogue -> grouped down GEMM -> weighted fp32
    combine (+ residual when called from the decoder layer).

    ``router_bias`` (optional (E,) fp32 buffer, None by default) is added to
    the router logits; the benchmark harness uses it to skew expert load.
    """

    def __init__(self, hidden_size: int, moe_intermediate_size: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool = True) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.moe_intermediate_size = moe_intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.gate_weight = nn.Parameter(torch.empty(num_experts, hidden_size))
        self.gate_up_proj = nn.Parameter(torch.empty(num_experts, 2 * moe_intermediate_size, hidden_size))
        self.down_proj = nn.Parameter(torch.empty(num_experts, hidden_size, moe_intermediate_size))
        self.router_bias: torch.Tensor | None = None
        self.reset_parameters()

    def reset_parameters(self) -> None:
        nn.init.normal_(self.gate_weight, std=0.02)
        nn.init.normal_(self.gate_up_proj, std=0.02)
        nn.init.normal_(self.down_proj, std=0.02)

    def _apply(self, fn, recurse=True):
        gw = self.gate_weight.data
        rb = self.router_bias
        out = super()._apply(fn, recurse)
        new = self.gate_weight.data
        if new.dtype != torch.float32:
            self.gate_weight.data = gw.to(device=new.device, dtype=torch.float32)
        if rb is not None:
            self.router_bias = rb.to(device=new.device, dtype=torch.float32)
        return out

    def _gate_split(self):
        """bf16 [hi | mid | lo] planes of the fp32 gate weight for the tensor-core
        router (rebuilt when the weight is replaced or modified in place)."""
        H, E = self.hidden_size, self.num_experts
        if H % 64 or E % 32:
            return None
        key = _params_key(self.gate_weight)
        cache = getattr(self, "_split_cache", None)
        if cache is None or cache[0] != key:
            with torch.no_grad():
                cache = (key, K.router_split_weights(self.gate_weight.detach()))
            self._split_cache = cache
        return cache[1]

    pack_expert_weights = False

    def _packed_experts(self):
        """Tile-packed copies of gate_up_proj / down_proj (contiguous 16 KB TMA
        boxes), rebuilt when a weight is replaced or modified in place.  Off by
        default: it costs one extra copy of the expert weights and measured no
        faster than streaming the parameters (``pack_expert_weights = True``
        enables it)."""
        I, H = self.moe_intermediate_size, self.hidden_size
        if not self.pack_expert_weights or I % 128 or H % 128:
            return None, None
        key = _params_key(self.gate_up_proj, self.down_proj)
        cache = getattr(self, "_pack_cache", None)
        if cache is None or cache[0] != key:
            with torch.no_grad():
                cache = (key, K.pack_b_tiles(self.gate_up_proj.detach()),
                         K.pack_b_tiles(self.down_proj.detach()))
            self._pack_cache = cache
        return cache[1], cache[2]

    def route(self, x2d: torch.Tensor, chunk_counts: bool = False):
        """Router only: (logits fp32 (T,E), top-k ids int32 (T,k), weights fp32 (T,k));
        with ``chunk_counts`` also the per-chunk expert counts for the one-launch
        permutation (None when the shape takes another router path)."""
        return K.router_topk(x2d, self.gate_weight, self.top_k, self.norm_topk_prob,
                             bias=self.router_bias, gate_split=self._gate_split(),
                             chunk_counts=chunk_counts)

    def experts(self, x2d: torch.Tensor, idx: torch.Tensor, weights: torch.Tensor,
                residual: torch.Tensor | None = None,
                chunk_counts: torch.Tensor | None = None) -> torch.Tensor:
        """Expert compute + weighted combine for routed tokens (T,H) -> (T,H)."""
        T, H = x2d.shape
        gu_p, dn_p = self._packed_experts()
        if chunk_counts is not None:
            perm = K.moe_permute_counted(idx, chunk_counts, self.num_experts)
        else:
            perm = K.moe_permute(idx, self.num_experts)
        xs = K.gather_rows(x2d, perm.sorted_tok)
        act = K.grouped_gateup_swiglu(xs, self.gate_up_proj, perm, w_packed=gu_p)
        y = K.grouped_down(act, self.down_proj, perm, w_packed=dn_p)
        return K.moe_combine(y, weights, perm.slot_pos, residual, T, H)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        B, S, H = x.shape
        x2d = x.reshape(-1, H)
        res2d = None if residual is None else residual.reshape(-1, H)
        if getattr(self, "exchange", None) is None:
            logits, idx, w, cc = self.route(x2d, chunk_counts=True)
            out = self.experts(x2d, idx, w, res2d, chunk_counts=cc)
        else:  # expert parallel: the receiving ranks permute what they receive
            logits, idx, w = self.route(x2d)
            out = self.experts(x2d, idx, w, res2d)
        return out.reshape(B, S, H), logits


# ------------------------------------------------------------------ decoder layer
class CudaTextDecoderLayer(nn.Module):
    """Pre-norm attention + residual, pre-norm MoE (or dense MLP) + residual
    (REF modules/text_decoder.py:14-65).  Both residual adds are fused into
    the producing kernels (o_proj epilogue, MoE combine), and the
    post-attention residual h = x + attn stays fp32 between them, so the
    layer output is rounded to bf16 once (the reference rounds h too)."""

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: int,
                 intermediate_size: int, rms_norm_eps: float, use_moe: bool = False,
                 num_experts: int = 0, top_k: int = 0, moe_intermediate_size: int = 0,
                 attention_bias: bool = False, expert_group=None, expert_placement=None) -> None:
        """``expert_group`` (a torch.distributed process group, optional) shards
        the MoE experts over its ranks (expert parallelism, see ep.py);
        ``expert_placement`` (optional) says which experts each rank owns."""
        super().__init__()
        self.input_layernorm = CudaRMSNorm(hidden_size, eps=rms_norm_eps)
        self.self_attn = CudaFullAttention(hidden_size=hidden_size, num_heads=num_heads,
                                           num_kv_heads=num_kv_heads, head_dim=head_dim,
                                           rms_norm_eps=rms_norm_eps, attention_bias=attention_bias)
        self.post_attention_layernorm = CudaRMSNorm(hidden_size, eps=rms_norm_eps)
        if use_moe and expert_group is not None:
            from .ep import ExpertParallelSparseMoE
            self.mlp = ExpertParallelSparseMoE(hidden_size, moe_intermediate_size, num_experts, top_k,
                                               group=expert_group, expert_placement=expert_placement)
        elif use_moe:
            self.mlp = CudaSparseMoE(hidden_size=hidden_size, moe_intermediate_size=moe_intermediate_size,
                                     num_experts=num_experts, top_k=top_k)
        else:
            self.mlp = CudaSwiGLUMLP(hidden_size, intermediate_size)
        self.use_moe = use_moe

    def forward(self, x: torch.Tensor, mrope_apply, past_kv: tuple[torch.Tensor, torch.Tensor] | None = None):
        x = x.contiguous()
        h, new_kv = self.self_attn(self.input_layernorm(x), mrope_apply, past_kv=past_kv,
                                   residual=x, out_dtype=torch.float32)
        mlp_in = self.post_attention_layernorm(h)
        if self.use_moe:
            x, router_logits = self.mlp(mlp_in, residual=h)
        else:
            x, router_logits = self.mlp(mlp_in, residual=h.to(torch.bfloat16)), None
        return x, router_logits, new_kv

"""CPU oracle: fp32 restatement of the reference's decoder-layer forward.

TEST INFRASTRUCTURE ONLY.  Only tests/, __graft_entry__.smoke() and the CPU
baseline leg of bench.py may import this module, and only as the checker or
the timed CPU baseline; the product path never calls it.

Each function restates the torch branch that the reference's op wrappers take
for CPU tensors (file:line in luozoupi/Qwen3_5_VL_CUDA_CUSTOM, paths relative
to CUDA_qwen3_5-main/, REF below), computed in fp32.  The restatement is
pinned against fixtures produced by running the reference itself
(tests/golden/make_golden.py -> tests/golden/*.pt, checked by
tests/test_oracle_golden.py).

Deviation by design: top-k uses a stable descending sort, so ties go to the
lower expert index as in the reference's CUDA top-k kernel
(REF csrc/moe_routing_op.cu:36-53, strict '>' comparisons); the reference's
CPU branch calls torch.topk, whose tie order is unspecified.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """REF cuda_qwen3_vl/kernels/rmsnorm.py:12-17."""
    x = x.float()
    var = x.pow(2).mean(dim=-1, keepdim=True)
    return x * torch.rsqrt(var + eps) * w.float()


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """REF kernels/matmul.py:63-64 (F.linear)."""
    return F.linear(x.float(), w.float(), None if b is None else b.float())


def inv_freq(dim: int, theta: float) -> torch.Tensor:
    """REF modules/rotary.py:43-44."""
    return 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim))


def mrope_cos_sin(position_ids: torch.Tensor, inv: torch.Tensor):
    """REF modules/rotary.py:46-55: (3,B,S) -> cos, sin (3,B,S,D)."""
    freqs = position_ids.float().unsqueeze(-1) * inv
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def mrope_select(cos3: torch.Tensor, sin3: torch.Tensor, sections, interleaved: bool = False):
    """Chunked section layout of REF kernels/mrope.py:19-35 (sections * 2
    chunks, chunk i from axis i % 3).  interleaved=True: HF Qwen3-VL layout
    (H at index % 3 == 1 below 3*s1, W at index % 3 == 2 below 3*s2)."""
    if not interleaved:
        secs = list(sections) * 2
        cs, ss, off = [], [], 0
        for i, m in enumerate(secs):
            cs.append(cos3[i % 3, ..., off:off + m])
            ss.append(sin3[i % 3, ..., off:off + m])
            off += m
        return torch.cat(cs, dim=-1), torch.cat(ss, dim=-1)
    D = cos3.shape[-1]
    half = D // 2
    axis = torch.zeros(D, dtype=torch.long)
    for j in range(D):
        jj = j % half
        if jj % 3 == 1 and jj < 3 * sections[1]:
            axis[j] = 1
        elif jj % 3 == 2 and jj < 3 * sections[2]:
            axis[j] = 2
    idx = torch.arange(D)
    return cos3[axis, ..., idx].movedim(0, -1), sin3[axis, ..., idx].movedim(0, -1)


def rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """REF kernels/mrope.py:38-50 on x (B,H,S,D), cos/sin (B,S,D)."""
    D_rope = cos.shape[-1]
    half = D_rope // 2
    x1, x2 = x[..., :half], x[..., half:D_rope]
    c = cos.unsqueeze(1)[..., :half]
    s = sin.unsqueeze(1)[..., :half]
    rot = torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)
    return torch.cat([rot, x[..., D_rope:]], dim=-1)


def attention(q, k, v, scale: float, causal: bool) -> torch.Tensor:
    """Softmax attention with GQA expansion (REF kernels/flash_attention.py:13-18).
    The causal mask is bottom-right aligned (identical to SDPA's when Sq == Skv)."""
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    g = Hq // Hkv
    k = k[:, :, None].expand(B, Hkv, g, Skv, D).reshape(B, Hq, Skv, D)
    v = v[:, :, None].expand(B, Hkv, g, Skv, D).reshape(B, Hq, Skv, D)
    s = torch.matmul(q.float(), k.float().transpose(-1, -2)) * scale
    if causal:
        qi = torch.arange(Sq).unsqueeze(1)
        kj = torch.arange(Skv).unsqueeze(0)
        s = s.masked_fill(kj > qi + (Skv - Sq), float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.matmul(p, v.float())


def canonical_topk(p: torch.Tensor, k: int):
    """Top-k sorted descending, ties to the lower index (stable sort)."""
    vals, idx = torch.sort(p, dim=-1, descending=True, stable=True)
    return vals[..., :k], idx[..., :k]


def router(x2d: torch.Tensor, wg: torch.Tensor, k: int, renorm: bool = True,
           bias: torch.Tensor | None = None):
    """REF modules/moe.py:60-65 in fp32: logits, softmax, top-k, renormalise.
    Returns (logits, probs, top_idx, top_w)."""
    logits = linear(x2d, wg)
    if bias is not None:
        logits = logits + bias.float()
    p = torch.softmax(logits, dim=-1)
    vals, idx = canonical_topk(p, k)
    if renorm:
        vals = vals / vals.sum(dim=-1, keepdim=True)
    return logits, p, idx, vals


def permutation(idx: np.ndarray, E: int, tile_m: int = 128):
    """(expert, token) order of the routed pairs, as the reference's
    per-expert ``(top_idx == e).nonzero()`` loop visits them
    (REF modules/moe.py:71-76).  Integer work in numpy.
    Returns counts, offsets, sorted_tok, slot_pos, tile_offsets (all int32)."""
    idx = np.asarray(idx, dtype=np.int64)
    T, k = idx.shape
    flat = idx.reshape(-1)
    counts = np.bincount(flat, minlength=E).astype(np.int32)
    offsets = np.zeros(E + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    tok = np.repeat(np.arange(T), k)
    order = np.lexsort((tok, flat))  # primary key expert, then token
    sorted_tok = tok[order].astype(np.int32)
    slot_pos = np.empty(T * k, dtype=np.int32)
    slot_pos[order] = np.arange(T * k, dtype=np.int32)
    tiles = (counts + tile_m - 1) // tile_m
    tile_offsets = np.zeros(E + 1, dtype=np.int32)
    tile_offsets[1:] = np.cumsum(tiles)
    return counts, offsets, sorted_tok, slot_pos, tile_offsets


def moe(x2d: torch.Tensor, wg, gate_up, down, k: int, renorm: bool = True, bias=None,
        force_idx: torch.Tensor | None = None):
    """CudaSparseMoE.forward in fp32 (REF modules/moe.py:54-85).
    ``force_idx`` (T,k) replaces the top-k choice (the weights are still the
    oracle's own probabilities at those experts, renormalised): it isolates the
    discrete routing decision when comparing against another implementation.
    Returns (out (T,H), logits (T,E), top_idx, top_w, probs)."""
    x2d = x2d.float()
    logits, p, idx, w = router(x2d, wg, k, renorm, bias)
    if force_idx is not None:
        idx = force_idx.long()
        w = torch.gather(p, 1, idx)
        if renorm:
            w = w / w.sum(dim=-1, keepdim=True)
    I = gate_up.shape[1] // 2
    final = torch.zeros_like(x2d)
    for e in range(gate_up.shape[0]):
        mask = idx == e
        if not bool(mask.any()):
            continue
        tok, slot = mask.nonzero(as_tuple=True)
        gu = linear(x2d[tok], gate_up[e])
        act = F.silu(gu[:, :I]) * gu[:, I:]
        out = linear(act, down[e])
        final.index_add_(0, tok, out * w[tok, slot, None])
    return final, logits, idx, w, p


def attention_block(x: torch.Tensor, P: dict, cfg, position_ids, past_kv=None,
                    interleaved: bool = False, prefix: str = "self_attn."):
    """CudaFullAttention.forward in fp32 (REF modules/attention.py:75-98),
    bottom-right causal whenever S > 1.  Returns (o_proj(out), (k, v))."""
    B, S, _ = x.shape
    Hq, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
    eps = cfg.rms_norm_eps
    q = linear(x, P[prefix + "q_proj.weight"]).reshape(B, S, Hq, D)
    k = linear(x, P[prefix + "k_proj.weight"]).reshape(B, S, Hkv, D)
    v = linear(x, P[prefix + "v_proj.weight"]).reshape(B, S, Hkv, D)
    q = rmsnorm(q, P[prefix + "q_norm.weight"], eps).transpose(1, 2)
    k = rmsnorm(k, P[prefix + "k_norm.weight"], eps).transpose(1, 2)
    v = v.transpose(1, 2)
    cos3, sin3 = mrope_cos_sin(position_ids, inv_freq(D, cfg.rope_theta))
    cos, sin = mrope_select(cos3, sin3, cfg.mrope_section, interleaved)
    q, k = rotate(q, cos, sin), rotate(k, cos, sin)
    if past_kv is not None:
        k = torch.cat([past_kv[0].float(), k], dim=2)
        v = torch.cat([past_kv[1].float(), v], dim=2)
    out = attention(q, k, v, D ** -0.5, causal=S > 1)
    out = out.transpose(1, 2).reshape(B, S, Hq * D)
    return linear(out, P[prefix + "o_proj.weight"]), (k, v)


def decoder_layer(x: torch.Tensor, P: dict, cfg, position_ids, past_kv=None,
                  interleaved: bool = False, router_bias=None, force_idx=None):
    """CudaTextDecoderLayer.forward for an MoE layer in fp32
    (REF modules/text_decoder.py:51-65).
    Returns dict(out, router_logits, top_idx, top_w, probs, k, v, h_attn)."""
    x = x.float()
    B, S, H = x.shape
    eps = cfg.rms_norm_eps
    a, (k, v) = attention_block(rmsnorm(x, P["input_layernorm.weight"], eps), P, cfg,
                                position_ids, past_kv, interleaved)
    h = x + a
    m_in = rmsnorm(h, P["post_attention_layernorm.weight"], eps)
    mo, logits, idx, w, p = moe(m_in.reshape(-1, H), P["mlp.gate_weight"], P["mlp.gate_up_proj"],
                                P["mlp.down_proj"], cfg.num_experts_per_tok, True, router_bias,
                                force_idx)
    out = h + mo.reshape(B, S, H)
    return dict(out=out, router_logits=logits, top_idx=idx, top_w=w, probs=p, k=k, v=v,
                h_attn=h, moe_in=m_in)


def swiglu_mlp(x: torch.Tensor, P: dict, prefix: str = "mlp.") -> torch.Tensor:
    """CudaSwiGLUMLP.forward in fp32 (REF modules/mlp.py:19-22):
    down(silu(gate(x)) * up(x)); REF kernels/swiglu.py:57-58 for the product."""
    x = x.float()
    g = linear(x, P[prefix + "gate_proj.weight"], P.get(prefix + "gate_proj.bias"))
    u = linear(x, P[prefix + "up_proj.weight"], P.get(prefix + "up_proj.bias"))
    return linear(F.silu(g) * u, P[prefix + "down_proj.weight"], P.get(prefix + "down_proj.bias"))


def dense_decoder_layer(x: torch.Tensor, P: dict, cfg, position_ids, past_kv=None,
                        interleaved: bool = False):
    """CudaTextDecoderLayer.forward for a dense (non-MoE) layer in fp32
    (REF modules/text_decoder.py:51-65 with the MLP branch)."""
    x = x.float()
    eps = cfg.rms_norm_eps
    a, (k, v) = attention_block(rmsnorm(x, P["input_layernorm.weight"], eps), P, cfg,
                                position_ids, past_kv, interleaved)
    h = x + a
    out = h + swiglu_mlp(rmsnorm(h, P["post_attention_layernorm.weight"], eps), P)
    return dict(out=out, k=k, v=v, h_attn=h)


def text_model(input_ids: torch.Tensor, P: dict, cfg, moe_layers, position_ids=None,
               force_idx=None):
    """CudaQwen3VLMoeModel.forward (text only) in fp32 (REF models/moe.py:59-73,
    85-97): embedding lookup (REF modules/embedding.py:26-27), the decoder
    layers, the final RMSNorm and lm_head.  ``moe_layers[i]`` says whether
    layer i is an MoE layer; ``force_idx[j]`` (optional) is the j-th MoE
    layer's top-k choice (see ``moe``).  Returns dict(logits, router_logits)."""
    B, S = input_ids.shape
    x = P["embed_tokens.weight"].float()[input_ids]
    if position_ids is None:
        pos = torch.arange(S).unsqueeze(0).expand(B, S)
        position_ids = torch.stack([pos, pos, pos], dim=0)
    rls = []
    mi = 0
    for i, is_moe in enumerate(moe_layers):
        pre = f"layers.{i}."
        Pl = {k[len(pre):]: v for k, v in P.items() if k.startswith(pre)}
        if is_moe:
            fi = None if force_idx is None else force_idx[mi]
            r = decoder_layer(x, Pl, cfg, position_ids, force_idx=fi)
            rls.append(r["router_logits"])
            mi += 1
        else:
            r = dense_decoder_layer(x, Pl, cfg, position_ids)
        x = r["out"]
    hidden = rmsnorm(x, P["norm.weight"], cfg.rms_norm_eps)
    return dict(logits=linear(hidden, P["lm_head.weight"]), router_logits=rls)


def near_tie_rows(probs: torch.Tensor, k: int, rel: float = 1e-5) -> torch.Tensor:
    """Rows where two neighbours among the sorted top-(k+1) probabilities differ
    by less than rel * the larger one: a logit computed in another summation
    order may legitimately swap them (the set at the k-th/(k+1)-th boundary,
    the order inside the top-k)."""
    vals, _ = canonical_topk(probs, min(k + 1, probs.shape[-1]))
    if vals.shape[-1] < 2:
        return torch.zeros(probs.shape[0], dtype=torch.bool)
    gap = vals[..., :-1] - vals[..., 1:]
    return (gap < rel * vals[..., :-1]).any(dim=-1)


def bf16_half_ulp(v: torch.Tensor) -> torch.Tensor:
    """Half a bf16 ulp at |v|: the rounding error any bf16 output must carry."""
    a = v.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 8)


def error_stats(got: torch.Tensor, ref: torch.Tensor) -> dict:
    """max-abs error, the same after removing the unavoidable bf16 output
    rounding (max(0, |d| - half_ulp(ref))), and the mean relative error
    sum|d| / sum|ref|."""
    g, r = got.float(), ref.float()
    d = (g - r).abs()
    dq = (d - bf16_half_ulp(r)).clamp_min(0.0)
    return {"max_abs": float(d.max()) if d.numel() else 0.0,
            "max_abs_over_bf16": float(dq.max()) if d.numel() else 0.0,
            "mean_rel": float(d.sum() / r.abs().sum().clamp_min(1e-30)),
            "finite": bool(torch.isfinite(g).all())}


def routing_agreement(got_idx: torch.Tensor, ref_idx: torch.Tensor, probs: torch.Tensor) -> dict:
    """Rows whose top-k expert SET differs, and the oracle's relative gap
    between its k-th and (k+1)-th probability on those rows."""
    k = ref_idx.shape[-1]
    g = torch.sort(got_idx.long(), dim=-1).values
    r = torch.sort(ref_idx.long(), dim=-1).values
    diff = (g != r).any(dim=-1)
    vals, _ = canonical_topk(probs, min(k + 1, probs.shape[-1]))
    if vals.shape[-1] > k:
        gap = (vals[..., k - 1] - vals[..., k]) / vals[..., k - 1]
    else:
        gap = torch.zeros(vals.shape[:-1])
    return {"rows": int(diff.numel()), "flipped": int(diff.sum()),
            "max_flipped_gap": float(gap[diff].max()) if bool(diff.any()) else 0.0,
            "flipped_mask": diff}


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("math", "np", "torch", "F")]

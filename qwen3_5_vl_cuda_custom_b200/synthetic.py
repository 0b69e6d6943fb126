"""Seeded synthetic inputs for the five benchmark configurations.

No checkpoint or dataset is involved: weights are random-init with the
layer's architecture and activations are Gaussian, generated on the CPU from
``torch.Generator().manual_seed(seed)`` in a fixed order so the GPU run, the
CPU oracle and the reference arm all see the same numbers:

  1. parameters in the decoder layer's ``named_parameters()`` order
     (input_layernorm, q/k/v/o_proj, q_norm, k_norm, post_attention_layernorm,
     gate_weight, gate_up_proj, down_proj), each ``normal_(0, 0.02)`` in fp32;
     with ``norm_mode="unit"`` the four RMSNorm weights are ``1 + N(0, 0.02)``
     instead (otherwise attention is close to uniform);
  2. the activations.
Every weight except the fp32 router gate is rounded to bf16 (the GPU dtype);
the values returned are the fp32 upcasts of those bf16 numbers.
"""
from __future__ import annotations

import torch

from .configs import MoETextConfig

NORM_KEYS = ("input_layernorm.weight", "self_attn.q_norm.weight", "self_attn.k_norm.weight",
             "post_attention_layernorm.weight")


def layer_param_shapes(cfg: MoETextConfig) -> list[tuple[str, tuple[int, ...]]]:
    H, D = cfg.hidden_size, cfg.head_dim
    Hq, Hkv = cfg.num_heads, cfg.num_kv_heads
    E, I = cfg.num_experts, cfg.moe_intermediate_size
    return [
        ("input_layernorm.weight", (H,)),
        ("self_attn.q_proj.weight", (Hq * D, H)),
        ("self_attn.k_proj.weight", (Hkv * D, H)),
        ("self_attn.v_proj.weight", (Hkv * D, H)),
        ("self_attn.o_proj.weight", (H, Hq * D)),
        ("self_attn.q_norm.weight", (D,)),
        ("self_attn.k_norm.weight", (D,)),
        ("post_attention_layernorm.weight", (H,)),
        ("mlp.gate_weight", (E, H)),
        ("mlp.gate_up_proj", (E, 2 * I, H)),
        ("mlp.down_proj", (E, H, I)),
    ]


def layer_params(cfg: MoETextConfig, gen: torch.Generator, norm_mode: str = "unit",
                 round_bf16: bool = True) -> dict[str, torch.Tensor]:
    """fp32 CPU state dict of one MoE decoder layer drawn from ``gen``."""
    out: dict[str, torch.Tensor] = {}
    for name, shape in layer_param_shapes(cfg):
        t = torch.empty(shape, dtype=torch.float32).normal_(0.0, 0.02, generator=gen)
        if name in NORM_KEYS and norm_mode == "unit":
            t += 1.0
        if round_bf16 and name != "mlp.gate_weight":
            t = t.to(torch.bfloat16).float()
        out[name] = t
    return out


def hidden_states(shape: tuple[int, ...], gen: torch.Generator, std: float = 1.0,
                  round_bf16: bool = True) -> torch.Tensor:
    x = torch.empty(shape, dtype=torch.float32).normal_(0.0, std, generator=gen)
    return x.to(torch.bfloat16).float() if round_bf16 else x


def text_positions(B: int, S: int, start: int = 0) -> torch.Tensor:
    """(3, B, S) int64 positions with t = h = w = start + i."""
    pos = torch.arange(start, start + S, dtype=torch.int64).unsqueeze(0).expand(B, S)
    return torch.stack([pos, pos, pos], dim=0).contiguous()


def multimodal_positions(B: int, S: int, img_off: int = 64, grid: int = 16) -> torch.Tensor:
    """Config-5 positions: grid*grid image tokens at ``img_off`` with t = start,
    h = start + row, w = start + col; text after the image resumes at
    start + grid on all three axes."""
    n_img = max(0, min(grid * grid, S - img_off))
    t = torch.arange(S, dtype=torch.int64)
    h = t.clone()
    w = t.clone()
    j = torch.arange(n_img, dtype=torch.int64)
    t[img_off:img_off + n_img] = img_off
    h[img_off:img_off + n_img] = img_off + j // grid
    w[img_off:img_off + n_img] = img_off + j % grid
    after = torch.arange(img_off + n_img, S, dtype=torch.int64)
    resume = img_off + grid + (after - (img_off + n_img))
    for a in (t, h, w):
        a[img_off + n_img:] = resume
    pos = torch.stack([t, h, w], dim=0)  # (3, S)
    return pos.unsqueeze(1).expand(3, B, S).contiguous()


def multimodal_hidden(B: int, S: int, H: int, gen: torch.Generator, img_off: int = 64,
                      n_img: int = 256) -> torch.Tensor:
    """Config-5 activations: image tokens ~ N(0, 1.5^2), text tokens ~ N(0, 1)."""
    x = torch.empty(B, S, H).normal_(0.0, 1.0, generator=gen)
    x[:, img_off:img_off + n_img] *= 1.5
    return x.to(torch.bfloat16).float()


def zipf_router_bias(E: int, gen: torch.Generator, alpha: float = 1.2) -> torch.Tensor:
    """Config-4 skew: b_e = 0.5 * log(pop_e), pop over a seeded expert permutation
    proportional to rank^-alpha."""
    perm = torch.randperm(E, generator=gen)
    ranks = torch.empty(E)
    ranks[perm] = torch.arange(1, E + 1, dtype=torch.float32)
    pop = ranks.pow(-alpha)
    pop = pop / pop.sum()
    return 0.5 * torch.log(pop)


def layer_flops(cfg: MoETextConfig, T: int, S: int) -> dict[str, float]:
    """Algorithmic FLOPs of one prefill layer (causal attention over S)."""
    H, D, Hq, Hkv = cfg.hidden_size, cfg.head_dim, cfg.num_heads, cfg.num_kv_heads
    I, k = cfg.moe_intermediate_size, cfg.num_experts_per_tok
    B = T // S
    proj = 2.0 * T * H * (Hq + 2 * Hkv) * D + 2.0 * T * Hq * D * H
    attn = B * Hq * 4.0 * D * S * (S + 1) / 2
    experts = T * k * (2.0 * H * 2 * I + 2.0 * I * H)
    return {"proj": proj, "attn": attn, "experts": experts, "total": proj + attn + experts,
            "router": 2.0 * T * H * cfg.num_experts}


def vision_param_shapes(vc) -> list[tuple[str, tuple[int, ...]]]:
    """Parameter names/shapes of CudaVisionTower (the reference's state-dict
    layout, REF models/common.py:25-76), in registration order."""
    C, I, O = vc.hidden_size, vc.intermediate_size, vc.out_hidden_size
    M = C * vc.spatial_merge_size ** 2
    out = [("patch_embed.weight", (C, vc.in_channels, vc.temporal_patch_size, vc.patch_size,
                                   vc.patch_size)),
           ("patch_embed.bias", (C,)),
           ("pos_embed.emb.weight", (vc.num_position_embeddings, C))]
    for i in range(vc.num_layers):
        b = f"blocks.{i}."
        out += [(b + "norm1.weight", (C,)), (b + "norm1.bias", (C,)),
                (b + "attn.qkv.weight", (3 * C, C)), (b + "attn.qkv.bias", (3 * C,)),
                (b + "attn.proj.weight", (C, C)), (b + "attn.proj.bias", (C,)),
                (b + "norm2.weight", (C,)), (b + "norm2.bias", (C,)),
                (b + "mlp.linear_fc1.weight", (I, C)), (b + "mlp.linear_fc1.bias", (I,)),
                (b + "mlp.linear_fc2.weight", (C, I)), (b + "mlp.linear_fc2.bias", (C,))]
    mergers = [("merger.", C)] + [(f"deepstack_mergers.{j}.", M)
                                  for j in range(len(vc.deepstack_layers))]
    for pre, nd in mergers:
        out += [(pre + "norm.weight", (nd,)), (pre + "norm.bias", (nd,)),
                (pre + "linear_fc1.weight", (M, M)), (pre + "linear_fc1.bias", (M,)),
                (pre + "linear_fc2.weight", (O, M)), (pre + "linear_fc2.bias", (O,))]
    return out


def vision_params(vc, gen: torch.Generator) -> dict[str, torch.Tensor]:
    """fp32 CPU state dict of a vision tower drawn from ``gen``: N(0, 0.02)
    everywhere, LayerNorm weights 1 + N(0, 0.02); bf16-rounded (the GPU dtype)."""
    out = {}
    for name, shape in vision_param_shapes(vc):
        t = torch.empty(shape, dtype=torch.float32).normal_(0.0, 0.02, generator=gen)
        if "norm" in name and name.endswith(".weight"):
            t += 1.0
        out[name] = t.to(torch.bfloat16).float()
    return out


def tiny_vision_config():
    """Small vision tower with the real head_dim (72 = 288 / 4): 3 blocks,
    deepstack after blocks 0 and 2, an 8 x 8 position grid."""
    from .configs import VisionConfig
    return VisionConfig(hidden_size=288, num_layers=3, num_heads=4, intermediate_size=512,
                        patch_size=16, temporal_patch_size=2, spatial_merge_size=2,
                        in_channels=3, num_position_embeddings=64, out_hidden_size=256,
                        rope_theta=10000.0, rms_norm_eps=1e-6, deepstack_layers=(0, 2))

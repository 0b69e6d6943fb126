"""Text-stack configuration, with the reference's field names.

Mirrors ``TextConfig`` / ``MoETextConfig`` / ``Qwen3VLConfig`` of
REF cuda_qwen3_vl/configs/config.py:9-115 (``VisionConfig`` drives the vision
tower of ``vision.py``), plus
the five benchmark shapes used by the tests and the bench harness.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


@dataclass
class VisionConfig:
    hidden_size: int = 1152
    num_layers: int = 27
    num_heads: int = 16
    intermediate_size: int = 4304
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    in_channels: int = 3
    num_position_embeddings: int = 2304
    out_hidden_size: int = 3584
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-6
    deepstack_layers: tuple[int, ...] = (8, 16, 24)


@dataclass
class TextConfig:
    hidden_size: int = 4096
    intermediate_size: int = 22016
    num_layers: int = 32
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = 128
    vocab_size: int = 151936
    max_position_embeddings: int = 128000
    rope_theta: float = 500000.0
    rms_norm_eps: float = 1e-6
    mrope_section: list[int] = field(default_factory=lambda: [24, 20, 20])
    attention_bias: bool = False
    tie_word_embeddings: bool = False


@dataclass
class MoETextConfig(TextConfig):
    num_experts: int = 60
    num_experts_per_tok: int = 4
    moe_intermediate_size: int = 1408
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: list[int] = field(default_factory=list)


@dataclass
class Qwen3VLConfig:
    family: str
    vision: VisionConfig
    text: TextConfig | MoETextConfig

    @classmethod
    def from_hf_config(cls, hf_config: Any) -> "Qwen3VLConfig":
        """Normalises a HF Qwen3-VL(-MoE) config dict/object (same rules as
        REF configs/config.py:58-115)."""
        raw = hf_config.to_dict() if hasattr(hf_config, "to_dict") else dict(hf_config)
        text_raw = raw.get("text_config", raw)
        n_exp = int(text_raw.get("num_local_experts") or text_raw.get("num_experts") or 0)
        is_moe = raw.get("model_type") == "qwen3_vl_moe" or n_exp > 0
        hidden = int(text_raw.get("hidden_size", 4096))
        heads = int(text_raw.get("num_attention_heads", 32))
        common = dict(
            hidden_size=hidden,
            intermediate_size=int(text_raw.get("intermediate_size", 22016)),
            num_layers=int(text_raw.get("num_hidden_layers", 32)),
            num_heads=heads,
            num_kv_heads=int(text_raw.get("num_key_value_heads", 8)),
            head_dim=int(text_raw.get("head_dim") or hidden // heads),
            vocab_size=int(text_raw.get("vocab_size", 151936)),
            max_position_embeddings=int(text_raw.get("max_position_embeddings", 128000)),
            rope_theta=float(text_raw.get("rope_theta", 500000.0)),
            rms_norm_eps=float(text_raw.get("rms_norm_eps", 1e-6)),
            mrope_section=list((text_raw.get("rope_scaling") or {}).get("mrope_section", [24, 20, 20])),
            attention_bias=bool(text_raw.get("attention_bias", False)),
            tie_word_embeddings=bool(raw.get("tie_word_embeddings", False)),
        )
        if is_moe:
            text: TextConfig = MoETextConfig(
                **common,
                num_experts=n_exp or 60,
                num_experts_per_tok=int(text_raw.get("num_experts_per_tok", 4)),
                moe_intermediate_size=int(text_raw.get("moe_intermediate_size", 1408)),
                norm_topk_prob=bool(text_raw.get("norm_topk_prob", True)),
                decoder_sparse_step=int(text_raw.get("decoder_sparse_step", 1)),
                mlp_only_layers=list(text_raw.get("mlp_only_layers", [])),
            )
        else:
            text = TextConfig(**common)
        return cls(family="moe" if is_moe else "dense", vision=VisionConfig(), text=text)


# ------------------------------------------------------------------ presets
def tiny_moe_text(num_layers: int = 1) -> MoETextConfig:
    """Config 1: hidden 256, 8/2 heads of 32, 16 experts top-4, intermediate 128."""
    return MoETextConfig(hidden_size=256, intermediate_size=512, num_layers=num_layers,
                         num_heads=8, num_kv_heads=2, head_dim=32, vocab_size=1024,
                         rope_theta=5e6, mrope_section=[8, 4, 4], num_experts=16,
                         num_experts_per_tok=4, moe_intermediate_size=128)


def a3b_moe_text(num_layers: int = 48) -> MoETextConfig:
    """Qwen3-VL-30B-A3B text shape: hidden 2048, 32/4 heads of 128, 128 experts
    top-8, moe intermediate 768, mRoPE [24,20,20], theta 5e6."""
    return MoETextConfig(hidden_size=2048, intermediate_size=6144, num_layers=num_layers,
                         num_heads=32, num_kv_heads=4, head_dim=128, vocab_size=151936,
                         rope_theta=5e6, mrope_section=[24, 20, 20], num_experts=128,
                         num_experts_per_tok=8, moe_intermediate_size=768)


def moe_config(text: MoETextConfig) -> Qwen3VLConfig:
    return Qwen3VLConfig(family="moe", vision=VisionConfig(), text=text)

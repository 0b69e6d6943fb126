"""Generates the golden fixtures that pin the CPU oracle to the reference.

Runs the reference package itself (luozoupi/Qwen3_5_VL_CUDA_CUSTOM, its
cuda_qwen3_vl modules on CPU tensors, i.e. the torch branch of every op
wrapper) on seeded config-1 inputs and stores its outputs.  Inputs are not
stored: they are regenerated from the seed by
``qwen3_5_vl_cuda_custom_b200.synthetic`` and a checksum of them is kept so a
generator change is detected.

Needs the reference importable, e.g. a copy installed with
``pip install --no-deps --target baseline/_ref <reference>``; run from the repo
root as ``python tests/golden/make_golden.py``.  The fixtures are committed; the
GPU box never runs this script.
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
os.environ.setdefault("CUDA_QWEN3_VL_AUTO_PRELOAD", "0")

from qwen3_5_vl_cuda_custom_b200 import synthetic as syn  # noqa: E402
from qwen3_5_vl_cuda_custom_b200.configs import tiny_moe_text  # noqa: E402

OUT = Path(__file__).resolve().parent


def checksum(ts) -> float:
    return float(sum(float(t.double().sum()) + float(t.double().abs().sum()) for t in ts))


def ref_layer(cfg):
    from cuda_qwen3_vl.modules import CudaTextDecoderLayer
    return CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                moe_intermediate_size=cfg.moe_intermediate_size)


def layer_case(cfg, seed: int, norm_mode: str, positions_fn, S: int = 128, decode_steps: int = 0):
    from cuda_qwen3_vl.modules import TextMRoPE
    g = torch.Generator().manual_seed(seed)
    P = syn.layer_params(cfg, g, norm_mode=norm_mode)
    x = syn.hidden_states((1, S, cfg.hidden_size), g)
    pos = positions_fn(1, S)
    layer = ref_layer(cfg)
    layer.load_state_dict(P)
    rot = TextMRoPE(cfg.head_dim, theta=cfg.rope_theta, mrope_section=cfg.mrope_section)
    with torch.no_grad():
        y, rl, (k, v) = layer(x, lambda q, kk: rot.apply(q, kk, pos))
        case = {"seed": seed, "norm_mode": norm_mode, "S": S,
                "input_checksum": checksum([x, pos.float(), *P.values()]),
                "out": y.clone(), "router_logits": rl.clone(), "k": k.clone(), "v": v.clone()}
        if decode_steps:
            xd = syn.hidden_states((1, 1, cfg.hidden_size), g)
            posd = syn.text_positions(1, 1, start=S)
            yd, rld, (kd, vd) = layer(xd, lambda q, kk: rot.apply(q, kk, posd), past_kv=(k, v))
            case.update({"decode_x_checksum": checksum([xd]), "decode_out": yd.clone(),
                         "decode_router_logits": rld.clone(), "decode_k_len": kd.shape[2]})
    return case


def moe_module_case(seed: int = 5):
    """The reference module test's tiny MoE shape (REF tests/test_modules.py:132-145)."""
    from cuda_qwen3_vl.modules import CudaSparseMoE
    g = torch.Generator().manual_seed(seed)
    m = CudaSparseMoE(64, 32, 4, 2)
    P = {n: torch.empty_like(p).normal_(0, 0.02, generator=g) for n, p in m.named_parameters()}
    m.load_state_dict(P)
    x = torch.empty(2, 8, 64).normal_(0, 1, generator=g)
    with torch.no_grad():
        out, logits = m(x)
    return {"seed": seed, "input_checksum": checksum([x, *P.values()]), "out": out,
            "router_logits": logits}


VISION_GRID = [[1, 8, 8], [2, 4, 4]]


def vision_case(seed: int = 11) -> dict:
    """The reference's CudaVisionTower (REF models/common.py:25-210) in fp32 on a
    small config with the real head_dim 72, two images (one of two frames)."""
    from cuda_qwen3_vl.configs import VisionConfig as RefVisionConfig
    from cuda_qwen3_vl.models.common import CudaVisionTower
    vc = syn.tiny_vision_config()
    g = torch.Generator().manual_seed(seed)
    P = syn.vision_params(vc, g)
    grid = torch.tensor(VISION_GRID)
    n = int(sum(t * h * w for t, h, w in VISION_GRID))
    feat = vc.in_channels * vc.temporal_patch_size * vc.patch_size ** 2
    x = syn.hidden_states((n, feat), g)
    ref_cfg = RefVisionConfig(**{k: getattr(vc, k) for k in vc.__dataclass_fields__})
    tower = CudaVisionTower(ref_cfg)
    tower.load_state_dict(P)
    with torch.no_grad():
        pooled, last, deep = tower(x, grid)
    return {"seed": seed, "grid_thw": VISION_GRID,
            "input_checksum": checksum([x, *P.values()]),
            "pooler_output": pooled.clone(), "last_hidden_state": last.clone(),
            "deepstack": [d.clone() for d in deep]}


def main_vision() -> None:
    torch.save(vision_case(), OUT / "vision_reference.pt")
    print("wrote", OUT / "vision_reference.pt")


def main() -> None:
    cfg = tiny_moe_text()
    cases = {
        "c1_unit": layer_case(cfg, 0, "unit", syn.text_positions, decode_steps=1),
        "c1_literal": layer_case(cfg, 0, "literal", syn.text_positions),
        "c1_multimodal": layer_case(cfg, 7, "unit",
                                    lambda B, S: syn.multimodal_positions(B, S, img_off=16, grid=8)),
        "moe_tiny": moe_module_case(),
    }
    torch.save(cases, OUT / "c1_reference.pt")
    print("wrote", OUT / "c1_reference.pt")
    main_vision()


if __name__ == "__main__":
    main_vision() if "--vision-only" in sys.argv else main()

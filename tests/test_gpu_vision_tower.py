"""The vision tower (qwen3_5_vl_cuda_custom_b200.vision) on the GPU against the
reference's own CudaVisionTower outputs (REF models/common.py:25-210, run in
fp32 on CPU by tests/golden/make_golden.py): a 3-block tower with the real
head_dim 72 (padded to 128 for the tcgen05 attention), two images, deepstack
after blocks 0 and 2.  bf16 outputs against the fp32 reference: max-abs beyond
bf16 rounding <= 4e-2 and mean relative error <= 1e-2, twice the decoder
layer's bounds: the residual stream between the three blocks is bf16, as in the
reference's own bf16 path (REF modules/vision_block.py:22-23 adds residuals in
the model dtype), and the mergers round fc1 and GELU outputs to bf16, so the
roundings of the stacked blocks accumulate (measured: last hidden state 2.9e-2 /
3.9e-3, merged output 5.5e-3 / 5.9e-3 at |out| ~ 0.2)."""
from pathlib import Path

import pytest
import torch

from oracle import layer_oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden" / "vision_reference.pt"


MAX_ABS_TOWER = 4e-2
MEAN_REL = 1e-2


def check(got, ref, what):
    s = O.error_stats(got.float().cpu(), ref)
    print(what, s)
    assert s["finite"], what
    assert s["max_abs_over_bf16"] <= MAX_ABS_TOWER and s["mean_rel"] <= MEAN_REL, (what, s)


def test_vision_tower_matches_reference_golden():
    from qwen3_5_vl_cuda_custom_b200 import build, kernels as K, synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.vision import CudaVisionTower
    build.build()
    case = torch.load(GOLDEN, weights_only=False)
    vc = syn.tiny_vision_config()
    g = torch.Generator().manual_seed(case["seed"])
    P = syn.vision_params(vc, g)
    grid = torch.tensor(case["grid_thw"])
    n = int(sum(t * h * w for t, h, w in case["grid_thw"]))
    x = syn.hidden_states((n, vc.in_channels * vc.temporal_patch_size * vc.patch_size ** 2), g)
    tower = CudaVisionTower(vc)
    tower.load_state_dict(P)
    tower = tower.to("cuda", torch.bfloat16)
    with torch.no_grad():
        pooled, last, deep = tower(x.to("cuda", torch.bfloat16), grid)
    K.device_error_check()
    check(last, case["last_hidden_state"], "last_hidden_state")
    check(pooled, case["pooler_output"], "pooler_output")
    assert len(deep) == len(case["deepstack"]) == 2
    for i, (d, r) in enumerate(zip(deep, case["deepstack"])):
        check(d, r, f"deepstack {i}")


def test_model_scatters_vision_features_into_image_tokens():
    """CudaQwen3VLMoeModel with pixel_values: the image tokens' embeddings are
    replaced by the tower's merged features (REF models/moe.py:86-90)."""
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import MoETextConfig, Qwen3VLConfig
    from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel
    vc = syn.tiny_vision_config()
    t = MoETextConfig(hidden_size=256, intermediate_size=512, num_layers=1, num_heads=8,
                      num_kv_heads=2, head_dim=32, vocab_size=512, rope_theta=5e6,
                      mrope_section=[8, 4, 4], num_experts=16, num_experts_per_tok=4,
                      moe_intermediate_size=128)
    torch.manual_seed(0)
    model = CudaQwen3VLMoeModel(Qwen3VLConfig(family="moe", vision=vc, text=t))
    model.visual.load_state_dict(syn.vision_params(vc, torch.Generator().manual_seed(2)))
    model = model.to("cuda", torch.bfloat16)
    grid = torch.tensor([[1, 8, 8]])
    px = torch.randn(64, 1536, generator=torch.Generator().manual_seed(3)).cuda().bfloat16()
    ids = torch.randint(0, 512, (1, 40), generator=torch.Generator().manual_seed(4)).cuda()
    mask = torch.zeros(1, 40, dtype=torch.bool, device="cuda")
    mask[0, 10:26] = True  # 16 merged image tokens
    with torch.no_grad():
        logits, _ = model(ids, pixel_values=px, vision_position_ids=grid, image_token_mask=mask)
        feats = model.visual(px, grid)[0]
        emb = model.embed_tokens(ids).clone()
        emb[mask] = feats
        ref_logits, _ = model(inputs_embeds=emb)
    assert torch.equal(logits, ref_logits)

"""Model-level and remaining-module parity on the GPU against the fp32 CPU
oracle: the text model's logits (embedding, MoE and dense layers, final norm,
lm_head; REF models/moe.py:59-97), the dense SwiGLU MLP (REF
modules/mlp.py:19-22), and a decode step through the preallocated KV cache
(REF modules/attention.py:79-95 semantics) -- each compared with the oracle
directly, not with another path of this library."""
import pytest
import torch

from oracle import layer_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda"
MAX_ABS = 2e-2
MEAN_REL = 5e-3


@pytest.fixture(scope="module", autouse=True)
def _ready():
    from qwen3_5_vl_cuda_custom_b200 import build
    build.build()
    yield
    from qwen3_5_vl_cuda_custom_b200 import kernels as K
    K.device_error_check()


def check(got, ref, what):
    s = O.error_stats(got.float().cpu(), ref)
    assert s["finite"], what
    assert s["max_abs_over_bf16"] <= MAX_ABS and s["mean_rel"] <= MEAN_REL, (what, s)
    return s


def _cpu_state(module) -> dict:
    return {k: v.detach().float().cpu() for k, v in module.state_dict().items()}


def test_text_model_logits_match_oracle_stack():
    """Two layers (layer 0 MoE, layer 1 dense via mlp_only_layers), vocab 512:
    the GPU model's logits vs the oracle stack re-run with the GPU's expert
    choice (recovered from the returned router logits)."""
    from qwen3_5_vl_cuda_custom_b200.configs import MoETextConfig, moe_config
    from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel, _layer_uses_moe
    t = MoETextConfig(hidden_size=256, intermediate_size=512, num_layers=2, num_heads=8,
                      num_kv_heads=2, head_dim=32, vocab_size=512, rope_theta=5e6,
                      mrope_section=[8, 4, 4], num_experts=16, num_experts_per_tok=4,
                      moe_intermediate_size=128, mlp_only_layers=[1])
    torch.manual_seed(3)
    model = CudaQwen3VLMoeModel(moe_config(t), vision=False).to(DEV, torch.bfloat16)
    moe_layers = [_layer_uses_moe(t, i) for i in range(t.num_layers)]
    assert moe_layers == [True, False]
    ids = torch.randint(0, t.vocab_size, (2, 96), generator=torch.Generator().manual_seed(4))
    with torch.no_grad():
        logits, rls = model(ids.to(DEV))
    P = _cpu_state(model)
    assert P["layers.0.mlp.gate_weight"].dtype == torch.float32
    force = []
    for rl in rls:
        p = torch.softmax(rl.float().cpu(), dim=-1)
        force.append(O.canonical_topk(p, t.num_experts_per_tok)[1])
    ref = O.text_model(ids, P, t, moe_layers, force_idx=force)
    assert len(ref["router_logits"]) == len(rls) == 1
    assert (rls[0].cpu() - ref["router_logits"][0]).abs().max() < 5e-3
    check(logits, ref["logits"], "model logits")


def test_swiglu_mlp_matches_oracle():
    from qwen3_5_vl_cuda_custom_b200.modules import CudaSwiGLUMLP
    torch.manual_seed(5)
    mlp = CudaSwiGLUMLP(512, 1024).to(DEV, torch.bfloat16)
    x = torch.randn(3, 77, 512, generator=torch.Generator().manual_seed(6)).bfloat16()
    with torch.no_grad():
        y = mlp(x.to(DEV))
    check(y, O.swiglu_mlp(x.float(), _cpu_state(mlp), prefix=""), "SwiGLU MLP")


def test_c3_decode_through_layer_kv_cache_matches_oracle():
    """Config-3 decode (64 sequences x 1 token over 8192 cached positions)
    through a preallocated LayerKVCache, against the oracle's decoder layer
    with the same past (a subset of the sequences: a token's math does not
    depend on other sequences)."""
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import a3b_moe_text
    from qwen3_5_vl_cuda_custom_b200.kv_cache import LayerKVCache
    from qwen3_5_vl_cuda_custom_b200.modules import CudaTextDecoderLayer, TextMRoPE
    cfg = a3b_moe_text(1)
    g = torch.Generator().manual_seed(2)
    P = syn.layer_params(cfg, g)
    B, L = 64, 8192
    x = syn.hidden_states((B, 1, cfg.hidden_size), g)
    layer = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                 num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                 moe_intermediate_size=cfg.moe_intermediate_size)
    layer.load_state_dict(P)
    layer = layer.to(DEV, torch.bfloat16)
    rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).to(DEV)
    cache = LayerKVCache(B, cfg.num_kv_heads, L + 4, cfg.head_dim, DEV)
    gk = torch.Generator(device=DEV).manual_seed(2)
    cache.k[:, :, :L].normal_(generator=gk)
    cache.v[:, :, :L].normal_(generator=gk)
    cache.length = L
    pos = syn.text_positions(B, 1, start=L)
    with torch.no_grad():
        y, _, kv = layer(x.to(DEV, torch.bfloat16), rot.bind(pos.to(DEV)), past_kv=cache)
    assert kv is cache and cache.length == L + 1
    sub = [0, 31, 63]
    past = (cache.k[sub, :, :L].float().cpu(), cache.v[sub, :, :L].float().cpu())
    ref = O.decoder_layer(x[sub], P, cfg, pos[:, sub], past_kv=past)
    check(y[sub], ref["out"], "decode through the KV cache")
    check(cache.k[sub, :, L:L + 1], ref["k"][:, :, L:], "appended k")
    check(cache.v[sub, :, L:L + 1], ref["v"][:, :, L:], "appended v")


def test_graphed_layer_with_kv_cache_keeps_length():
    """GraphedDecoderLayer over a LayerKVCache: construction leaves the cache
    length where it was, and a replay equals the eager step at that length."""
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import tiny_moe_text
    from qwen3_5_vl_cuda_custom_b200.graphs import GraphedDecoderLayer
    from qwen3_5_vl_cuda_custom_b200.kv_cache import LayerKVCache
    from qwen3_5_vl_cuda_custom_b200.modules import CudaTextDecoderLayer, TextMRoPE
    cfg = tiny_moe_text()
    g = torch.Generator().manual_seed(8)
    P = syn.layer_params(cfg, g)
    layer = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                 num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                 moe_intermediate_size=cfg.moe_intermediate_size)
    layer.load_state_dict(P)
    layer = layer.to(DEV, torch.bfloat16)
    rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).to(DEV)
    B, past = 4, 100
    cache = LayerKVCache(B, cfg.num_kv_heads, past + 8, cfg.head_dim, DEV)
    cache.k[:, :, :past].normal_()
    cache.v[:, :, :past].normal_()
    cache.length = past
    x = syn.hidden_states((B, 1, cfg.hidden_size), g).to(DEV, torch.bfloat16)
    pos = syn.text_positions(B, 1, start=past).to(DEV)
    gl = GraphedDecoderLayer(layer, rot, x, pos, past_kv=cache)
    assert cache.length == past
    got = gl(x)[0].clone()
    with torch.no_grad():
        ref, _, _ = layer(x, rot.bind(pos), past_kv=cache)
    assert torch.equal(got, ref)

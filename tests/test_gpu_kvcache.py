"""Preallocated KV cache (in-place append, attention over the cache buffers)
against the reference API's ``past_kv = (k, v)`` concatenation path: the same
kernels run with a per-head row stride of the cache capacity instead of the
sequence length, so the results must be identical."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _ready():
    from qwen3_5_vl_cuda_custom_b200 import build
    build.build()
    yield
    from qwen3_5_vl_cuda_custom_b200 import kernels as K
    K.device_error_check()


def K():
    from qwen3_5_vl_cuda_custom_b200 import kernels
    return kernels


@pytest.mark.parametrize("B,Hq,Hkv,D,past,Sq,cap", [
    (2, 32, 4, 128, 300, 200, 1024),   # tcgen05 prefill over a cache
    (1, 8, 2, 64, 0, 130, 256),        # mma.sync prefill, empty history
    (4, 32, 4, 128, 777, 1, 1000),     # split-KV decode
    (3, 8, 2, 32, 90, 1, 97),          # decode, D = 32
])
def test_attention_over_cache_matches_concat(B, Hq, Hkv, D, past, Sq, cap):
    g = torch.Generator().manual_seed(B * 1000 + past + Sq)
    bf = torch.bfloat16
    k_past = torch.randn(B, Hkv, past, D, generator=g).to(bf).to(DEV)
    v_past = torch.randn(B, Hkv, past, D, generator=g).to(bf).to(DEV)
    q = torch.randn(B, Hq, Sq, D, generator=g).to(bf).to(DEV)
    k_new = torch.randn(B, Hkv, Sq, D, generator=g).to(bf).to(DEV)
    v_new = torch.randn(B, Hkv, Sq, D, generator=g).to(bf).to(DEV)
    kc = torch.zeros(B, Hkv, cap, D, dtype=bf, device=DEV)
    vc = torch.zeros_like(kc)
    Kk = K()
    Kk.kv_append(k_past, v_past, kc, vc, 0)
    Kk.kv_append(k_new, v_new, kc, vc, past)
    k_all = torch.cat([k_past, k_new], dim=2)
    v_all = torch.cat([v_past, v_new], dim=2)
    assert torch.equal(kc[:, :, :past + Sq], k_all) and torch.equal(vc[:, :, :past + Sq], v_all)
    assert not kc[:, :, past + Sq:].any()
    causal = Sq > 1
    scale = D ** -0.5
    ref = Kk.attention_tokens(q, k_all, v_all, scale, causal)
    got = Kk.attention_cache(q, kc, vc, past + Sq, scale, causal)
    assert torch.equal(got, ref)


def test_kv_append_rejects_overflow():
    Kk = K()
    kc = torch.zeros(1, 2, 8, 32, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(1, 2, 3, 32, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="capacity"):
        Kk.kv_append(k, k, kc, kc.clone(), 6)


def test_decoder_layer_with_cache_matches_tuple_past():
    """Prefill then three decode steps: cache path == concatenation path."""
    from qwen3_5_vl_cuda_custom_b200 import synthetic as syn
    from qwen3_5_vl_cuda_custom_b200.configs import a3b_moe_text
    from qwen3_5_vl_cuda_custom_b200.kv_cache import LayerKVCache
    from qwen3_5_vl_cuda_custom_b200.modules import CudaTextDecoderLayer, TextMRoPE
    cfg = a3b_moe_text(1)
    g = torch.Generator().manual_seed(5)
    layer = CudaTextDecoderLayer(cfg.hidden_size, cfg.num_heads, cfg.num_kv_heads, cfg.head_dim,
                                 cfg.intermediate_size, cfg.rms_norm_eps, use_moe=True,
                                 num_experts=cfg.num_experts, top_k=cfg.num_experts_per_tok,
                                 moe_intermediate_size=cfg.moe_intermediate_size)
    layer.load_state_dict(syn.layer_params(cfg, g))
    layer = layer.to(DEV, torch.bfloat16)
    rot = TextMRoPE(cfg.head_dim, cfg.rope_theta, cfg.mrope_section).to(DEV)
    B, S0, steps = 2, 300, 3
    cache = LayerKVCache(B, cfg.num_kv_heads, S0 + steps + 5, cfg.head_dim, DEV)
    past = None
    with torch.no_grad():
        for i in range(1 + steps):
            S = S0 if i == 0 else 1
            start = 0 if i == 0 else S0 + i - 1
            x = syn.hidden_states((B, S, cfg.hidden_size), g).to(DEV, torch.bfloat16)
            pos = torch.arange(start, start + S, device=DEV).expand(B, S)
            bound = rot.bind(torch.stack([pos, pos, pos]))
            ref, ref_rl, past = layer(x, bound, past_kv=past)
            got, got_rl, ret = layer(x, bound, past_kv=cache)
            assert ret is cache and cache.length == start + S
            assert torch.equal(got, ref) and torch.equal(got_rl, ref_rl)
            k_view, v_view = cache
            assert torch.equal(k_view, past[0]) and torch.equal(v_view, past[1])


def test_model_generate_matches_tuple_past_loop():
    """Greedy generate with a KVCache == the same greedy loop on (k, v) tuples."""
    from qwen3_5_vl_cuda_custom_b200.configs import MoETextConfig, moe_config
    from qwen3_5_vl_cuda_custom_b200.models import CudaQwen3VLMoeModel
    t = MoETextConfig(hidden_size=256, intermediate_size=512, num_layers=2, num_heads=4,
                      num_kv_heads=2, head_dim=64, vocab_size=512, rope_theta=1e4,
                      mrope_section=[16, 8, 8], num_experts=32, num_experts_per_tok=2,
                      moe_intermediate_size=64)
    torch.manual_seed(0)
    model = CudaQwen3VLMoeModel(moe_config(t), vision=False).to(DEV, torch.bfloat16)
    ids = torch.randint(0, 512, (2, 12), device=DEV)
    with torch.no_grad():
        out = model.generate(ids, max_new_tokens=5)
        logits, _, kvs = model(ids, return_kv=True)
        seq = [ids]
        nxt = logits[:, -1].argmax(-1)
        for _ in range(4):
            seq.append(nxt[:, None])
            logits, _, kvs = model(nxt[:, None], past_key_values=kvs, return_kv=True)
            nxt = logits[:, -1].argmax(-1)
        seq.append(nxt[:, None])
        ref = torch.cat(seq, dim=1)
    assert out.shape == (2, 17)
    assert torch.equal(out, ref)

"""Host-side behaviour of the preallocated KV cache (no GPU needed): tuple
compatibility of LayerKVCache and bookkeeping of KVCache."""
import torch

from qwen3_5_vl_cuda_custom_b200.kv_cache import KVCache, LayerKVCache


def test_layer_cache_unpacks_like_the_reference_tuple():
    c = LayerKVCache(2, 4, 16, 8, "cpu")
    assert c.capacity == 16 and c.length == 0 and not c.k.any()
    c.k[:, :, :5] = 1.0
    c.length = 5
    k, v = c
    assert k.shape == (2, 4, 5, 8) and v.shape == (2, 4, 5, 8)
    assert c[0].shape[2] == 5 and bool((c[0] == 1).all())
    assert len(c) == 2
    c.reset()
    assert c.length == 0 and c[0].shape[2] == 0


def test_model_cache_indexing_and_reset():
    cache = KVCache(3, 1, 2, 32, 16, "cpu", dtype=torch.float32)
    assert len(cache) == 3 and cache.length == 0
    for layer in cache:
        layer.length = 7
    assert cache.length == 7 and cache[2].k.dtype == torch.float32
    assert cache[0][0].shape == (1, 2, 7, 16)
    cache.reset()
    assert all(layer.length == 0 for layer in cache)

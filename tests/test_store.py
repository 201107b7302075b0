"""The per-token cache store: the oracle against the reference's torch store path (golden), on CPU."""

import numpy as np

from oracle.kv_oracle import store_kvcache, store_latents


def test_the_oracle_store_matches_the_reference_on_nhd_and_hnd_caches(golden):
    meta, arrays = golden
    slots = arrays["store_slots"]
    key, value = arrays["store_key"], arrays["store_value"]
    for layout in ("NHD", "HND"):
        cache = arrays[f"store_{layout}_before"].copy()
        view = cache if layout == "NHD" else cache.swapaxes(2, 3)  # (2, blocks, block, heads, dim) either way
        store_kvcache(key, value, view[0], view[1], slots)
        assert np.array_equal(cache, arrays[f"store_{layout}_after"]), layout


def test_the_oracle_latent_store_matches_the_reference(golden):
    _, arrays = golden
    cache = arrays["store_latent_before"].copy()
    store_latents(arrays["store_latent"], cache[0], arrays["store_slots"])
    assert np.array_equal(cache, arrays["store_latent_after"])


def test_padding_slots_leave_the_cache_alone(golden):
    _, arrays = golden
    cache = arrays["store_NHD_before"].copy()
    store_kvcache(arrays["store_key"], arrays["store_value"], cache[0], cache[1], np.full(10, -1))
    assert np.array_equal(cache, arrays["store_NHD_before"])


def test_the_kvx_store_refuses_rows_that_would_not_fit_their_slots():
    """kvx_store copies rows as bytes: a dtype, head count or head size that differs from the cache's would write
    past each slot, so the wrappers refuse it before anything reaches the device (these run on CPU tensors)."""
    import pytest
    import torch

    from lean_vllm_b200.attention.kvx_cache import store_kvcache, store_latents

    key = torch.zeros(4, 2, 8, dtype=torch.bfloat16)
    cache = torch.zeros(3, 16, 2, 8, dtype=torch.bfloat16)
    slots = torch.arange(4)
    with pytest.raises(TypeError, match="share a dtype"):
        store_kvcache(key.float(), key.float(), cache, cache, slots)
    with pytest.raises(ValueError, match="2 heads of 8 into a cache of 4 heads of 8"):
        wide = torch.zeros(3, 16, 4, 8, dtype=torch.bfloat16)
        store_kvcache(key, key, wide, wide, slots)
    with pytest.raises(ValueError, match="shapes must match"):
        store_kvcache(key, key[:, :1], cache, cache, slots)
    with pytest.raises(ValueError, match="latents of 8 into a cache"):
        store_latents(key[:, 0], torch.zeros(3, 16, 16, dtype=torch.bfloat16), slots)
    with pytest.raises(TypeError, match="share a dtype"):
        store_latents(key[:, 0].float(), torch.zeros(3, 16, 8, dtype=torch.bfloat16), slots)
